"""Multi-GPU host logic on CPU: world_size-2 `gloo` ranks, no GPU.

Each rank takes its block of rows, balanced on nnz plus SHARD_ROW_WEIGHT per row
(vcsrmc_partition_rows_weighted, the partition `bench.py --gpus N` uses), builds the VCSR-MC
format of that block on its own (the reference builder applied to a row slice), and computes its
rows of C with the fp64 oracle from the format alone. The ranks exchange their results; rank 0
checks that the blocks tile the matrix and that the assembled C equals the single-process
oracle result. This is exactly the data path of `bench.py --gpus N` minus the kernels (which the
GPU tests cover): no collective is needed to compute C.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _format_spmm_fp64(fmt: dict, M: int, B: np.ndarray) -> np.ndarray:
    """C = A*B from the VCSR-MC arrays alone (groups x lanes x depth slots)."""
    C = np.zeros((M, B.shape[1]), dtype=np.float64)
    gp, gd, gs, gr = fmt["group_ptr"], fmt["group_depth"], fmt["group_seg_base"], fmt["group_rows"]
    for g in range(gd.size):
        for lane in range(16):
            row = gr[g * 16 + lane]
            if row < 0:
                continue
            for d in range(gd[g]):
                s = gp[g] + d * 16 + lane
                lc = fmt["lcol"][s]
                if lc >= 0:
                    C[row] += np.float64(fmt["val"][s]) * B[gs[g] + lc].astype(np.float64)
    return C


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch
    import torch.distributed as dist
    import vcsr_mc_b200 as vm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 11, seed=7)  # same matrix on every rank (seeded)
        rp, col, val = A.arrays()
        B = vm.gen_dense_host(A.N, 8, seed=7)
        w = vm.SHARD_ROW_WEIGHT  # the partition the benchmark's GPU ranks use
        cuts = vm.partition_rows(rp, world, row_weight=w)
        r0, r1 = int(cuts[rank]), int(cuts[rank + 1])
        shard = A.row_slice(r0, r1)
        fmt = vm.csr_to_vcsr_mc(shard, fp32=True, segw=32).arrays()
        C_local = _format_spmm_fp64(fmt, r1 - r0, B)
        # exchange (row range, result) through the process group
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([r1 - r0], dtype=torch.int64))
        maxrows = int(max(s.item() for s in sizes))
        buf = torch.zeros((maxrows, 8), dtype=torch.float64)
        buf[: r1 - r0] = torch.from_numpy(C_local)
        gathered = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(gathered, buf)
        cuts_all = [torch.zeros(world + 1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(cuts_all, torch.from_numpy(cuts.astype(np.int64)))
        if rank == 0:
            from oracle import bind as ob
            for c in cuts_all:
                assert np.array_equal(c.numpy(), cuts_all[0].numpy()), "ranks disagree on the partition"
            C = np.concatenate([gathered[k][: int(sizes[k].item())].numpy() for k in range(world)])
            ref = ob.spmm_fp64(rp, col, val, B)
            assert C.shape == ref.shape
            assert np.allclose(C, ref, rtol=1e-12, atol=1e-12)
            # balance: each block costs about (nnz + w * rows) / world; a row is never split, so blocks
            # differ by at most one row's cost
            cost = [float(rp[cuts[k + 1]] - rp[cuts[k]]) + w * float(cuts[k + 1] - cuts[k]) for k in range(world)]
            assert max(cost) - min(cost) <= float(np.max(np.diff(rp))) + w + 1
            assert cuts[0] == 0 and cuts[-1] == A.M and np.all(np.diff(cuts) >= 0)
            open(os.path.join(out_dir, "ok"), "w").close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_row_sharding_gloo(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
        assert p.exitcode == 0, p.exitcode
    assert (tmp_path / "ok").exists()
