#!/usr/bin/env python
"""VCSR-MC SpMM benchmark (one JSON line on rank 0).

Default workload: BASELINE config 4, the one the 1/2/4/8-GPU metric and the north_star roofline
target are quoted on: R-MAT A with 2^24 rows/cols (2^28 samples, (a,b,c) = (.57,.19,.19),
duplicates removed, ~261M nnz, values U(-1,1)), B 2^24 x 128 fp16 U(-1,1), C fp32, FP16 path
(tcgen05), segw 32, tileK 128. Synthetic, seeded inputs (seed 0) stand in for the dataset.

A step = C = A*B over the whole matrix: zero C, then one VCSR-MC SpMM launch (C += A*B, the
reference's contract). With --gpus P (torchrun, one rank per GPU) A is cut into P nnz-balanced
row blocks, B is replicated, each rank owns its rows of C; there is no collective on the data
path (strong scaling: the total work is fixed). Time = max over ranks of the device time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload rmat|c1|c2|c3] [--dtype fp16|fp32]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
_RESULT_FD = 1


def emit(obj: dict) -> None:
    """Writes the single JSON result line to the original stdout."""
    os.write(_RESULT_FD, (json.dumps(obj) + "\n").encode())
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

O_COLS = 128
L2_BYTES = 126 * (1 << 20)
SEED = 0
# Generated CSRs are cached inside the checkout (a git-ignored folder) so that every rank of a
# multi-GPU run, and later runs, load the same matrix instead of generating it again.
CACHE_DIR = os.environ.get("VCSRMC_BENCH_CACHE", os.path.join(ROOT, ".bench_cache"))


def log(msg: str) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(f"[bench] {msg}", file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------------------------
def workload_spec(name: str, scale: int) -> dict:
    import vcsr_mc_b200 as vm
    if name == "rmat":
        return {"kind": vm.GEN_RMAT, "param": scale,
                "desc": f"config4 R-MAT 2^{scale} rows, 2^{scale + 4} samples (a,b,c)=(0.57,0.19,0.19), dedup"}
    if name == "c1":
        return {"kind": vm.GEN_UNIFORM_POISSON, "param": 4096, "desc": "config1 4096^2 Poisson(16)"}
    if name == "c2":
        return {"kind": vm.GEN_ZIPF, "param": 262144, "desc": "config2 262144^2 Zipf(1.8) mean 10 cap 8192"}
    if name == "c3":
        return {"kind": vm.GEN_STENCIL27, "param": 100, "desc": "config3 27-point stencil 100^3"}
    if name == "c3links":
        return {"kind": vm.GEN_STENCIL27_LINKS, "param": 100,
                "desc": "27-point stencil 100^3 plus 3 random long-range links per row (not a BASELINE config)"}
    raise SystemExit(f"unknown workload {name}")


def load_or_generate_csr(spec: dict, rank: int, world: int, dist_barrier) -> tuple:
    """Rank 0 generates the CSR (all host threads) into a shared-memory cache; all ranks load it."""
    import vcsr_mc_b200 as vm
    key = f"k{spec['kind']}_p{spec['param']}_s{SEED}"
    d = os.path.join(CACHE_DIR, key)
    done = os.path.join(d, "done")
    if rank == 0 and not os.path.exists(done):
        t = time.time()
        A = vm.CSR.generate(spec["kind"], spec["param"], seed=SEED)
        rp, col, val = A.arrays(copy=False)
        try:
            os.makedirs(d, exist_ok=True)
            np.save(os.path.join(d, "row_ptr.npy"), rp)
            np.save(os.path.join(d, "col.npy"), col)
            np.save(os.path.join(d, "val.npy"), val)
            with open(os.path.join(d, "meta.json"), "w") as f:
                json.dump({"M": A.M, "N": A.N, "nnz": A.nnz}, f)
            open(done, "w").close()
            cached = True
        except OSError:
            cached = False
        log(f"generated {spec['desc']}: nnz={A.nnz} in {time.time() - t:.1f}s (cached={cached})")
        if world == 1 or not cached:
            if world > 1:
                raise SystemExit("multi-rank runs need the shared CSR cache")
            return A.M, A.N, np.array(rp), np.array(col), np.array(val)
    dist_barrier()
    with open(os.path.join(d, "meta.json")) as f:
        meta = json.load(f)
    rp = np.load(os.path.join(d, "row_ptr.npy"), mmap_mode="r")
    col = np.load(os.path.join(d, "col.npy"), mmap_mode="r")
    val = np.load(os.path.join(d, "val.npy"), mmap_mode="r")
    return meta["M"], meta["N"], rp, col, val


def algorithmic_bytes(nnz: int, M: int, D: int, O: int, s_ab: int) -> int:
    """Compulsory bytes of one SpMM: A (col int32 + value), row_ptr, the D distinct rows of B
    that A touches, and C (fp32) written once."""
    return nnz * (4 + s_ab) + (M + 1) * 4 + D * O * s_ab + M * O * 4


# ---------------------------------------------------------------------------------------------
# clocks (sampled with nvidia-smi during the timed region)
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, window=None) -> dict:
        """Summary of the samples taken in window = (t0, t1) (wall-clock seconds around the timed
        region), or of all samples when none fall inside it."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0,
                    "timed_region_only": False}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        return summarize_clock_samples(self.lines, window)


CLOCK_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


def summarize_clock_samples(lines, window=None) -> dict:
    """lines: (arrival time, one nvidia-smi csv line of ClockSampler.QUERY). A line arrives after it
    was taken, so the window is widened by 0.1 s (two sampling intervals) at its end."""
    def parse(sel):
        sm, smax, reasons = [], [], set()
        for _, ln in sel:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(CLOCK_REASONS, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return sm, smax, reasons

    in_window = window is not None
    sm, smax, reasons = parse([x for x in lines if window[0] <= x[0] <= window[1] + 0.1] if in_window else lines)
    if in_window and not sm:  # a timed region shorter than one interval: every sample
        in_window = False
        sm, smax, reasons = parse(lines)
    return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons), "samples": len(sm), "timed_region_only": in_window}


# ---------------------------------------------------------------------------------------------
# CPU baselines (the reference's own fp64 CSR loop, src/main.cpp:202-207, from oracle/_ref)
# ---------------------------------------------------------------------------------------------
def mem_available_bytes() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except (OSError, ValueError, IndexError):
        pass
    return 0


def cpu_sample(M, N, rp, col, val, target_nnz: int, fp16_b: bool):
    """Every k-th row of A (k chosen for ~target_nnz), with the full N x O fp32 B holding the GPU
    run's values (rounded to fp16 on the FP16 path), so that the CPU gathers B rows over the same
    address span as the whole job. Only when host memory cannot hold four copies of B are the
    columns compacted to the rows of B the sample touches. Returns (row_ptr, col, val, B,
    description, nnz)."""
    nnz = int(rp[M])
    k = max(1, int(round(nnz / max(1, target_nnz))))
    rows = np.arange(0, M, k, dtype=np.int64)
    starts, ends = np.asarray(rp[rows], dtype=np.int64), np.asarray(rp[rows + 1], dtype=np.int64)
    lens = ends - starts
    srp = np.zeros(rows.size + 1, dtype=np.int64)
    np.cumsum(lens, out=srp[1:])
    idx = np.repeat(starts - srp[:-1], lens) + np.arange(srp[-1])
    scol = np.asarray(col)[idx]
    sval = np.asarray(val)[idx].astype(np.float32)
    full_bytes = N * O_COLS * 4
    if mem_available_bytes() > 4 * full_bytes:
        import vcsr_mc_b200 as vm
        Bs = vm.gen_dense_host(N, O_COLS, SEED)  # the same stream as the GPU's B
        if fp16_b:
            for s in range(0, N, 1 << 20):
                Bs[s:s + (1 << 20)] = Bs[s:s + (1 << 20)].astype(np.float16).astype(np.float32)
        bdesc = f"the full {N} x {O_COLS} fp32 B"
        out_col = scol.astype(np.int32)
    else:
        uniq, inv = np.unique(scol, return_inverse=True)
        from vcsr_mc_b200 import rng
        Bs = np.empty((uniq.size, O_COLS), dtype=np.float32)
        for s in range(0, uniq.size, 1 << 16):  # rows of the dense stream = the GPU's B values
            Bs[s:s + (1 << 16)] = rng.dense_rows(uniq[s:s + (1 << 16)], O_COLS, SEED)
        if fp16_b:
            Bs = Bs.astype(np.float16).astype(np.float32)
        bdesc = f"B compacted to the {uniq.size} rows those touch (host memory too small for the full B), fp32"
        out_col = inv.astype(np.int32)
    desc = f"every {k}-th row of A ({rows.size} rows, {int(srp[-1])} nnz), {bdesc}, O={O_COLS}"
    return srp.astype(np.int32), out_col, sval, Bs, desc, int(srp[-1])


def time_reference_cpu(M, N, rp, col, val, steps: int, warmup: int, target_nnz: int, fp16_b: bool):
    from oracle import bind as ob
    if not ob.ref_available():
        raise RuntimeError("oracle/_ref/libvcsr_ref.so not built")
    srp, scol, sval, Bs, desc, snnz = cpu_sample(M, N, rp, col, val, target_nnz, fp16_b)
    cores = len(os.sched_getaffinity(0))
    runner = ob.RefSpmm(srp, scol, sval, Bs, nslices=cores)
    for _ in range(warmup):
        runner.run()
    t = time.perf_counter()
    for _ in range(steps):
        runner.run()
    dt = (time.perf_counter() - t) / max(1, steps)
    runner.close()
    # the same loop on one core, one pass after one warm-up pass
    one = ob.RefSpmm(srp, scol, sval, Bs, nslices=1)
    one.run()
    t = time.perf_counter()
    one.run()
    dt1 = time.perf_counter() - t
    one.close()
    return {"value": 2.0 * snnz * O_COLS / dt / 1e9, "unit": "GFLOP/s", "cores": cores, "kind": "reference",
            "sample": desc + f"; reference loop src/main.cpp:202-207 on {cores} row slices/threads, "
                             f"{steps} timed passes after {warmup} warm-up",
            "ms_per_step": dt * 1e3, "cpu_model": cpu_model(),
            "single_core": {"value": 2.0 * snnz * O_COLS / dt1 / 1e9, "unit": "GFLOP/s", "ms_per_step": dt1 * 1e3}}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_cusparse(rp, col, val, r0, r1, p0, p1, N, B, fp16: bool, stream) -> dict:
    """cuSPARSE CSR SpMM (libvcsrmc_cusparse.so) on this rank's rows and the same device B:
    FP16 A/B with FP32 compute and C for the FP16 path, FP32 otherwise. Median of 10 launches."""
    import ctypes
    import torch
    path = os.path.join(ROOT, "vcsr_mc_b200", "libvcsrmc_cusparse.so")
    if not os.path.exists(path):
        return {"unavailable": "libvcsrmc_cusparse.so not built"}
    lib = ctypes.CDLL(path)
    lib.vcsrmc_cusparse_last_error.restype = ctypes.c_char_p
    d_rp = torch.from_numpy(np.asarray(rp[r0:r1 + 1], dtype=np.int64) - p0).to(torch.int32).cuda()
    d_col = torch.from_numpy(np.array(col[p0:p1], dtype=np.int32)).cuda()
    v = torch.from_numpy(np.array(val[p0:p1], dtype=np.float32)).cuda()
    d_val = v.half() if fp16 else v
    C = torch.empty((max(r1 - r0, 1), B.shape[1]), dtype=torch.float32, device="cuda")
    ms = ctypes.c_float()
    rc = lib.vcsrmc_cusparse_spmm(ctypes.c_int32(r1 - r0), ctypes.c_int32(N), ctypes.c_int64(p1 - p0),
                                  ctypes.c_void_p(d_rp.data_ptr()), ctypes.c_void_p(d_col.data_ptr()),
                                  ctypes.c_void_p(d_val.data_ptr()), 1 if fp16 else 0, ctypes.c_void_p(B.data_ptr()),
                                  1 if fp16 else 0, ctypes.c_int32(B.shape[1]), ctypes.c_void_p(C.data_ptr()),
                                  ctypes.c_float(1.0), 3, 10, ctypes.c_void_p(stream.cuda_stream), ctypes.byref(ms))
    if rc != 0:
        return {"unavailable": lib.vcsrmc_cusparse_last_error().decode()}
    nnz = p1 - p0
    return {"algo": "cusparseSpMM CSR_ALG_DEFAULT " + ("fp16 A/B, fp32 C" if fp16 else "fp32"),
            "ms": ms.value, "gflops": 2.0 * nnz * B.shape[1] / (ms.value * 1e6), "rows": r1 - r0, "nnz": nnz}


# ---------------------------------------------------------------------------------------------
def shard_balance(args, spec: dict, fp16: bool) -> None:
    """Per-shard SpMM times of N-way row partitions, measured shard by shard on one GPU."""
    import torch
    import vcsr_mc_b200 as vm
    M, N, rp, col, val = load_or_generate_csr(spec, 0, 1, lambda: None)
    rp32 = np.asarray(rp, dtype=np.int32)
    plan = {"rows": vm.PLAN_ROWS, "segment": vm.PLAN_SEGMENT, "band": vm.PLAN_BAND, "hybrid": vm.PLAN_HYBRID}[args.plan]
    B = torch.empty((N, O_COLS), dtype=torch.float16 if fp16 else torch.float32, device="cuda")
    vm.gen_dense_device(B, SEED)

    def shard_ms(r0: int, r1: int) -> float:
        p0, p1 = int(rp[r0]), int(rp[r1])
        d_rp = torch.from_numpy(np.asarray(rp[r0:r1 + 1], dtype=np.int64) - p0).to(torch.int32).cuda()
        d_col = torch.from_numpy(np.asarray(col[p0:p1])).cuda()
        d_val = torch.from_numpy(np.asarray(val[p0:p1])).cuda()
        dV = vm.build_vcsr_mc_device(d_rp, d_col, d_val, r1 - r0, N, fp32=not fp16, segw=args.segw, device=0,
                                     plans=[plan])
        del d_rp, d_col, d_val
        C = torch.empty((max(r1 - r0, 1), O_COLS), dtype=torch.float32, device="cuda")
        for _ in range(args.warmup):
            vm.spmm(dV, B, C, tileK=args.tileK, plan=plan)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            vm.spmm(dV, B, C, tileK=args.tileK, plan=plan)
        b.record()
        torch.cuda.synchronize()
        dV.free()
        return a.elapsed_time(b) / args.steps

    full = shard_ms(0, M)
    out = {"mode": "shard_balance", "workload": spec["desc"], "dtype": args.dtype, "plan": args.plan,
           "one_gpu_ms": full, "partitions": []}
    for world in [int(x) for x in args.shard_balance.split(",") if x]:
        for w in [float(x) for x in args.row_weights.split(",") if x]:
            cuts = vm.partition_rows(rp32, world, row_weight=w)
            ms = [shard_ms(int(cuts[k]), int(cuts[k + 1])) for k in range(world)]
            out["partitions"].append({"gpus": world, "row_weight": w, "shard_ms": ms,
                                      "predicted_efficiency": full / (world * max(ms))})
            log(f"{world} GPUs, row weight {w}: shards {[round(x, 3) for x in ms]} "
                f"-> efficiency {full / (world * max(ms)):.3f}")
    emit(out)


def main() -> None:
    # Only the result line goes to stdout: everything else (libraries included, e.g. NCCL's
    # version banner) is sent to stderr at the file-descriptor level.
    result_fd = os.dup(1)
    os.dup2(2, 1)
    global _RESULT_FD
    _RESULT_FD = result_fd
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["rmat", "c1", "c2", "c3", "c3links"], default="rmat")
    ap.add_argument("--scale", type=int, default=24)
    ap.add_argument("--dtype", choices=["fp16", "fp32"], default="fp16")
    ap.add_argument("--segw", type=int, default=32)
    ap.add_argument("--tileK", type=int, default=128)
    ap.add_argument("--plan", choices=["rows", "segment", "band", "hybrid"], default="rows")
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cusparse", action="store_true")
    ap.add_argument("--no-c-gather", action="store_true", help="skip the separately timed gather of C to rank 0 (N > 1)")
    ap.add_argument("--cpu-sample-nnz", type=int, default=8_000_000)
    ap.add_argument("--build", choices=["host", "device"], default="device",
                    help="format construction: device (GPU builder, about 0.3 s on config 4) or host (bit-identical "
                         "to the reference builder, about 15 s on config 4 and all host cores per rank)")
    ap.add_argument("--unit-nnz", type=int, default=0,
                    help="ROWS plan: entries per work unit (0 = the library's choice for the matrix)")
    ap.add_argument("--hot-rows", type=int, default=0,
                    help="ROWS plan hot columns (opt-in): rank this many most used columns (0 = none)")
    ap.add_argument("--hot-budget-mib", type=int, default=0,
                    help="hot columns: MiB of their B rows copied into a compact buffer per call (0 = no copy)")
    ap.add_argument("--hot-persist", type=int, default=0, help="hot columns: persisting L2 window on the copy")
    ap.add_argument("--hot-evict-first", type=int, default=0,
                    help="hot columns: read the rows of unranked columns with evict-first loads")
    ap.add_argument("--row-weight", type=float, default=None,
                    help="shard balance: cost = nnz + row_weight * rows (0 = nnz balance; default: the "
                         "library's SHARD_ROW_WEIGHT)")
    ap.add_argument("--shard-balance", default="",
                    help="e.g. 2,4,8: time every shard of each N-way row partition one after another on this "
                         "GPU (the path has no collective, so the slowest shard predicts the N-GPU step) and "
                         "print that instead of the bench line")
    ap.add_argument("--row-weights", default="0,3,3.8,5.4", help="row weights tried by --shard-balance")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.row_weight is None:
        import vcsr_mc_b200 as vm
        args.row_weight = vm.SHARD_ROW_WEIGHT

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    spec = workload_spec(args.workload, args.scale)
    fp16 = args.dtype == "fp16"
    config = {"workload": spec["desc"], "O": O_COLS, "segw": args.segw, "tileK": args.tileK,
              "path": (("fp16 A/B, fp32 accumulate, " if fp16 else "fp32, ") +
                       ("CUDA-core FFMA" if (args.plan == "rows" or not fp16) else "tcgen05 MMA, TMEM accumulator")),
              "plan": {"rows": "rows: row-stationary over the VCSR-MC row view (for a GPU-built format the row view "
                               "is the CSR itself with fp16 values, so this is a CSR SpMM; the VCSR-MC arrays feed the "
                               "SEGMENT/BAND plans and validation), C stored once",
                       "segment": "segment: reference dataflow, per-item B segment, C reductions",
                       "band": "band: {band_rows}-row bands x {band_cols}-column tiles on tcgen05 (transposed product, "
                               "MMA M = 128 columns of C, N = {band_n} band rows), TMEM accumulator, C stored once",
                       "hybrid": "hybrid: band tiles ({hybrid_rows}-row bands) with >= 64 entries on tcgen05 (C stored "
                                 "once), the other entries on the rows plan added into C"}[args.plan],
              "parallelism": f"row-shard x{args.gpus} (balanced on nnz + {args.row_weight} x rows), B replicated",
              "l2": None}

    if args.shard_balance:
        shard_balance(args, spec, fp16)
        return

    if args.impl == "reference":
        # The reference's own CPU implementation of the path (oracle/_ref), rank 0 only.
        if rank != 0:
            return
        config["path"] = ("the reference's fp64 CSR SpMM loop (src/main.cpp:202-207, built from its sources into "
                          "oracle/_ref), fp64 accumulate, on host cores; B holds the GPU run's values" +
                          (" rounded to fp16" if fp16 else ""))
        config["plan"] = "reference CPU loop, rows split into one slice per host thread"
        try:
            M, N, rp, col, val = load_or_generate_csr(spec, 0, 1, lambda: None)
            cb = time_reference_cpu(M, N, rp, col, val, args.steps, args.warmup, args.cpu_sample_nnz, fp16)
        except Exception as e:  # noqa: BLE001
            emit({"impl": "reference", "unavailable": f"{type(e).__name__}: {e}"})
            return
        emit({
            "impl": "reference", "metric": "SpMM effective GFLOP/s (2*nnz*N/t)", "value": cb["value"],
            "unit": "GFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f64" , "data": "synthetic", "config": config,
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model", "single_core")},
            "e2e": {"value": cb["value"], "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return

    import torch
    import vcsr_mc_b200 as vm

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist  # noqa: F811
        dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=20), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    cores = len(os.sched_getaffinity(0))
    t0 = time.time()
    M, N, rp, col, val = load_or_generate_csr(spec, rank, world, barrier)
    nnz_total = int(rp[M])
    cuts = vm.partition_rows(np.asarray(rp, dtype=np.int32), world, row_weight=args.row_weight)
    r0, r1 = int(cuts[rank]), int(cuts[rank + 1])
    p0, p1 = int(rp[r0]), int(rp[r1])
    shard = vm.CSR.from_arrays(r1 - r0, N, np.asarray(rp[r0:r1 + 1], dtype=np.int64) - p0,
                               np.asarray(col[p0:p1]), np.asarray(val[p0:p1]))
    nthreads = max(1, cores // world)
    plan = {"rows": vm.PLAN_ROWS, "segment": vm.PLAN_SEGMENT, "band": vm.PLAN_BAND, "hybrid": vm.PLAN_HYBRID}[args.plan]
    hot = {"hot_rows": args.hot_rows, "hot_budget_mib": args.hot_budget_mib, "hot_persist": args.hot_persist,
           "hot_evict_first": args.hot_evict_first}
    torch.cuda.synchronize()
    tb = time.time()
    if args.build == "device":
        # the shard's CSR goes to the GPU once and the format is built there
        d_rp = torch.from_numpy(np.asarray(shard.arrays(copy=False)[0])).cuda()
        d_col = torch.from_numpy(np.asarray(shard.arrays(copy=False)[1])).cuda()
        d_val = torch.from_numpy(np.asarray(shard.arrays(copy=False)[2])).cuda()
        dV = vm.build_vcsr_mc_device(d_rp, d_col, d_val, shard.M, shard.N, fp32=not fp16, segw=args.segw,
                                     device=local, plans=[plan], rows_unit_nnz=args.unit_nnz, **hot)
        del d_rp, d_col, d_val
    else:
        V = vm.csr_to_vcsr_mc(shard, fp32=not fp16, segw=args.segw, nthreads=nthreads)
        dV = vm.upload_vcsr_mc_device(V, device=local, plans=[plan], rows_unit_nnz=args.unit_nnz, **hot)
        del V
    torch.cuda.synchronize()
    build_s = time.time() - tb
    D = int(np.unique(np.asarray(col[p0:p1])).size) if p1 > p0 else 0
    Ms = r1 - r0
    info = dV.info()
    # this library's kernels per step: the SpMM kernel, plus (ROWS plan) the zeroing of the rows
    # split into chunks that are reduced into C
    launches_per_step = (2 if plan == vm.PLAN_HYBRID and info["hybrid_rows_nnz"] > 0 else 1) + \
        (1 if plan == vm.PLAN_ROWS and info["n_split_rows"] > 0 else 0) + \
        (1 if plan == vm.PLAN_ROWS and info["n_hot"] > 0 and args.hot_budget_mib > 0 else 0)
    groups, slots, items = info["n_groups"], info["n_slots"], info["n_items"]
    config["plan"] = config["plan"].format(band_cols=info["band_cols"], band_rows=info["band_rows"],
                                           band_n=64 if info["band_rows"] <= 64 else 128,
                                           hybrid_rows=info["hybrid_band_rows"])
    log(f"rank {rank}: rows [{r0},{r1}) nnz {p1 - p0} format build + upload ({args.build}) {build_s:.2f}s "
        f"setup {time.time() - t0:.1f}s")

    dt = torch.float16 if fp16 else torch.float32
    B = torch.empty((N, O_COLS), dtype=dt, device="cuda")
    vm.gen_dense_device(B, SEED)
    C = torch.empty((max(Ms, 1), O_COLS), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    # Inputs that do not dwarf the L2 would be served from it on the next step: flush it by
    # writing a buffer twice its size before every step and time only the SpMM call (per-step
    # events on the launching stream).
    s_ab = 2 if fp16 else 4
    footprint = (p1 - p0) * (4 + s_ab) + (Ms + 1) * 4 + N * O_COLS * s_ab + Ms * O_COLS * 4
    flush = footprint < 4 * L2_BYTES
    l2buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda") if flush else None
    config["l2"] = (f"footprint {footprint / 1e6:.0f} MB < 4 x L2: L2 flushed (write of {2 * L2_BYTES >> 20} MiB) "
                    "before every step; time = per-step CUDA events around the SpMM call" if flush else
                    f"footprint {footprint / 1e9:.2f} GB, larger than L2 (126 MB): no flush; time = K back-to-back steps")

    def step(ev_k0=None, ev_k1=None, i=0):
        if flush:
            l2buf.fill_(i & 0xff)
        # ROWS plan: every C row is stored once, so no zeroing pass; SEGMENT plan: C += A*B
        # through reductions needs C zeroed first (the reference's caller does the same).
        if plan == vm.PLAN_SEGMENT:
            C.zero_()
        if ev_k0 is not None:
            ev_k0.record(stream)
        vm.spmm(dV, B, C, tileK=args.tileK, accumulate=plan == vm.PLAN_SEGMENT, stream=stream, plan=plan)
        if ev_k1 is not None:
            ev_k1.record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    per_step_events = flush or plan == vm.PLAN_SEGMENT
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    tw0 = time.time()
    start.record(stream)
    for i in range(args.steps):
        # per-step events only where something else runs between the SpMM calls (the L2 flush, or
        # the SEGMENT plan's zeroing of C); otherwise the K calls run back to back and the SpMM time
        # is the whole region over K
        if per_step_events:
            step(*kev[i], i=i)
        else:
            step(i=i)
    stop.record(stream)
    torch.cuda.synchronize()
    tw1 = time.time()
    barrier()
    clk = clocks.stop(window=(tw0, tw1))
    total_ms = start.elapsed_time(stop)
    kern_ms = float(np.mean([a.elapsed_time(b) for a, b in kev])) if per_step_events else total_ms / args.steps
    status = dV.status()
    # max over ranks
    t = torch.tensor([total_ms, kern_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, kern_max_ms = float(t[0]), float(t[1])
    ms_per_step = kern_max_ms if flush else total_ms / args.steps
    flops = 2.0 * nnz_total * O_COLS
    value = flops / (ms_per_step * 1e-3) / 1e9

    # roofline of the SpMM kernel on this rank (algorithmic bytes of this rank's launch)
    bytes_alg = algorithmic_bytes(p1 - p0, Ms, D, O_COLS, s_ab)
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    if os.path.exists(peaks_path):
        with open(peaks_path) as f:
            peak = float(json.load(f)["hbm_gbs"])
        peak_src = "measured (MEASURED_PEAKS.json hbm_gbs)"
    achieved = bytes_alg / (kern_ms * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "measured_traffic.json")
    tkey = f"{args.workload}{args.scale if args.workload == 'rmat' else ''}/{args.dtype}/{args.plan}"
    if world == 1 and os.path.exists(tpath):
        with open(tpath) as f:
            rec = json.load(f).get(tkey)
        if rec:
            traffic = rec["dram_bytes_read"] + rec["dram_bytes_write"]

    # The reference's own contract, C += A*B into a C that its caller zeroed outside the timed
    # region (src/main.cpp:242-243, src/vcsr_mc.cu:352-394): the same K steps in accumulate mode,
    # C zeroed once before the warm-up. Reported beside the headline, which stores C = A*B and so
    # needs no zeroed C; the SEGMENT plan's headline already is this contract.
    acc_line = None
    if plan != vm.PLAN_SEGMENT:
        C.zero_()

        def acc_step(ev0=None, ev1=None, i=0):
            if flush:
                l2buf.fill_(i & 0xff)
            if ev0 is not None:
                ev0.record(stream)
            vm.spmm(dV, B, C, tileK=args.tileK, accumulate=True, stream=stream, plan=plan)
            if ev1 is not None:
                ev1.record(stream)

        for _ in range(args.warmup):
            acc_step()
        torch.cuda.synchronize()
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for i in range(args.steps):
            if flush:
                acc_step(*kev[i], i=i)
            else:
                acc_step(i=i)
        a1.record(stream)
        torch.cuda.synchronize()
        acc_ms = float(np.mean([x.elapsed_time(y) for x, y in kev])) if flush else a0.elapsed_time(a1) / args.steps
        ta = torch.tensor([acc_ms], dtype=torch.float64, device="cuda")
        if dist is not None:
            dist.all_reduce(ta, op=dist.ReduceOp.MAX)
        acc_ms = float(ta[0])
        acc_line = {"contract": "C += A*B (the reference's run_vcsr_mc_spmm_gpu), C zeroed once before the "
                                "warm-up as the reference's caller zeroes it outside its timed region",
                    "ms_per_step": acc_ms, "value": flops / (acc_ms * 1e-3) / 1e9, "unit": "GFLOP/s",
                    "steps": args.steps, "warmup": args.warmup, "status": dV.status()}

    # End to end through the C ABI with host buffers: every step uploads its B from pinned host
    # memory, runs the SpMM and downloads its C. Steps alternate between two device copies of B
    # and C so that the upload of step i+1 (copy stream 1) overlaps the download of step i (copy
    # stream 2): PCIe moves both directions at once. With several ranks each rank uploads 1/N of
    # B's rows and the ranks all-gather the full B over NVLink (NCCL), instead of every rank
    # pushing the whole B through its own PCIe link. Timed with events on the compute stream, max
    # over ranks.
    e2e = None
    if not args.no_e2e and args.e2e_steps > 0:
        if world > 1:
            piece = (N + world - 1) // world
            lo, hi = min(rank * piece, N), min((rank + 1) * piece, N)
            hB = torch.zeros((piece, O_COLS), dtype=B.dtype).pin_memory()
            hB[: hi - lo] = B[lo:hi].cpu()
            Bfull = [torch.empty((world * piece, O_COLS), dtype=B.dtype, device="cuda") for _ in range(2)]
            Bpiece = [torch.empty((piece, O_COLS), dtype=B.dtype, device="cuda") for _ in range(2)]
            Bd = [t[:N] for t in Bfull]
        else:
            hB = B.cpu().pin_memory()
            Bd = [B, torch.empty_like(B)]
        hC = torch.empty(C.shape, dtype=torch.float32).pin_memory()
        Cd = [C, torch.empty_like(C)]
        up_stream, down_stream = torch.cuda.Stream(), torch.cuda.Stream()
        ev_up = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_down = [torch.cuda.Event() for _ in range(2)]

        def e2e_steps(n: int, first: int) -> None:
            for i in range(first, first + n):
                k = i % 2
                if i >= 2:  # buffer k was read by the SpMM of step i - 2
                    up_stream.wait_event(ev_comp[k])
                with torch.cuda.stream(up_stream):
                    if world > 1:
                        Bpiece[k].copy_(hB, non_blocking=True)
                        dist.all_gather_into_tensor(Bfull[k], Bpiece[k])
                    else:
                        Bd[k].copy_(hB, non_blocking=True)
                    ev_up[k].record(up_stream)
                stream.wait_event(ev_up[k])
                if i >= 2:  # C buffer k was read by the download of step i - 2
                    stream.wait_event(ev_down[k])
                if plan == vm.PLAN_SEGMENT:
                    Cd[k].zero_()
                vm.spmm(dV, Bd[k], Cd[k], tileK=args.tileK, accumulate=plan == vm.PLAN_SEGMENT, stream=stream,
                        plan=plan)
                ev_comp[k].record(stream)
                down_stream.wait_event(ev_comp[k])
                with torch.cuda.stream(down_stream):
                    hC.copy_(Cd[k], non_blocking=True)
                    ev_down[k].record(down_stream)

        e2e_steps(2, 0)  # warm-up: both buffer pairs once
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        up_stream.wait_stream(stream)
        e2e_steps(args.e2e_steps, 2)
        stream.wait_event(ev_down[(args.e2e_steps + 1) % 2])
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.e2e_steps], dtype=torch.float64, device="cuda")
        if dist is not None:
            dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        # The link's own floor for one step: this rank's B upload and C download timed alone and
        # together (the two directions of PCIe run at once), the same bytes as a step.
        def copy_ms(up: bool, down: bool) -> float:
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            up_stream.wait_stream(stream)
            down_stream.wait_stream(stream)
            if up:
                with torch.cuda.stream(up_stream):
                    (Bpiece[0] if world > 1 else Bd[0]).copy_(hB, non_blocking=True)
            if down:
                with torch.cuda.stream(down_stream):
                    hC.copy_(Cd[0], non_blocking=True)
            stream.wait_stream(up_stream)
            stream.wait_stream(down_stream)
            b.record(stream)
            torch.cuda.synchronize()
            return a.elapsed_time(b)

        up_ms, down_ms, both_ms = copy_ms(True, False), copy_ms(False, True), copy_ms(True, True)
        h2d_b, d2h_b = hB.numel() * hB.element_size(), hC.numel() * hC.element_size()
        # per rank: its copy times and rates; the job's step takes the slowest rank's, and its bytes
        # are the sum over ranks
        local = torch.tensor([up_ms, down_ms, both_ms, -h2d_b / max(up_ms, 1e-6) * 1e-6,
                              -d2h_b / max(down_ms, 1e-6) * 1e-6], dtype=torch.float64, device="cuda")
        total = torch.tensor([float(h2d_b), float(d2h_b)], dtype=torch.float64, device="cuda")
        if dist is not None:
            dist.all_reduce(local, op=dist.ReduceOp.MAX)
            dist.all_reduce(total, op=dist.ReduceOp.SUM)
        up_ms, down_ms, both_ms, up_rate, down_rate = (float(x) for x in local.tolist())
        e2e = {"value": flops / (float(e2e_ms) * 1e-3) / 1e9, "unit": "GFLOP/s",
               "h2d_bytes_per_step": int(total[0]), "d2h_bytes_per_step": int(total[1]),
               "bytes_scope": "summed over ranks" if world > 1 else "one rank",
               "ms_per_step": float(e2e_ms),
               "pipelining": "upload of step i+1 overlaps download of step i (two device buffers, two copy streams)",
               "steps": args.e2e_steps,
               "link": {"h2d_ms": up_ms, "d2h_ms": down_ms, "both_ms": both_ms,
                        "h2d_GBps": -up_rate, "d2h_GBps": -down_rate,
                        "floor_ms_per_step": both_ms,
                        "frac": both_ms / max(float(e2e_ms), 1e-6),
                        "how": "this step's H2D and D2H copies of each rank timed alone and at once; times are "
                               "the slowest rank's, GB/s the slowest rank's own bytes over its own time"},
               "b_staging": ("each rank uploads 1/N of B, NCCL all-gather over NVLink" if world > 1 else
                             "B uploaded whole"),
               "a_resident": True,
               "a_scope": "A's format is built and uploaded once before the timed region (persistent A, as the "
                          "reference's upload_vcsr_mc_device); only B up, the SpMM and C down are timed per step",
               "format_build": args.build, "format_build_upload_s": build_s}
        del Bd, Cd, hB, hC

    # Optional gather of C to rank 0 over NVLink (NCCL point-to-point), timed on its own: the
    # SpMM needs no collective, so this is not part of the step.
    c_gather = None
    if dist is not None and not args.no_c_gather:
        Cfull = torch.empty((M, O_COLS), dtype=torch.float32, device="cuda") if rank == 0 else None

        def gather() -> None:
            if rank == 0:
                Cfull[r0:r1].copy_(C[:Ms])
                ops = [dist.P2POp(dist.irecv, Cfull[int(cuts[k]):int(cuts[k + 1])], k) for k in range(1, world)
                       if cuts[k + 1] > cuts[k]]
            else:
                ops = [dist.P2POp(dist.isend, C[:Ms], 0)] if Ms > 0 else []
            for q in (dist.batch_isend_irecv(ops) if ops else []):  # empty shards send nothing
                q.wait()

        gather()  # the first point-to-point exchange also sets up NCCL's connections: untimed
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        gather()
        g1.record(stream)
        torch.cuda.synchronize()
        gms = torch.tensor([g0.elapsed_time(g1)], dtype=torch.float64, device="cuda")
        dist.all_reduce(gms, op=dist.ReduceOp.MAX)
        moved = (M - (r1 - r0 if rank == 0 else 0)) * O_COLS * 4
        c_gather = {"ms": float(gms), "bytes_to_rank0": int(moved),
                    "GB_per_s": moved / (float(gms) * 1e-3) / 1e9 if float(gms) > 0 else None,
                    "how": "NCCL batch_isend_irecv into one M x O buffer on rank 0, max over ranks"}
        del Cfull
        barrier()

    cusparse = None
    if rank == 0 and not args.no_cusparse:
        cusparse = time_cusparse(rp, col, val, r0, r1, p0, p1, N, B, fp16, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cb = time_reference_cpu(M, N, rp, col, val, args.steps, args.warmup, args.cpu_sample_nnz, fp16)
            cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model", "single_core")}
        except Exception as e:  # noqa: BLE001
            cpu = {"value": None, "unavailable": f"{type(e).__name__}: {e}"}

    if rank == 0:
        line = {
            "metric": "SpMM effective GFLOP/s (2*nnz*N/t)", "value": value, "unit": "GFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16" if fp16 else "f32",
            "data": "synthetic (seeded generator, seed 0)",
            "config": config,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                                           "(profiles/measured_traffic.json)" if traffic else None,
                         "kernel": {"rows": "vcsr_rows_kernel", "band": "vcsr_band_kernel", "hybrid": "vcsr_band_kernel",
                                    "segment": "vcsr_mc_fp16_tc_kernel" if fp16 else "vcsr_mc_fp32_kernel"}[args.plan],
                         "kernel_ms": kern_ms, "kernel_ms_max_over_ranks": kern_max_ms,
                         "algorithmic_bytes": bytes_alg},
            "cpu_baseline": cpu, "e2e": e2e, "cusparse": cusparse, "c_gather": c_gather,
            "gpu_launches": args.steps * launches_per_step,
            "accumulate": acc_line,
            "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            "detail": {"nnz": nnz_total, "M": M, "N": N, "rank0_rows": Ms, "rank0_distinct_cols": D,
                       "groups": groups, "slots": slots, "items": items, "device_status": status,
                       "format_build": args.build, "format_build_upload_s": build_s,
                       "rows_unit_nnz": info["rows_unit_nnz"], "band_rows": info["band_rows"],
                       "band_tiles": info["n_tiles"], "clock_samples": clk["samples"],
                       "clock_samples_timed_region_only": clk["timed_region_only"],
                       "hot_columns": {**hot, "n_hot": info["n_hot"]}},
        }
        emit(line)
    dV.free()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
