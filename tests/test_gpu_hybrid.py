"""HYBRID plan on the GPU, through the C ABI, against the fp64 oracle.

The band tiles with at least 64 entries run on the tensor cores (BAND kernel, every row of C written
or added to), every other entry then runs on the rows plan, added into C. Cases: the config-2
power-law matrix (no dense tile: all entries on the rows plan), the config-3 stencil (nearly every
entry in dense tiles), an R-MAT (dense tiles only where heavy rows meet popular columns) and a
stencil with random long-range entries added (both parts large), with store and accumulate, fp16
and fp32 B, and ragged widths.
"""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16

pytestmark = pytest.mark.gpu


MATRICES = {
    "c2": lambda: vm.CSR.generate(vm.GEN_ZIPF, 1 << 16, seed=0),
    "c3": lambda: vm.CSR.generate(vm.GEN_STENCIL27, 40, seed=0),
    "rmat14": lambda: vm.CSR.generate(vm.GEN_RMAT, 14, seed=0),
    "mixed": lambda: vm.CSR.generate(vm.GEN_STENCIL27_LINKS, 32, seed=1),
}
_cache = {}


def matrix(name):
    if name not in _cache:
        _cache[name] = MATRICES[name]()
    return _cache[name]


def run_hybrid(torch, A, O, b_half, accumulate_into=None, band_rows=0):
    V = vm.csr_to_vcsr_mc(A, fp32=False, segw=32)
    dV = vm.upload_vcsr_mc_device(V, device=0, plans=[vm.PLAN_HYBRID], band_rows=band_rows)
    info = dV.info()
    B32 = vm.gen_dense_host(A.N, O, seed=3)
    B = torch.from_numpy(B32).cuda()
    B = B.half() if b_half else B
    C = torch.full((A.M, O), 2.0, device="cuda")
    if accumulate_into is not None:
        C.copy_(torch.from_numpy(accumulate_into))
    vm.spmm(dV, B, C, accumulate=accumulate_into is not None, O=O, plan=vm.PLAN_HYBRID)
    torch.cuda.synchronize()
    assert dV.status() == 0
    dV.free()
    return C.cpu().numpy(), B.float().cpu().numpy(), info


@pytest.mark.parametrize("name", list(MATRICES))
@pytest.mark.parametrize("accumulate", [False, True], ids=["store", "accumulate"])
def test_hybrid_matches_oracle(cuda, name, accumulate):
    A = matrix(name)
    base = np.random.default_rng(5).uniform(-1, 1, size=(A.M, 128)).astype(np.float32) if accumulate else None
    C, Bu, info = run_hybrid(cuda, A, 128, True, accumulate_into=base)
    assert info["hybrid_band_nnz"] + info["hybrid_rows_nnz"] == A.nnz
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, Bu, with_abs=True)
    if base is not None:
        ref, ab = ref + base, ab + np.abs(base)
    check_fp16(C, ref, ab)


def test_split_follows_the_matrix(cuda):
    """No dense tile on the power-law matrix; nearly all entries dense on the stencil; both parts
    large on the stencil with random long-range entries."""
    parts = {}
    for name in ("c2", "c3", "mixed"):
        A = matrix(name)
        dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=[vm.PLAN_HYBRID])
        i = dV.info()
        parts[name] = (i["hybrid_band_nnz"] / A.nnz, i["hybrid_tiles"])
        dV.free()
    assert parts["c2"] == (0.0, 0)
    assert parts["c3"][0] > 0.95
    assert 0.5 < parts["mixed"][0] < 0.95


@pytest.mark.parametrize("O,b_half", [(130, True), (64, False), (256, True)], ids=["O130-f16B", "O64-f32B", "O256-f16B"])
def test_hybrid_widths_and_b_types(cuda, O, b_half):
    A = matrix("mixed")
    C, Bu, _ = run_hybrid(cuda, A, O, b_half)
    if not b_half:
        Bu = Bu.astype(np.float16).astype(np.float32)  # the tensor cores multiply fp16 B
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, Bu, with_abs=True)
    check_fp16(C, ref, ab)


@pytest.mark.parametrize("band_rows", [64, 100, 128])
def test_hybrid_band_heights(cuda, band_rows):
    A = matrix("mixed")
    C, Bu, info = run_hybrid(cuda, A, 128, True, band_rows=band_rows)
    assert info["hybrid_band_rows"] == band_rows
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, Bu, with_abs=True)
    check_fp16(C, ref, ab)


def test_auto_picks_the_resident_hybrid_layout(cuda):
    A = matrix("mixed")
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=[vm.PLAN_HYBRID])
    B = cuda.from_numpy(vm.gen_dense_host(A.N, 128, seed=3)).cuda().half()
    C = cuda.zeros((A.M, 128), device="cuda")
    vm.spmm(dV, B, C, accumulate=False)  # AUTO
    cuda.cuda.synchronize()
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    check_fp16(C.cpu().numpy(), ref, ab)
    dV.free()


def test_hybrid_errors(cuda):
    A = matrix("rmat14")
    with pytest.raises(vm.VcsrmcError) as e:  # tensor cores: FP16 format only
        vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=True, segw=32), device=0, plans=[vm.PLAN_HYBRID])
    assert e.value.status == 1
    rp, col, val = A.arrays()
    t = lambda a, dt: cuda.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dt)
    with pytest.raises(vm.VcsrmcError) as e:  # FP32 format on the GPU builder too
        vm.build_vcsr_mc_device(t(rp, cuda.int32), t(col, cuda.int32), t(val, cuda.float32), A.M, A.N, fp32=True,
                                plans=[vm.PLAN_HYBRID])
    assert e.value.status == 1
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=[vm.PLAN_ROWS])
    B = cuda.zeros((A.N, 128), device="cuda").half()
    C = cuda.zeros((A.M, 128), device="cuda")
    with pytest.raises(vm.VcsrmcError) as e:  # not resident
        vm.spmm(dV, B, C, plan=vm.PLAN_HYBRID)
    assert e.value.status == 1
    dV.free()


def test_default_layouts(cuda):
    """An upload (or a GPU build) without a plan mask adds BAND on the stencil, HYBRID on the stencil
    with random links (most entries in dense tiles, the mean tile too sparse for BAND alone), neither
    on the power-law matrix; AUTO then runs that plan."""
    want = {"c3": vm.PLAN_BAND, "mixed": vm.PLAN_HYBRID, "c2": None}
    for (name, plan), builder in [(x, b) for x in want.items() for b in ("upload", "device")]:
        A = matrix(name)
        if builder == "upload":
            dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0)
        else:
            rp, col, val = A.arrays()
            t = lambda a, dt: cuda.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dt)
            dV = vm.build_vcsr_mc_device(t(rp, cuda.int32), t(col, cuda.int32), t(val, cuda.float32), A.M, A.N,
                                         fp32=False, segw=32)
        plans = dV.info()["plans"]
        tensor = [p for p in plans if p in (vm.PLAN_BAND, vm.PLAN_HYBRID)]
        assert tensor == ([] if plan is None else [plan]), (name, plans)
        B = cuda.from_numpy(vm.gen_dense_host(A.N, 128, seed=6)).cuda().half()
        C = cuda.zeros((A.M, 128), device="cuda")
        vm.spmm(dV, B, C, accumulate=False)
        cuda.cuda.synchronize()
        rp, col, val = A.arrays()
        ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
        check_fp16(C.cpu().numpy(), ref, ab)
        dV.free()


@pytest.mark.parametrize("shape", ["empty-rows", "one-row", "narrow-N", "tiny"])
def test_hybrid_edge_shapes(cuda, shape):
    """Matrices with empty rows (whole empty bands), a single row, fewer columns than a tile, and a
    handful of entries: the band part may have no tile at all and the rows part no entry."""
    from tests.helpers import random_csr
    M, N, d = {"empty-rows": (700, 900, 0.05), "one-row": (1, 300, 0.5), "narrow-N": (500, 20, 0.5),
               "tiny": (5, 7, 0.3)}[shape]
    rp, col, val = random_csr(M, N, d, seed=11, empty_rows=shape == "empty-rows")
    if shape == "empty-rows":  # rows 200 .. 455 empty: two whole bands without entries
        keep = np.repeat(np.arange(M), np.diff(rp))
        mask = (keep < 200) | (keep >= 456)
        counts = np.bincount(keep[mask], minlength=M)
        rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        col, val = col[mask], val[mask]
    A = vm.CSR.from_arrays(M, N, rp, col, val)
    C, Bu, info = run_hybrid(cuda, A, 40, True)
    assert info["hybrid_band_nnz"] + info["hybrid_rows_nnz"] == A.nnz
    ref, ab = ob.spmm_fp64(rp, col, val, Bu, with_abs=True)
    check_fp16(C, ref, ab)


@pytest.mark.parametrize("name", ["mixed", "c3", "rmat14", "c2"])
def test_device_built_hybrid_equals_upload(cuda, name):
    """The GPU builder's HYBRID layout is the upload's: the same band height, dense tiles and entry
    split, and the same C (bit for bit outside rows reduced atomically in chunks, which are within
    fp32 rounding)."""
    A = matrix(name)
    rp, col, val = A.arrays()
    t = lambda a, dt: cuda.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dt)
    dD = vm.build_vcsr_mc_device(t(rp, cuda.int32), t(col, cuda.int32), t(val, cuda.float32), A.M, A.N, fp32=False,
                                 segw=32, plans=[vm.PLAN_HYBRID])
    dH = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0, plans=[vm.PLAN_HYBRID])
    iD, iH = dD.info(), dH.info()
    for k in ("hybrid_band_rows", "hybrid_tiles", "hybrid_band_nnz", "hybrid_rows_nnz"):
        assert iD[k] == iH[k], (k, iD[k], iH[k])
    assert vm.PLAN_BAND not in iD["plans"] and vm.PLAN_HYBRID in iD["plans"]
    B = cuda.from_numpy(vm.gen_dense_host(A.N, 128, seed=8)).cuda().half()
    out = []
    for dV in (dD, dH):
        C = cuda.full((A.M, 128), 4.0, device="cuda")
        vm.spmm(dV, B, C, accumulate=False, plan=vm.PLAN_HYBRID)
        cuda.cuda.synchronize()
        assert dV.status() == 0
        out.append(C.cpu().numpy())
        dV.free()
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    check_fp16(out[0], ref, ab)
    diff = np.abs(out[0].astype(np.float64) - out[1])
    assert np.all(diff <= 1e-5 * ab + 1e-30)
