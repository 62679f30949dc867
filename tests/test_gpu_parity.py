"""GPU parity of the VCSR-MC SpMM kernels against the fp64 CPU oracle, through the C ABI.

Every case builds A with the product's host builder (bit-identical to the reference builder),
uploads it, runs the sm_100a kernel (FP32: CUDA-core FFMA; FP16: tcgen05 tensor cores) and
compares C with the oracle's fp64 CSR SpMM (src/main.cpp:202-207) under the tolerances in
tests/helpers.py.
"""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16, check_fp32, random_csr

pytestmark = pytest.mark.gpu


PLANS = [vm.PLAN_SEGMENT, vm.PLAN_ROWS, vm.PLAN_BAND]
PLAN_IDS = ["segment", "rows", "band"]


def run_gpu(torch, A: vm.CSR, B32: np.ndarray, fp32: bool, segw: int, tileK: int, b_half: bool,
            accumulate_into=None, ldb_pad: int = 0, ldc_pad: int = 0, plan: int = vm.PLAN_SEGMENT,
            unit_nnz: int = 0, band_rows: int = 0):
    """C = A*B (or C = accumulate_into + A*B) on cuda:0 with one plan; returns (C, B values used)."""
    if plan == vm.PLAN_BAND and fp32:
        pytest.skip("the BAND plan runs on the tensor cores: FP16 format only")
    O = B32.shape[1]
    V = vm.csr_to_vcsr_mc(A, fp32=fp32, segw=segw)
    dV = vm.upload_vcsr_mc_device(V, device=0, plans=[plan], rows_unit_nnz=unit_nnz, band_rows=band_rows)
    dt = torch.float16 if b_half else torch.float32
    Bfull = torch.zeros((B32.shape[0], O + ldb_pad), dtype=dt, device="cuda")
    Bfull[:, :O] = torch.from_numpy(B32).to(device="cuda", dtype=dt)
    Cfull = torch.full((A.M, O + ldc_pad), 7.0, dtype=torch.float32, device="cuda")
    if accumulate_into is not None:
        Cfull[:, :O] = torch.from_numpy(accumulate_into).cuda()
    vm.spmm(dV, Bfull, Cfull, tileK=tileK, accumulate=accumulate_into is not None, O=O, plan=plan)
    torch.cuda.synchronize()
    assert dV.status() == 0, "a bounded device wait expired"
    C = Cfull[:, :O].cpu().numpy()
    Bused = Bfull[:, :O].float().cpu().numpy()
    dV.free()
    return C, Bused


def oracle_check(A: vm.CSR, C, Bused, fp32: bool, base=None):
    rp, col, val = A.arrays()
    ref, absref = ob.spmm_fp64(rp, col, val, Bused, with_abs=True)
    if base is not None:
        ref = ref + base
        absref = absref + np.abs(base)
    return check_fp32(C, ref, absref) if fp32 else check_fp16(C, ref, absref)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("segw", [16, 32, 48, 64])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_config1_segw(cuda, plan, fp32, segw):
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 4096, seed=0)
    B = vm.gen_dense_host(4096, 128, seed=0)
    C, Bu = run_gpu(cuda, A, B, fp32, segw, 128, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("tileK", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_config1_tilek(cuda, plan, fp32, tileK):
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 4096, seed=0)
    B = vm.gen_dense_host(4096, 256, seed=1)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, tileK, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_fp16_with_fp32_b(cuda, plan):
    """The reference's FP16 kernel reads fp32 B and converts it (src/vcsr_mc.cu:184-196)."""
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 4096, seed=3)
    B = vm.gen_dense_host(4096, 128, seed=3)
    C, _ = run_gpu(cuda, A, B, False, 32, 128, b_half=False, plan=plan)
    Bh = B.astype(np.float16).astype(np.float32)  # the values the tensor cores multiply
    oracle_check(A, C, Bh, False)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_zipf_power_law(cuda, plan, fp32):
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 16, seed=0)
    B = vm.gen_dense_host(1 << 16, 128, seed=0)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 128, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("unit_nnz", [16, 64, 1024])
@pytest.mark.parametrize("accumulate", [False, True], ids=["store", "accumulate"])
def test_rows_unit_sizes(cuda, unit_nnz, fp32, accumulate):
    """ROWS plan work units of 16 .. 1024 entries: heavy rows split into many or few chunks."""
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 14, seed=5)
    B = vm.gen_dense_host(1 << 14, 128, seed=5)
    base = np.random.default_rng(6).uniform(-1, 1, size=(A.M, 128)).astype(np.float32) if accumulate else None
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 128, b_half=not fp32, accumulate_into=base, plan=vm.PLAN_ROWS,
                    unit_nnz=unit_nnz)
    oracle_check(A, C, Bu, fp32, base=None if base is None else base.astype(np.float64))


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("O", [1, 8, 16, 24, 32, 33, 48, 64, 65])
@pytest.mark.parametrize("accumulate", [False, True], ids=["store", "accumulate"])
@pytest.mark.parametrize("aligned", [True, False], ids=["aligned", "unaligned"])
def test_rows_narrow_widths(cuda, O, fp32, accumulate, aligned):
    """ROWS plan on narrow B: with 16-byte aligned rows the main kernel (idle lanes masked); with
    unaligned rows the element-wise path, where 2 or 4 entries share a lane group for O <= 64
    (rows split across folds and steps, heavy-row chunks reduced into C)."""
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 14, seed=7)
    B = np.random.default_rng(O).uniform(-1, 1, size=(A.N, O)).astype(np.float32)
    base = np.random.default_rng(8).uniform(-1, 1, size=(A.M, O)).astype(np.float32) if accumulate else None
    elem = 4 if fp32 else 2
    # pad B's rows so that their pitch is (or is not) a multiple of 16 bytes
    pad = next(p for p in range(16) if (((O + p) * elem) % 16 == 0) == aligned)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 64, b_half=not fp32, accumulate_into=base, plan=vm.PLAN_ROWS,
                    unit_nnz=32, ldb_pad=pad)
    oracle_check(A, C, Bu, fp32, base=None if base is None else base.astype(np.float64))


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_stencil27(cuda, plan, fp32):
    A = vm.CSR.generate(vm.GEN_STENCIL27, 24, seed=0)
    B = vm.gen_dense_host(A.N, 128, seed=0)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 128, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_rmat_small(cuda, plan, fp32):
    A = vm.CSR.generate(vm.GEN_RMAT, 14, seed=0)
    B = vm.gen_dense_host(A.N, 128, seed=0)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 128, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("O", [1, 7, 40, 100, 130])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_ragged_width(cuda, plan, fp32, O):
    """O not a multiple of 4, of 16 or of the slab; O < 64 takes the non-TMA staging path."""
    rp, col, val = random_csr(301, 777, 0.02, seed=O)
    A = vm.CSR.from_arrays(301, 777, rp, col, val)
    B = np.random.default_rng(O).uniform(-1, 1, size=(777, O)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 64, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_strided_b_and_c(cuda, plan, fp32):
    rp, col, val = random_csr(200, 300, 0.05, seed=5, empty_rows=True)
    A = vm.CSR.from_arrays(200, 300, rp, col, val)
    B = np.random.default_rng(5).uniform(-1, 1, size=(300, 96)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, fp32, 16, 64, b_half=not fp32, ldb_pad=8, ldc_pad=12, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_accumulate_into_c(cuda, plan, fp32):
    """C += A*B: the reference's contract (its caller zeroes C first, src/main.cpp:242)."""
    rp, col, val = random_csr(128, 256, 0.05, seed=9)
    A = vm.CSR.from_arrays(128, 256, rp, col, val)
    B = np.random.default_rng(9).uniform(-1, 1, size=(256, 128)).astype(np.float32)
    base = np.random.default_rng(10).uniform(-1, 1, size=(128, 128)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, fp32, 32, 128, b_half=not fp32, accumulate_into=base, plan=plan)
    oracle_check(A, C, Bu, fp32, base=base.astype(np.float64))


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_tiny_and_partial_segment(cuda, plan, fp32):
    """N < segw, M not a multiple of 16, last partial segment zero-filled (src/vcsr_mc.cu:185)."""
    rp, col, val = random_csr(5, 7, 0.6, seed=2)
    A = vm.CSR.from_arrays(5, 7, rp, col, val)
    B = np.random.default_rng(2).uniform(-1, 1, size=(7, 64)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, fp32, 64, 64, b_half=not fp32, plan=plan)
    oracle_check(A, C, Bu, fp32)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_empty_matrix(cuda, plan, fp32):
    A = vm.CSR.from_arrays(10, 10, np.zeros(11, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32))
    B = np.ones((10, 32), np.float32)
    C, _ = run_gpu(cuda, A, B, fp32, 32, 64, b_half=not fp32, plan=plan)
    assert np.all(C == 0)


@pytest.mark.parametrize("amax", [1e6, 1e-6], ids=["large", "tiny"])
@pytest.mark.parametrize("plan", PLANS, ids=PLAN_IDS)
def test_half_scale_triggers(cuda, plan, amax):
    """|A| beyond the fp16 range is scaled by half_scale and C multiplied back (src/vcsr_mc.cu:14-22)."""
    rp, col, val = random_csr(64, 96, 0.1, seed=4, scale=amax)
    A = vm.CSR.from_arrays(64, 96, rp, col, val)
    assert vm.half_scale(A) != 1.0
    B = np.random.default_rng(4).uniform(-1, 1, size=(96, 64)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, False, 32, 64, b_half=True, plan=plan)
    oracle_check(A, C, Bu, False)


def test_spmm_overwrite_and_repeat(cuda):
    """accumulate=0 overwrites C; two launches give the same result within tolerance."""
    torch = cuda
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 2048, seed=7)
    B32 = vm.gen_dense_host(2048, 128, seed=7)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32))
    B = torch.from_numpy(B32).cuda().half()
    C = torch.full((2048, 128), 123.0, device="cuda")
    vm.spmm(dV, B, C, tileK=128, accumulate=False)
    C1 = C.cpu().numpy()
    vm.spmm(dV, B, C, tileK=128, accumulate=False)
    C2 = C.cpu().numpy()
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    check_fp16(C1, ref, ab)
    check_fp16(C2, ref, ab)
    dV.free()


def test_dense_device_generator_matches_host(cuda):
    torch = cuda
    h = vm.gen_dense_host(333, 77, seed=11)
    d32 = vm.gen_dense_device(torch.empty((333, 77), device="cuda"), seed=11)
    d16 = vm.gen_dense_device(torch.empty((333, 77), device="cuda", dtype=torch.float16), seed=11)
    torch.cuda.synchronize()
    assert np.array_equal(d32.cpu().numpy(), h)
    assert np.array_equal(d16.cpu().numpy(), h.astype(np.float16))


@pytest.mark.parametrize("n", [1, 40, 100, 128, 129, 300])
def test_band_plan_shapes(cuda, n):
    """BAND plan: partial last band, bands without entries, tiles at the last columns, N below the tile width."""
    rp, col, val = random_csr(n, n, min(1.0, 6.0 / n), seed=n, empty_rows=True)
    A = vm.CSR.from_arrays(n, n, rp, col, val)
    B = np.random.default_rng(n).uniform(-1, 1, size=(n, 128)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, False, 32, 128, b_half=True, plan=vm.PLAN_BAND)
    oracle_check(A, C, Bu, False)


@pytest.mark.parametrize("band_rows", [1, 37, 64, 126, 128])
@pytest.mark.parametrize("accumulate", [False, True], ids=["store", "accumulate"])
def test_band_plan_heights(cuda, band_rows, accumulate):
    """BAND plan at fixed band heights: tiles start at any column (greedy), rows past a band's
    height are never stored, C += A*B adds."""
    A = vm.CSR.generate(vm.GEN_STENCIL27, 12, seed=0)
    B = vm.gen_dense_host(A.N, 128, seed=3)
    base = np.random.default_rng(4).uniform(-1, 1, size=(A.M, 128)).astype(np.float32) if accumulate else None
    C, Bu = run_gpu(cuda, A, B, False, 32, 128, b_half=True, accumulate_into=base, plan=vm.PLAN_BAND,
                    band_rows=band_rows)
    oracle_check(A, C, Bu, False, base=None if base is None else base.astype(np.float64))


def test_band_plan_dense_tiles(cuda):
    """Tiles with more entries than the producers keep in registers (whole-tile clears)."""
    rp, col, val = random_csr(256, 96, 0.9, seed=8)
    A = vm.CSR.from_arrays(256, 96, rp, col, val)
    B = np.random.default_rng(8).uniform(-1, 1, size=(96, 200)).astype(np.float32)
    C, Bu = run_gpu(cuda, A, B, False, 32, 128, b_half=True, plan=vm.PLAN_BAND)
    oracle_check(A, C, Bu, False)


def test_band_plan_needs_fp16_format(cuda):
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 256, seed=1)
    with pytest.raises(vm.VcsrmcError) as e:
        vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=True, segw=32), plans=[vm.PLAN_BAND])
    assert e.value.status == 1 and "FP16" in str(e.value)


def test_auto_plan_prefers_band_when_resident(cuda):
    torch = cuda
    A = vm.CSR.generate(vm.GEN_STENCIL27, 16, seed=0)
    B32 = vm.gen_dense_host(A.N, 128, seed=2)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), plans=[vm.PLAN_BAND])
    B = torch.from_numpy(B32).cuda().half()
    C = torch.full((A.M, 128), 5.0, device="cuda")
    vm.spmm(dV, B, C, accumulate=False)  # AUTO -> BAND, the only resident layout
    torch.cuda.synchronize()
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    check_fp16(C.cpu().numpy(), ref, ab)
    assert dV.status() == 0
    with pytest.raises(vm.VcsrmcError):
        vm.spmm(dV, B, C, plan=vm.PLAN_ROWS)  # not uploaded
    dV.free()


def test_errors_are_status_codes(cuda):
    torch = cuda
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 256, seed=1)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=True, segw=32))
    B = torch.zeros((256, 64), device="cuda", dtype=torch.float16)
    C = torch.zeros((256, 64), device="cuda")
    with pytest.raises(vm.VcsrmcError) as e:
        vm.spmm(dV, B, C)  # fp16 B with the FP32 format
    assert e.value.status == 1
    with pytest.raises(vm.VcsrmcError):
        vm.spmm(dV, B.float(), C, tileK=48)
    dV.free()


def test_reference_style_timed_call(cuda):
    """run_vcsr_mc_spmm_gpu: blocking, event-timed, C += A*B on a caller-zeroed C (src/main.cpp:242-245)."""
    torch = cuda
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 4096, seed=0)
    B32 = vm.gen_dense_host(4096, 128, seed=0)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=True, segw=32))
    B = torch.from_numpy(B32).cuda()
    C = torch.zeros((4096, 128), device="cuda")
    ms = vm.run_vcsr_mc_spmm_gpu(dV, B, 128, 128, C)
    assert ms > 0.0
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, B32, with_abs=True)
    check_fp32(C.cpu().numpy(), ref, ab)
    dV.free()
