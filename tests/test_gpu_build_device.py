"""The GPU-side VCSR-MC builder (vcsrmc_build_device) against the oracle and the host builder.

The device builder orders rows with equal per-segment counts by ascending row, which is the
oracle's canonical build (oracle_build_vcsr), so every array must equal the oracle's bit for bit
(FP16 formats hold their values on the device rounded to fp16). Against the host builder, which
reproduces the reference's hash-map order, the tie-independent arrays are equal and the others
are equal after canonicalisation. SpMM on a device-built format is checked against the fp64
oracle on every plan.
"""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16, check_fp32, random_csr

pytestmark = pytest.mark.gpu

TIE_FREE = ("group_ptr", "group_depth", "group_seg_base", "item_gbeg", "item_gend")


def matrices():
    yield "c1", vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 4096, seed=0)
    yield "zipf", vm.CSR.generate(vm.GEN_ZIPF, 1 << 14, seed=1)
    yield "stencil", vm.CSR.generate(vm.GEN_STENCIL27, 12, seed=0)
    yield "rmat", vm.CSR.generate(vm.GEN_RMAT, 12, seed=2)
    rp, col, val = random_csr(300, 500, 0.03, seed=4, empty_rows=True)
    yield "empty_rows", vm.CSR.from_arrays(300, 500, rp, col, val)


MATS = dict(matrices())


def device_build(torch, A: vm.CSR, fp32: bool, segw: int, **kw) -> vm.DeviceVCSRMC:
    rp, col, val = A.arrays()
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dt)
    return vm.build_vcsr_mc_device(t(rp, torch.int32), t(col, torch.int32), t(val, torch.float32), A.M, A.N,
                                   fp32=fp32, segw=segw, **kw)


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("segw", [16, 32, 48, 64])
@pytest.mark.parametrize("name", list(MATS))
def test_device_build_equals_oracle(cuda, name, segw, fp32):
    A = MATS[name]
    rp, col, val = A.arrays()
    ref = ob.build_vcsr(A.M, A.N, rp, col, val, fp32, segw)
    dV = device_build(cuda, A, fp32, segw)
    got = dV.download().arrays()
    for k in ("group_ptr", "group_depth", "group_seg_base", "group_rows", "lcol", "item_gbeg", "item_gend"):
        assert np.array_equal(got[k], ref[k]), k
    want_val = ref["val"] if fp32 else ref["val"].astype(np.float16).astype(np.float32)
    assert np.array_equal(got["val"], want_val)
    assert dV.scale == ref["scale"]
    dV.free()


@pytest.mark.parametrize("segw", [16, 32])
@pytest.mark.parametrize("name", ["c1", "zipf", "rmat"])
def test_device_build_vs_host_builder(cuda, name, segw):
    A = MATS[name]
    host = vm.csr_to_vcsr_mc(A, fp32=True, segw=segw).arrays()
    host["segw"] = segw
    dV = device_build(cuda, A, True, segw)
    got = dV.download().arrays()
    for k in TIE_FREE:
        assert np.array_equal(got[k], host[k]), k
    canon = ob.canonicalize(host)
    for k in ("group_rows", "lcol", "val"):
        assert np.array_equal(got[k], canon[k]), k
    dV.free()


@pytest.mark.parametrize("fp32", [True, False], ids=["fp32", "fp16"])
@pytest.mark.parametrize("plan", [vm.PLAN_SEGMENT, vm.PLAN_ROWS, vm.PLAN_BAND], ids=["segment", "rows", "band"])
@pytest.mark.parametrize("name", ["zipf", "stencil", "empty_rows"])
def test_spmm_on_device_built_format(cuda, name, plan, fp32):
    if plan == vm.PLAN_BAND and fp32:
        pytest.skip("the BAND plan runs on the tensor cores: FP16 format only")
    torch = cuda
    A = MATS[name]
    dV = device_build(torch, A, fp32, 32, plans=[plan], rows_unit_nnz=64 if name == "zipf" else 0)
    assert dV.info()["plans"] == [plan]
    B32 = vm.gen_dense_host(A.N, 128, seed=9)
    B = torch.from_numpy(B32).cuda()
    if not fp32:
        B = B.half()
    C = torch.full((A.M, 128), 3.0, device="cuda")
    vm.spmm(dV, B, C, accumulate=False, plan=plan)
    torch.cuda.synchronize()
    assert dV.status() == 0
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    (check_fp32 if fp32 else check_fp16)(C.cpu().numpy(), ref, ab)
    dV.free()


@pytest.mark.parametrize("name", ["c1", "zipf", "rmat", "empty_rows"])
def test_device_build_rows_units_match_host(cuda, name):
    """The ROWS layout's work units follow the same packing whichever builder made the format."""
    A = MATS[name]
    a = device_build(cuda, A, False, 32, plans=[vm.PLAN_ROWS]).info()
    b = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), plans=[vm.PLAN_ROWS]).info()
    for k in ("n_units", "rows_unit_nnz", "n_split_rows"):
        assert a[k] == b[k], k


BAND_CASES = [("c1", 0), ("zipf", 0), ("stencil", 0), ("stencil", 37), ("stencil", 1), ("rmat", 64),
              ("rmat", 0), ("empty_rows", 0), ("empty_rows", 128)]


@pytest.mark.parametrize("name,H", BAND_CASES, ids=[f"{n}-H{h}" for n, h in BAND_CASES])
def test_device_band_view_equals_host(cuda, name, H):
    """The BAND view built on the device (segmented sort, one warp per band cutting the greedy
    tiles) is the host-built view: same band height (chosen from the same sampled bands when H is
    0), same band and tile counts, and bit-identical SpMM results, which needs the same tiles with
    their entries in the same order."""
    torch = cuda
    A = MATS[name]
    a = device_build(torch, A, False, 32, plans=[vm.PLAN_BAND], band_rows=H)
    b = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), plans=[vm.PLAN_BAND], band_rows=H)
    ia, ib = a.info(), b.info()
    for k in ("band_rows", "n_bands", "n_tiles"):
        assert ia[k] == ib[k], k
    assert a.scale == b.scale
    B = torch.from_numpy(vm.gen_dense_host(A.N, 96, seed=5)).cuda().half()
    Ca = torch.full((A.M, 96), float("nan"), device="cuda")
    Cb = torch.full((A.M, 96), float("nan"), device="cuda")
    vm.spmm(a, B, Ca, accumulate=False, plan=vm.PLAN_BAND)
    vm.spmm(b, B, Cb, accumulate=False, plan=vm.PLAN_BAND)
    torch.cuda.synchronize()
    assert a.status() == 0 and b.status() == 0
    assert torch.equal(Ca, Cb)
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, B.float().cpu().numpy(), with_abs=True)
    check_fp16(Ca.cpu().numpy(), ref, ab)
    a.free()
    b.free()


@pytest.mark.parametrize("name", ["stencil", "zipf", "c1"])
def test_device_build_default_plans_follow_upload(cuda, name):
    """With the default plans the device builder adds BAND exactly where an upload does."""
    A = MATS[name]
    a = device_build(cuda, A, False, 32).info()
    b = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32)).info()
    assert a["plans"] == b["plans"]
    assert (vm.PLAN_BAND in a["plans"]) == (name == "stencil")
    if vm.PLAN_BAND in a["plans"]:
        assert a["band_rows"] == b["band_rows"] and a["n_tiles"] == b["n_tiles"]
    assert vm.PLAN_BAND not in device_build(cuda, A, True, 32).info()["plans"]


def test_device_build_half_scale(cuda):
    rp, col, val = random_csr(64, 96, 0.1, seed=4, scale=1e6)
    A = vm.CSR.from_arrays(64, 96, rp, col, val)
    dV = device_build(cuda, A, False, 32)
    assert dV.scale == vm.half_scale(A) != 1.0
    dV.free()


def test_device_build_empty(cuda):
    A = vm.CSR.from_arrays(10, 20, np.zeros(11, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32))
    dV = device_build(cuda, A, False, 16)
    info = dV.info()
    assert info["n_groups"] == 0 and info["n_items"] == 0
    C = cuda.full((10, 64), 1.0, device="cuda")
    vm.spmm(dV, cuda.zeros((20, 64), device="cuda", dtype=cuda.float16), C, accumulate=False)
    assert float(C.abs().max()) == 0.0
    dV.free()


def test_device_build_rejects_unsorted_rows_and_bad_row_ptr(cuda):
    torch = cuda
    rp = torch.tensor([0, 2, 3], dtype=torch.int32, device="cuda")
    col = torch.tensor([5, 1, 0], dtype=torch.int32, device="cuda")  # row 0 not ascending
    val = torch.ones(3, dtype=torch.float32, device="cuda")
    with pytest.raises(vm.VcsrmcError) as e:
        vm.build_vcsr_mc_device(rp, col, val, 2, 8)
    assert e.value.status == 1
    bad_rp = torch.tensor([0, 3, 2], dtype=torch.int32, device="cuda")
    with pytest.raises(vm.VcsrmcError) as e:
        vm.build_vcsr_mc_device(bad_rp, torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda"), val, 2, 8)
    assert e.value.status == 1
    with pytest.raises(vm.VcsrmcError) as e:
        vm.build_vcsr_mc_device(rp, torch.tensor([0, 1, 9], dtype=torch.int32, device="cuda"), val, 2, 8)  # col >= N
    assert e.value.status == 1


def test_device_build_rejects_bad_band_requests(cuda):
    """BAND needs the FP16 format and a band height in [0, 128]; both are argument errors,
    reported before any device work."""
    torch = cuda
    rp = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    col = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    val = torch.ones(2, dtype=torch.float32, device="cuda")
    with pytest.raises(vm.VcsrmcError) as e:
        vm.build_vcsr_mc_device(rp, col, val, 2, 8, fp32=True, plans=[vm.PLAN_BAND])
    assert e.value.status == 1 and "FP16" in str(e.value)
    for H in (-1, 129):
        with pytest.raises(vm.VcsrmcError) as e:
            vm.build_vcsr_mc_device(rp, col, val, 2, 8, plans=[vm.PLAN_BAND], band_rows=H)
        assert e.value.status == 1
    dV = vm.build_vcsr_mc_device(rp, col, val, 2, 8, plans=[vm.PLAN_BAND], band_rows=1)
    info = dV.info()
    assert info["plans"] == [vm.PLAN_BAND] and info["band_rows"] == 1 and info["n_bands"] == 2
    assert info["n_tiles"] == 2 and info["band_cols"] in (32, 64)
    dV.free()
