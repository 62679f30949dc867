"""ROWS plan hot columns (an opt-in upload option) on the GPU, through the C ABI.

The hot-column path reads the most used rows of B from a compact copy made by each call (up to a
copy budget), resolves the other ranked columns through a lookup, and can read unranked columns
with evict-first loads; the values multiplied and the order of the fused multiply-adds are those
of the plain path. So every row of C that one lane group computes
must be bit-identical with and without hot columns, on every variant of the rows kernel (fp16/fp32
B, fp16/fp32 format, 16-byte and element-wise loads, ragged and narrow widths, store and
accumulate), whether every ranked column is copied or only some of them (a copy budget below the
hot set). Rows longer than a work unit are split into chunks whose partial rows are added into C
with atomics in no fixed order, so those rows (the same in both runs) are compared within fp32
rounding instead. One case per B type is also checked against the fp64 oracle; uploads without the option have no hot columns.
"""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16, check_fp32

pytestmark = pytest.mark.gpu

_mats = {}
_units = {}


def same_rows(A, plain, hot, Bused):
    """Bit-identical rows, except rows split into atomically reduced chunks: those differ only in the
    order in which chunk sums are added (into C's initial values, |C| <= 1 in these tests), within
    1e-5 of sum_p |a_ip b_pj| (the fp64 oracle's) + 1."""
    rp, col, val = A.arrays()
    split = np.diff(rp) > _units[id(A)]
    assert np.array_equal(plain[~split].view(np.uint32), hot[~split].view(np.uint32))
    if split.any():
        rows = np.flatnonzero(split).astype(np.int32)
        _, absref = ob.spmm_fp64_rows(rp, col, val, Bused, rows, with_abs=True)
        diff = np.abs(plain[rows].astype(np.float64) - hot[rows].astype(np.float64))
        assert np.all(diff <= 1e-5 * (absref + 1.0))


def rmat(scale: int) -> vm.CSR:
    if scale not in _mats:
        _mats[scale] = vm.CSR.generate(vm.GEN_RMAT, scale, seed=1)
    return _mats[scale]


def spmm(torch, A, B32, fp32: bool, b_half: bool, O: int, hot_rows: int, budget_mib: int = 16, persist: int = 0,
         ldb_pad: int = 0, accumulate_into=None, device_build: bool = False, evict_first: int = 0):
    if device_build:
        rp, col, val = A.arrays()
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dt)
        dV = vm.build_vcsr_mc_device(t(rp, torch.int32), t(col, torch.int32), t(val, torch.float32), A.M, A.N,
                                     fp32=fp32, segw=32, plans=[vm.PLAN_ROWS], hot_rows=hot_rows,
                                     hot_budget_mib=budget_mib, hot_persist=persist, hot_evict_first=evict_first)
    else:
        V = vm.csr_to_vcsr_mc(A, fp32=fp32, segw=32)
        dV = vm.upload_vcsr_mc_device(V, device=0, plans=[vm.PLAN_ROWS], hot_rows=hot_rows,
                                      hot_budget_mib=budget_mib, hot_persist=persist, hot_evict_first=evict_first)
    dt = torch.float16 if b_half else torch.float32
    Bfull = torch.zeros((A.N, O + ldb_pad), dtype=dt, device="cuda")
    Bfull[:, :O] = torch.from_numpy(B32[:, :O]).to(device="cuda", dtype=dt)
    C = torch.full((A.M, O), 3.0, dtype=torch.float32, device="cuda")
    if accumulate_into is not None:
        C.copy_(torch.from_numpy(accumulate_into))
    vm.spmm(dV, Bfull, C, tileK=128, accumulate=accumulate_into is not None, O=O, plan=vm.PLAN_ROWS)
    if accumulate_into is None:  # a second overwrite reuses the handle's hot-row buffer
        vm.spmm(dV, Bfull, C, tileK=128, accumulate=False, O=O, plan=vm.PLAN_ROWS)
    torch.cuda.synchronize()
    assert dV.status() == 0
    info = dV.info()
    n_hot = info["n_hot"]
    _units[id(A)] = info["rows_unit_nnz"]
    out = C.cpu().numpy()
    Bused = Bfull[:, :O].float().cpu().numpy()
    dV.free()
    return out, Bused, n_hot


@pytest.mark.parametrize("kind", ["fp16", "fp16-formats-fp32-B", "fp32"])
@pytest.mark.parametrize("O", [128, 130, 256, 32, 64, 1])
@pytest.mark.parametrize("accumulate", [False, True], ids=["store", "accumulate"])
@pytest.mark.parametrize("mode", ["copy", "evict-first"])
def test_hot_path_is_bit_identical(cuda, kind, O, accumulate, mode):
    A = rmat(16)
    fp32, b_half = kind == "fp32", kind == "fp16"
    B = vm.gen_dense_host(A.N, O, seed=2)
    base = np.random.default_rng(4).uniform(-1, 1, size=(A.M, O)).astype(np.float32) if accumulate else None
    plain, Bu, n0 = spmm(cuda, A, B, fp32, b_half, O, hot_rows=0, accumulate_into=base)
    copy = mode == "copy"
    hot, _, n1 = spmm(cuda, A, B, fp32, b_half, O, hot_rows=4096, accumulate_into=base, budget_mib=16 if copy else 0,
                      evict_first=0 if copy else 1)
    assert n0 == 0 and n1 == 4096
    same_rows(A, plain, hot, Bu)


@pytest.mark.parametrize("budget_mib", [1, 2], ids=["1MiB", "2MiB"])
def test_copy_budget_below_the_hot_set(cuda, budget_mib):
    """Ranks past the copy budget are looked up: still bit-identical."""
    A = rmat(16)
    B = vm.gen_dense_host(A.N, 128, seed=5)
    plain, Bu, _ = spmm(cuda, A, B, False, True, 128, hot_rows=0)
    hot, _, n = spmm(cuda, A, B, False, True, 128, hot_rows=20000, budget_mib=budget_mib)
    assert n == 20000  # 20000 x 256 B = 4.9 MiB > budget
    same_rows(A, plain, hot, Bu)


def test_unaligned_b_rows(cuda):
    """B rows not 16-byte aligned (ldb = O + 1 halves): element-wise loads for B and for the copy."""
    A = rmat(15)
    B = vm.gen_dense_host(A.N, 128, seed=6)
    plain, Bu, _ = spmm(cuda, A, B, False, True, 128, hot_rows=0, ldb_pad=1)
    hot, _, n = spmm(cuda, A, B, False, True, 128, hot_rows=3000, ldb_pad=1)
    assert n == 3000
    same_rows(A, plain, hot, Bu)


def test_persisting_window(cuda):
    """The copy under a persisting L2 access-policy window changes caching only."""
    A = rmat(16)
    B = vm.gen_dense_host(A.N, 128, seed=7)
    plain, Bu, _ = spmm(cuda, A, B, False, True, 128, hot_rows=0)
    hot, _, n = spmm(cuda, A, B, False, True, 128, hot_rows=8192, persist=1)
    assert n == 8192
    same_rows(A, plain, hot, Bu)


def test_device_built_format_ranks_the_same_columns(cuda):
    A = rmat(16)
    B = vm.gen_dense_host(A.N, 128, seed=8)
    host, Bu, nh = spmm(cuda, A, B, False, True, 128, hot_rows=5000)
    dev, _, nd = spmm(cuda, A, B, False, True, 128, hot_rows=5000, device_build=True)
    assert nh == nd == 5000
    same_rows(A, host, dev, Bu)


@pytest.mark.parametrize("fp32", [False, True], ids=["fp16", "fp32"])
def test_hot_path_against_the_oracle(cuda, fp32):
    A = rmat(15)
    B = vm.gen_dense_host(A.N, 128, seed=9)
    C, Bu, n = spmm(cuda, A, B, fp32, not fp32, 128, hot_rows=2048)
    assert n == 2048
    rp, col, val = A.arrays()
    ref, ab = ob.spmm_fp64(rp, col, val, Bu, with_abs=True)
    (check_fp32 if fp32 else check_fp16)(C, ref, ab)


def test_no_hot_columns_by_default(cuda):
    A = rmat(14)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=False, segw=32), device=0)
    assert dV.info()["n_hot"] == 0
    dV.free()


def test_bad_hot_options(cuda):
    A = rmat(12)
    V = vm.csr_to_vcsr_mc(A, fp32=False, segw=32)
    for kw in ({"hot_rows": -1}, {"hot_budget_mib": -1}, {"hot_budget_mib": 5000}, {"hot_persist": 2},
               {"hot_persist": -1}, {"hot_evict_first": 2}):
        with pytest.raises(vm.VcsrmcError) as e:
            vm.upload_vcsr_mc_device(V, device=0, plans=[vm.PLAN_ROWS], **kw)
        assert e.value.status == 1, kw
