"""Parity at the benchmark configurations' full sizes (configs 1-4), through properties that do
not depend on size:

  * sampled rows: 2000 rows (random, plus the first, the last and the longest) compared element by
    element with the fp64 oracle (oracle_spmm_fp64_rows, the reference's CPU loop src/main.cpp:202-207
    restated), under the tolerances of tests/helpers.py;
  * checksums over every row: C x == A (B x) in fp64 for x = ones and two random vectors, within
    1e-4 of |A| (|B| |x|) (fp32 accumulation error; the reference side uses the A values the GPU
    multiplies, i.e. rounded to fp16 on the FP16 path).

Config 4 (R-MAT 2^24, 263 M nnz) runs on a GPU-built format (vcsrmc_build_device; FP16 and FP32,
every plan) and on a host-built one (the builder that is bit-identical to the reference's), and
config 5's wide widths (O = 256, 512) run on the config-2 matrix with and without RCM.
"""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob
from tests.helpers import check_fp16, check_fp32

pytestmark = pytest.mark.gpu

CONFIGS = {"c1": (vm.GEN_UNIFORM_POISSON, 4096), "c2": (vm.GEN_ZIPF, 262144), "c3": (vm.GEN_STENCIL27, 100),
           "c4": (vm.GEN_RMAT, 24)}
_cache = {}


def matrix(name):
    if name not in _cache:
        _cache.clear()  # one full-size matrix in host memory at a time
        kind, param = CONFIGS[name]
        _cache[name] = vm.CSR.generate(kind, param, seed=0)
    return _cache[name]


def sampled_rows(rp, M, rng):
    lengths = np.diff(rp)
    rows = np.concatenate([rng.choice(M, size=min(M, 2000), replace=False), [0, M - 1, int(np.argmax(lengths))]])
    return np.unique(rows).astype(np.int64)


def check_sampled_rows(torch, rp, col, val, B, C, rows, fp32):
    starts, ends = rp[rows].astype(np.int64), rp[rows + 1].astype(np.int64)
    lens = ends - starts
    sub_rp = np.zeros(rows.size + 1, np.int64)
    np.cumsum(lens, out=sub_rp[1:])
    idx = np.repeat(starts - sub_rp[:-1], lens) + np.arange(sub_rp[-1])
    cols = col[idx]
    uniq, remap = np.unique(cols, return_inverse=True)
    Bsub = B[torch.from_numpy(uniq.astype(np.int64)).cuda()].float().cpu().numpy()
    ref, ab = ob.spmm_fp64_rows(sub_rp.astype(np.int32), remap.astype(np.int32), val[idx], Bsub,
                                np.arange(rows.size, dtype=np.int32), with_abs=True)
    got = C[torch.from_numpy(rows).cuda()].cpu().numpy()
    (check_fp32 if fp32 else check_fp16)(got, ref, ab)


def check_checksums(torch, rp, col, val, B, C, fp32, scale, seed):
    M, O = C.shape
    a = val.astype(np.float64)
    if not fp32:  # the values the tensor/FMA units multiply
        a = (val / np.float32(scale)).astype(np.float16).astype(np.float64) * scale
    row_ids = np.repeat(np.arange(M, dtype=np.int32), np.diff(rp))
    rng = np.random.default_rng(seed)
    for x in (np.ones(O), rng.uniform(-1, 1, O), rng.standard_normal(O)):
        xd = torch.from_numpy(x).cuda()
        step = 1 << 20
        t = torch.cat([B[i:i + step].double() @ xd for i in range(0, B.shape[0], step)]).cpu().numpy()
        tb = torch.cat([B[i:i + step].double().abs() @ xd.abs() for i in range(0, B.shape[0], step)]).cpu().numpy()
        y = torch.cat([C[i:i + step].double() @ xd for i in range(0, M, step)]).cpu().numpy()
        ref = np.bincount(row_ids, weights=a * t[col], minlength=M)
        bound = np.bincount(row_ids, weights=np.abs(a) * tb[col], minlength=M)
        err = np.abs(y - ref)
        worst = float(np.max(err - 1e-4 * bound - 1e-9))
        assert np.all(np.isfinite(y)) and worst <= 0.0, f"checksum exceeds its bound by {worst:.3e}"


# (config, FP32 format, plan, where the format is built, hot-column upload options)
HOT = {"hot_rows": 393216, "hot_budget_mib": 96}
CASES = [("c1", False, vm.PLAN_AUTO, "host", None), ("c1", True, vm.PLAN_AUTO, "host", None),
         ("c2", False, vm.PLAN_AUTO, "host", None), ("c2", True, vm.PLAN_AUTO, "host", None),
         ("c3", False, vm.PLAN_AUTO, "host", None), ("c3", False, vm.PLAN_ROWS, "host", None),
         ("c3", False, vm.PLAN_SEGMENT, "host", None), ("c3", True, vm.PLAN_AUTO, "host", None),
         ("c4", False, vm.PLAN_AUTO, "device", None), ("c4", False, vm.PLAN_ROWS, "device", None),
         ("c4", False, vm.PLAN_SEGMENT, "device", None), ("c4", True, vm.PLAN_AUTO, "device", None),
         ("c4", True, vm.PLAN_ROWS, "device", None), ("c4", True, vm.PLAN_SEGMENT, "device", None),
         ("c4", False, vm.PLAN_ROWS, "host", None), ("c4", False, vm.PLAN_ROWS, "device", HOT)]
PLAN_NAMES = {0: "auto", 1: "segment", 2: "rows", 3: "band"}


@pytest.mark.parametrize("name,fp32,plan,build,hot", CASES,
                         ids=[f"{n}-{'fp32' if f else 'fp16'}-{PLAN_NAMES[p]}-{b}{'-hot' if h else ''}"
                              for n, f, p, b, h in CASES])
def test_full_size(cuda, name, fp32, plan, build, hot):
    """Configs 1-4 at full size; config 4 on a GPU-built format (FP16 and FP32, every plan), on a
    host-built one (bit-identical to the reference builder), and with hot columns."""
    torch = cuda
    A = matrix(name)
    rp, col, val = A.arrays(copy=False)
    if build == "device":
        t = lambda x: torch.from_numpy(np.asarray(x)).cuda()
        dV = vm.build_vcsr_mc_device(t(rp), t(col), t(val), A.M, A.N, fp32=fp32, segw=32, **(hot or {}))
    else:
        dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=fp32, segw=32), device=0, **(hot or {}))
    if name == "c3" and not fp32 and plan == vm.PLAN_AUTO:
        assert vm.PLAN_BAND in dV.info()["plans"]  # the default layouts add BAND on the stencil
    if hot:
        assert dV.info()["n_hot"] == hot["hot_rows"]
    B = torch.empty((A.N, 128), dtype=torch.float32 if fp32 else torch.float16, device="cuda")
    vm.gen_dense_device(B, seed=11)
    C = torch.full((A.M, 128), float("nan"), device="cuda")
    vm.spmm(dV, B, C, accumulate=False, plan=plan)
    torch.cuda.synchronize()
    assert dV.status() == 0
    check_sampled_rows(torch, rp, col, val, B, C, sampled_rows(rp, A.M, np.random.default_rng(3)), fp32)
    check_checksums(torch, rp, col, val, B, C, fp32, dV.scale, seed=4)
    dV.free()
    del B, C
    torch.cuda.empty_cache()


# Config 5: the config-2 matrix at the sweep's wide dense widths, both segment widths, with and without
# the reference's RCM column permutation (include/reorder.hpp), on the ROWS plan and on the SEGMENT
# plan at tileK 128 and 256 (the format does not depend on tileK; tileK 256 is new, the reference
# stops at 128).
_c5 = {}


def c5_problem(rcm: bool, O: int):
    key = (rcm, O)
    if key not in _c5:
        _c5.clear()
        A = vm.CSR.generate(vm.GEN_ZIPF, 262144, seed=0)
        B = vm.gen_dense_host(A.N, O, seed=21)
        if rcm:
            B = vm.apply_column_permutation(A, B, vm.rcm_column_order(A))
        _c5[key] = (A, B)
    return _c5[key]


C5 = [(O, fp32, segw, rcm, plan, tk) for O in (256, 512) for rcm in (False, True) for fp32 in (False, True)
      for segw in (16, 32) for plan, tk in ((vm.PLAN_ROWS, 128), (vm.PLAN_SEGMENT, 128), (vm.PLAN_SEGMENT, 256))]


@pytest.mark.parametrize("O,fp32,segw,rcm,plan,tileK", C5,
                         ids=[f"O{o}-{'fp32' if f else 'fp16'}-s{w}-{'rcm' if r else 'natural'}-{PLAN_NAMES[p]}-tk{t}"
                              for o, f, w, r, p, t in C5])
def test_config5_wide(cuda, O, fp32, segw, rcm, plan, tileK):
    torch = cuda
    A, B32 = c5_problem(rcm, O)
    rp, col, val = A.arrays(copy=False)
    dV = vm.upload_vcsr_mc_device(vm.csr_to_vcsr_mc(A, fp32=fp32, segw=segw), device=0, plans=[plan])
    B = torch.from_numpy(B32).to(device="cuda", dtype=torch.float32 if fp32 else torch.float16)
    C = torch.full((A.M, O), float("nan"), device="cuda")
    vm.spmm(dV, B, C, tileK=tileK, accumulate=False, plan=plan)
    torch.cuda.synchronize()
    assert dV.status() == 0
    check_sampled_rows(torch, rp, col, val, B, C, sampled_rows(rp, A.M, np.random.default_rng(5)), fp32)
    check_checksums(torch, rp, col, val, B, C, fp32, dV.scale, seed=6)
    dV.free()
