"""Pins the oracle (oracle/oracle.c, the C restatement) against the reference itself.

Two independent pins:
  * tests/golden/golden.npz — outputs of the reference implementation compiled from its own
    sources (written by tests/golden/make_golden.py); always available.
  * oracle/_ref/libvcsr_ref.so — the reference's host code, called live on larger, seeded
    inputs; those tests skip where it was not built.
The oracle orders rows with equal per-segment counts by ascending row id, so tie-dependent arrays
(group_rows, lcol, val) are compared after canonicalising the reference's output; everything
else is compared bit for bit.
"""
import os

import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
TIE_FREE = ("group_ptr", "group_depth", "group_seg_base", "item_gbeg", "item_gend")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def golden_cases(g):
    return sorted({k.split("/")[0] for k in g.files})


def golden_csr(g, name):
    M, N = (int(x) for x in g[f"{name}/shape"])
    return M, N, g[f"{name}/row_ptr"], g[f"{name}/col"], g[f"{name}/val"]


def golden_vcsr(g, name, segw, fp32):
    pre = f"{name}/vcsr_s{segw}_f{fp32}/"
    d = {k: g[pre + k] for k in ob.VCSR_ARRAYS}
    d["segw"] = segw
    return d


def test_golden_has_cases(golden):
    assert len(golden_cases(golden)) >= 7


@pytest.mark.parametrize("segw", [16, 32, 48, 64])
@pytest.mark.parametrize("fp32", [0, 1])
def test_oracle_builder_vs_golden(golden, segw, fp32):
    for name in golden_cases(golden):
        M, N, rp, col, val = golden_csr(golden, name)
        ref = golden_vcsr(golden, name, segw, fp32)
        mine = ob.build_vcsr(M, N, rp, col, val, bool(fp32), segw)
        for k in TIE_FREE:
            assert np.array_equal(mine[k], ref[k]), (name, k)
        canon = ob.canonicalize(ref)
        for k in ("group_rows", "lcol", "val"):
            assert np.array_equal(mine[k], canon[k]), (name, k)
        meta = golden[f"{name}/vcsr_s{segw}_f{fp32}/meta"]
        assert mine["num_segments"] == int(meta[0]) and mine["bundle"] == int(meta[1])
        assert np.float32(mine["scale"]) == np.float32(meta[2])


def test_oracle_half_scale_vs_golden(golden):
    for name in golden_cases(golden):
        val = golden[f"{name}/val"]
        assert np.float32(ob.half_scale(val)) == golden[f"{name}/half_scale"][0], name
    # the triggers exist in the fixture set
    assert golden["large_values/half_scale"][0] != 1.0
    assert golden["tiny_values/half_scale"][0] != 1.0


def test_oracle_spmm_vs_golden(golden):
    """Same summation order as the reference loop, so the fp64 results are identical."""
    for name in golden_cases(golden):
        M, N, rp, col, val = golden_csr(golden, name)
        out = ob.spmm_fp64(rp, col, val, golden[f"{name}/B"], nthreads=2)
        assert np.array_equal(out, golden[f"{name}/spmm_fp64"]), name


def test_oracle_rcm_vs_golden(golden):
    """Cases whose neighbour lists are short enough that the reference's sort is stable."""
    for name in ("stencil2d_20", "uniform_300"):
        M, N, rp, col, val = golden_csr(golden, name)
        assert np.array_equal(ob.rcm_column_order(M, N, rp, col), golden[f"{name}/rcm"]), name


def test_oracle_apply_permutation_semantics(golden):
    M, N, rp, col, val = golden_csr(golden, "stencil2d_20")
    pos = golden["stencil2d_20/rcm"]
    B = golden["stencil2d_20/B"]
    c2, v2, B2 = ob.apply_column_permutation(M, N, rp, col, val, B, pos)
    # C is unchanged by the permutation (A P)(P^T B) = A B
    assert np.allclose(ob.spmm_fp64(rp, c2, v2, B2), golden["stencil2d_20/spmm_fp64"], rtol=0, atol=1e-12)
    for r in range(M):
        assert np.all(np.diff(c2[rp[r]:rp[r + 1]]) > 0)


def test_canonicalize_is_idempotent_and_a_row_permutation(golden):
    ref = golden_vcsr(golden, "zipf_512", 32, 0)
    ref.update(segw=32)
    c1 = ob.canonicalize(ref)
    c2 = ob.canonicalize(c1)
    for k in ob.VCSR_ARRAYS:
        assert np.array_equal(c1[k], c2[k])
    # same multiset of (row, lcol, val) triples
    def triples(f):
        out = []
        gp, gd, gr = f["group_ptr"], f["group_depth"], f["group_rows"]
        for g in range(gd.size):
            for lane in range(16):
                row = gr[g * 16 + lane]
                for d in range(gd[g]):
                    s = gp[g] + d * 16 + lane
                    if f["lcol"][s] >= 0:
                        out.append((row, g, f["lcol"][s], f["val"][s]))
        return sorted((r, lc, v) for r, _, lc, v in out)
    assert triples(ref) == triples(c1)


# ---- live reference (skips where oracle/_ref was not built) ------------------------------------
needs_ref = pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built here")


@needs_ref
@pytest.mark.parametrize("kind,param", [(vm.GEN_UNIFORM_POISSON, 4096), (vm.GEN_ZIPF, 1 << 15),
                                        (vm.GEN_STENCIL27, 20), (vm.GEN_RMAT, 13)])
@pytest.mark.parametrize("segw", [16, 32])
def test_oracle_builder_vs_live_reference(kind, param, segw):
    A = vm.CSR.generate(kind, param, seed=3)
    rp, col, val = A.arrays()
    for fp32 in (False, True):
        ref = ob.ref_build_vcsr(A.M, A.N, rp, col, val, fp32, segw)
        mine = ob.build_vcsr(A.M, A.N, rp, col, val, fp32, segw)
        for k in TIE_FREE:
            assert np.array_equal(mine[k], ref[k]), k
        canon = ob.canonicalize(ref)
        for k in ("group_rows", "lcol", "val"):
            assert np.array_equal(mine[k], canon[k]), k


@needs_ref
def test_oracle_spmm_vs_live_reference_loop():
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 14, seed=5)
    rp, col, val = A.arrays()
    B = vm.gen_dense_host(A.N, 32, seed=5)
    ref = np.empty((A.M, 32), dtype=np.float64)
    runner = ob.RefSpmm(rp, col, val, B, nslices=4)
    runner.run(ref)
    runner.close()
    assert np.array_equal(ob.spmm_fp64(rp, col, val, B, nthreads=4), ref)
