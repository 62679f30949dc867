"""Host library (libvcsrmc.so, no GPU needed) against the reference and the golden vectors.

The product's host code must reproduce the reference bit for bit: the VCSR-MC builder
(src/vcsr_mc.cu:25-123, including the order of rows with equal counts), the Matrix Market
reader and COO->CSR (include/mmio.hpp:19-75, include/csr.hpp:16-41), RCM
(include/reorder.hpp:17-108) and half_scale.
"""
import os
import re

import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden", "golden.npz")
needs_ref = pytest.mark.skipif(not ob.ref_available(), reason="oracle/_ref not built here")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def names(g):
    return sorted({k.split("/")[0] for k in g.files})


# ---- C ABI -----------------------------------------------------------------------------------
def test_library_exports_every_declared_symbol():
    """Every function declared in include/vcsrmc.h is exported by libvcsrmc.so (no GPU call)."""
    header = open(os.path.join(ROOT, "include", "vcsrmc.h")).read()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    declared = set(re.findall(r"\b(vcsrmc_[a-z0-9_]+)\s*\(", header))
    assert len(declared) >= 25
    lib = vm.lib()
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared) == set(vm._lib.PROTOTYPES), "binding prototypes out of sync with the header"


def test_status_codes_and_messages():
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 64, seed=1)
    with pytest.raises(vm.VcsrmcError) as e:
        vm.csr_to_vcsr_mc(A, segw=20)
    assert e.value.status == 1 and "segw" in str(e.value)
    with pytest.raises(vm.VcsrmcError) as e:
        vm.read_matrix_market("/nonexistent/file.mtx")
    assert e.value.status == 5
    # upload options are checked before any device work
    import ctypes
    V = vm.csr_to_vcsr_mc(A, segw=32)
    for bad in (8, 48, 2048):
        opts = vm._lib.UploadOptions()
        opts.rows_unit_nnz = bad
        with pytest.raises(vm.VcsrmcError) as e:
            vm._lib.call("vcsrmc_upload_opts", V.handle, 0, ctypes.byref(opts), None, ctypes.byref(ctypes.c_void_p()))
        assert e.value.status == 1 and "rows_unit_nnz" in str(e.value)


# ---- builder ---------------------------------------------------------------------------------
@pytest.mark.parametrize("segw", [16, 32, 48, 64])
def test_builder_vs_golden_bit_exact(golden, segw):
    for name in names(golden):
        M, N = (int(x) for x in golden[f"{name}/shape"])
        A = vm.CSR.from_arrays(M, N, golden[f"{name}/row_ptr"], golden[f"{name}/col"], golden[f"{name}/val"])
        for fp32 in (0, 1):
            V = vm.csr_to_vcsr_mc(A, fp32=bool(fp32), segw=segw)
            for k in ob.VCSR_ARRAYS:
                assert np.array_equal(V.array(k), golden[f"{name}/vcsr_s{segw}_f{fp32}/{k}"]), (name, k)
            meta = golden[f"{name}/vcsr_s{segw}_f{fp32}/meta"]
            assert V.num_segments == int(meta[0]) and V.bundle == int(meta[1])
            assert np.float32(V.scale) == np.float32(meta[2])


@needs_ref
@pytest.mark.parametrize("kind,param", [(vm.GEN_UNIFORM_POISSON, 4096), (vm.GEN_ZIPF, 1 << 16),
                                        (vm.GEN_STENCIL27, 24), (vm.GEN_RMAT, 15)])
def test_builder_vs_live_reference_bit_exact(kind, param):
    A = vm.CSR.generate(kind, param, seed=11)
    rp, col, val = A.arrays()
    for segw in (16, 32):
        for fp32 in (False, True):
            ref = ob.ref_build_vcsr(A.M, A.N, rp, col, val, fp32, segw)
            V = vm.csr_to_vcsr_mc(A, fp32=fp32, segw=segw)
            for k in ob.VCSR_ARRAYS:
                assert np.array_equal(V.array(k), ref[k]), (segw, fp32, k)


def test_builder_independent_of_thread_count():
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 14, seed=2)
    a = vm.csr_to_vcsr_mc(A, segw=32, nthreads=1).arrays()
    b = vm.csr_to_vcsr_mc(A, segw=32, nthreads=7).arrays()
    for k in a:
        assert np.array_equal(a[k], b[k]), k


@needs_ref
def test_builder_unsorted_and_duplicate_columns_match_reference():
    """CSR given as arrays may have unsorted rows and repeated columns; the builder then sorts each
    (segment, row) run exactly as the reference does."""
    rng = np.random.default_rng(8)
    M, N = 60, 90
    lens = rng.integers(0, 12, size=M)
    rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    col = rng.integers(0, N, size=rp[-1]).astype(np.int32)  # unsorted, may repeat
    val = rng.uniform(-1, 1, size=rp[-1]).astype(np.float32)
    A = vm.CSR.from_arrays(M, N, rp, col, val)
    for segw in (16, 32):
        ref = ob.ref_build_vcsr(M, N, rp, col, val, False, segw)
        V = vm.csr_to_vcsr_mc(A, segw=segw)
        for k in ob.VCSR_ARRAYS:
            assert np.array_equal(V.array(k), ref[k]), k


def test_half_scale_vs_golden(golden):
    for name in names(golden):
        M, N = (int(x) for x in golden[f"{name}/shape"])
        A = vm.CSR.from_arrays(M, N, golden[f"{name}/row_ptr"], golden[f"{name}/col"], golden[f"{name}/val"])
        assert np.float32(vm.half_scale(A)) == golden[f"{name}/half_scale"][0]


def test_empty_matrix_format():
    A = vm.CSR.from_arrays(3, 5, np.zeros(4, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32))
    V = vm.csr_to_vcsr_mc(A, segw=16)
    assert V.n_groups == 0 and V.n_items == 0 and list(V.array("group_ptr")) == [0]


# ---- RCM ---------------------------------------------------------------------------------------
def test_rcm_vs_golden(golden):
    for name in names(golden):
        if f"{name}/rcm" not in golden.files:
            continue
        M, N = (int(x) for x in golden[f"{name}/shape"])
        A = vm.CSR.from_arrays(M, N, golden[f"{name}/row_ptr"], golden[f"{name}/col"], golden[f"{name}/val"])
        assert np.array_equal(vm.rcm_column_order(A), golden[f"{name}/rcm"]), name


@needs_ref
@pytest.mark.parametrize("kind,param", [(vm.GEN_ZIPF, 1 << 13), (vm.GEN_RMAT, 12), (vm.GEN_STENCIL27, 12)])
def test_rcm_and_permutation_vs_live_reference(kind, param):
    """Includes high-degree vertices, where the reference's unstable neighbour sort matters."""
    A = vm.CSR.generate(kind, param, seed=4)
    rp, col, val = A.arrays()
    pos = vm.rcm_column_order(A)
    assert np.array_equal(pos, ob.ref_rcm_column_order(A.M, A.N, rp, col))
    B = vm.gen_dense_host(A.N, 8, seed=4)
    B2 = vm.apply_column_permutation(A, B, pos)
    c_ref, v_ref, B_ref = ob.ref_apply_column_permutation(A.M, A.N, rp, col, val, B, pos)
    rp2, col2, val2 = A.arrays()
    assert np.array_equal(col2, c_ref) and np.array_equal(val2, v_ref) and np.array_equal(B2, B_ref)


def test_apply_permutation_rejects_non_permutation():
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, 32, seed=1)
    with pytest.raises(vm.VcsrmcError):
        vm.apply_column_permutation(A, None, np.zeros(32, np.int32))


# ---- Matrix Market reader + COO->CSR ------------------------------------------------------------
MTX_CASES = {
    "general_real": "%%MatrixMarket matrix coordinate real general\n% c\n3 4 4\n1 1 1.5\n3 4 -2e1\n2 2 .25\n1 3 7\n",
    "symmetric": "%%MatrixMarket matrix coordinate real symmetric\n3 3 3\n1 1 2\n2 1 -1\n3 2 4.5\n",
    "skew": "%%MatrixMarket matrix coordinate real skew-symmetric\n3 3 2\n2 1 3\n3 1 -1\n",
    "pattern": "%%MatrixMarket matrix coordinate pattern general\n2 3 3\n1 2\n2 1\n2 3\n",
    "integer": "%%MatrixMarket matrix coordinate integer symmetric\n2 2 2\n1 1 5\n2 1 -3\n",
    "blank_lines": "%%MatrixMarket matrix coordinate real general\n\n%x\n2 2 1\n\n2 2 1.0\n\n",
    # malformed
    "bad_banner": "%%MatrixMarket matrix array real general\n2 2\n1\n2\n3\n4\n",
    "bad_field": "%%MatrixMarket matrix coordinate complex general\n1 1 1\n1 1 1 0\n",
    "truncated": "%%MatrixMarket matrix coordinate real general\n2 2 3\n1 1 1\n2 2 2\n",
    "extra": "%%MatrixMarket matrix coordinate real general\n2 2 1\n1 1 1\n2 2 2\n",
    "extra_field": "%%MatrixMarket matrix coordinate pattern general\n2 2 1\n1 1 9\n",
    "out_of_range": "%%MatrixMarket matrix coordinate real general\n2 2 1\n3 1 1\n",
    "zero_based": "%%MatrixMarket matrix coordinate real general\n2 2 1\n0 1 1\n",
    "duplicate": "%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1\n1 1 2\n",
    "sym_not_square": "%%MatrixMarket matrix coordinate real symmetric\n2 3 1\n1 1 1\n",
    "skew_diag": "%%MatrixMarket matrix coordinate real skew-symmetric\n2 2 1\n1 1 1\n",
    "not_finite": "%%MatrixMarket matrix coordinate real general\n1 1 1\n1 1 1e40\n",
    "bad_entry": "%%MatrixMarket matrix coordinate real general\n1 1 1\n1 x 1\n",
}


@pytest.mark.parametrize("case", sorted(MTX_CASES))
def test_mtx_reader_matches_reference(tmp_path, case):
    path = str(tmp_path / f"{case}.mtx")
    with open(path, "w") as f:
        f.write(MTX_CASES[case])
    try:
        A = vm.read_matrix_market(path)
        mine = (A.M, A.N) + tuple(A.arrays())
        err = None
    except vm.VcsrmcError as e:
        mine, err = None, e
    if ob.ref_available():
        try:
            ref = ob.ref_read_mtx(path)
        except ob.RefError:
            ref = None
        assert (mine is None) == (ref is None), (case, err)
        if ref is not None:
            assert mine[:2] == ref[:2]
            for a, b in zip(mine[2:], ref[2:]):
                assert np.array_equal(a, b), case
    expect_ok = case in ("general_real", "symmetric", "skew", "pattern", "integer", "blank_lines")
    assert (mine is not None) == expect_ok, (case, err)
    if err is not None:
        assert err.status in (5, 6), err


def test_mtx_symmetric_expansion():
    import tempfile
    with tempfile.NamedTemporaryFile("w", suffix=".mtx", delete=False) as f:
        f.write(MTX_CASES["skew"])
    A = vm.read_matrix_market(f.name)
    rp, col, val = A.arrays()
    dense = np.zeros((3, 3))
    for r in range(3):
        for p in range(rp[r], rp[r + 1]):
            dense[r, col[p]] = val[p]
    assert np.array_equal(dense, np.array([[0, -3, 1], [3, 0, 0], [-1, 0, 0]]))
    os.unlink(f.name)


def test_coo_to_csr_sorts_and_rejects_duplicates():
    A = vm.coo_to_csr(2, 4, [1, 0, 1, 0], [3, 2, 0, 1], [1.0, 2.0, 3.0, 4.0])
    rp, col, val = A.arrays()
    assert list(rp) == [0, 2, 4] and list(col) == [1, 2, 0, 3] and list(val) == [4.0, 2.0, 3.0, 1.0]
    with pytest.raises(vm.VcsrmcError) as e:
        vm.coo_to_csr(2, 2, [0, 0], [1, 1], [1.0, 2.0])
    assert e.value.status == 6
    with pytest.raises(vm.VcsrmcError):
        vm.coo_to_csr(2, 2, [0], [5], [1.0])


# ---- generators and partition -------------------------------------------------------------------
def test_config1_generator_matches_numpy_restatement():
    """The C++ generator against an independent numpy restatement of the same streams."""
    from vcsr_mc_b200 import rng
    M = N = 512
    A = vm.CSR.generate(vm.GEN_UNIFORM_POISSON, M, seed=0)
    rp, col, val = A.arrays()
    klen, kcols, kvals = (rng.key(0, s) for s in (rng.STREAM_ROWLEN, rng.STREAM_COLS, rng.STREAM_VALS))
    u = rng.u01(rng.at(klen, np.arange(M)))
    exp = np.zeros(M + 1, dtype=np.int64)
    for r in range(M):
        k, p = 0, np.exp(-16.0)
        F = p
        while u[r] >= F and k < 260:
            k += 1
            p *= 16.0 / k
            F += p
        chosen = []
        draws = rng.at(kcols, (np.uint64(r) << np.uint64(32)) + np.arange(k, dtype=np.uint64))
        for t in range(k):
            j = N - k + t
            x = int(draws[t] % np.uint64(j + 1))
            chosen.append(j if x in chosen else x)
        exp[r + 1] = exp[r] + k
        assert list(col[rp[r]:rp[r + 1]]) == sorted(chosen), r
    assert np.array_equal(rp, exp)
    assert np.array_equal(val, rng.sym(rng.at(kvals, np.arange(exp[-1]))))


def test_stencil_links_generator_matches_numpy_restatement():
    """The stencil-plus-links generator: the stencil of GEN_STENCIL27 plus, per row, the columns of
    the links stream that are not already in the row, each with the stream's next draw as value."""
    from vcsr_mc_b200 import rng
    n, links = 9, 3
    A = vm.CSR.generate(vm.GEN_STENCIL27_LINKS, n, seed=4)
    S = vm.CSR.generate(vm.GEN_STENCIL27, n, seed=4)
    rp, col, val = A.arrays()
    srp, scol, sval = S.arrays()
    M = n ** 3
    kl = rng.key(4, rng.STREAM_LINKS)
    for r in range(M):
        want = dict(zip(scol[srp[r]:srp[r + 1]].tolist(), sval[srp[r]:srp[r + 1]].tolist()))
        d = 2 * (r * links + np.arange(links, dtype=np.uint64))
        cs = (rng.at(kl, d) % np.uint64(M)).astype(np.int64)
        vs = rng.sym(rng.at(kl, d + np.uint64(1)))
        for c, v in zip(cs.tolist(), vs.tolist()):
            if c not in want:
                want[c] = v
        cols = sorted(want)
        assert col[rp[r]:rp[r + 1]].tolist() == cols, r
        assert np.array_equal(val[rp[r]:rp[r + 1]], np.array([want[c] for c in cols], dtype=np.float32)), r


def test_generators_deterministic_and_thread_independent():
    for kind, param in [(vm.GEN_ZIPF, 4096), (vm.GEN_RMAT, 12), (vm.GEN_STENCIL27, 8), (vm.GEN_STENCIL27_LINKS, 8)]:
        a = vm.CSR.generate(kind, param, seed=1, nthreads=1).arrays()
        b = vm.CSR.generate(kind, param, seed=1, nthreads=5).arrays()
        for x, y in zip(a, b):
            assert np.array_equal(x, y)


def test_generator_properties():
    S = vm.CSR.generate(vm.GEN_STENCIL27, 10, seed=0)
    rp, col, val = S.arrays()
    assert S.nnz == (3 * 10 - 2) ** 3  # 27-point stencil on n^3: (3n-2)^3 entries
    diag = [val[p] for r in range(S.M) for p in range(rp[r], rp[r + 1]) if col[p] == r]
    assert len(diag) == S.M and all(d == 26.0 for d in diag)
    R = vm.CSR.generate(vm.GEN_RMAT, 12, seed=0)
    rp, col, val = R.arrays()
    for r in range(R.M):
        assert np.all(np.diff(col[rp[r]:rp[r + 1]]) > 0)
    assert 0.7 * 2 ** 16 < R.nnz <= 2 ** 16  # 2^(scale+4) samples, duplicates removed
    Z = vm.CSR.generate(vm.GEN_ZIPF, 1 << 16, seed=0)
    assert 9.0 < Z.nnz / Z.M < 11.5
    assert np.all(np.abs(val) <= 1.0)


def test_dense_generator_matches_numpy_restatement():
    from vcsr_mc_b200 import rng
    h = vm.gen_dense_host(37, 19, seed=5)
    assert np.array_equal(h, rng.dense_rows(np.arange(37), 19, 5))


def test_partition_rows():
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 14, seed=3)
    rp, _, _ = A.arrays()
    for parts in (1, 2, 3, 8):
        cuts = vm.partition_rows(rp, parts)
        assert cuts[0] == 0 and cuts[-1] == A.M and np.all(np.diff(cuts) >= 0)
        for k in range(1, parts):
            target = -(-k * A.nnz // parts)
            assert rp[cuts[k]] >= target and (cuts[k] == 0 or rp[cuts[k] - 1] < target)


def test_partition_rows_weighted():
    A = vm.CSR.generate(vm.GEN_RMAT, 14, seed=3)
    rp, _, _ = A.arrays()
    w = 5.4
    for parts in (2, 4, 8):
        cuts = vm.partition_rows(rp, parts, row_weight=w)
        assert cuts[0] == 0 and cuts[-1] == A.M and np.all(np.diff(cuts) >= 0)
        cost = rp.astype(np.float64) + w * np.arange(A.M + 1)
        for k in range(1, parts):
            target = cost[-1] * k / parts
            assert cost[cuts[k]] >= target and (cuts[k] == 0 or cost[cuts[k] - 1] < target)
    assert np.array_equal(vm.partition_rows(rp, 4, row_weight=0.0), vm.partition_rows(rp, 4))
