"""Matrix Market ingest at scale and the binary CSR cache (host library, no GPU).

Files above 1 MB are parsed in parallel chunks cut at line boundaries; the result, the accepted
and rejected inputs and the error messages must be those of the sequential reader
(include/mmio.hpp:19-75 of the reference), so every case is compared with the reference's own
reader (oracle/_ref) where it is built, and with a numpy restatement of coo_to_csr
(include/csr.hpp:16-41). Inputs of 2^20 entries and more take the parallel coo_to_csr.
"""
import numpy as np
import pytest

import vcsr_mc_b200 as vm
from oracle import bind as ob


def csr_from_coo_np(M, rows, cols, vals):
    order = np.lexsort((cols, rows))
    rp = np.zeros(M + 1, np.int64)
    np.add.at(rp, rows + 1, 1)
    return np.cumsum(rp).astype(np.int32), cols[order].astype(np.int32), vals[order].astype(np.float32)


def write_mtx(path, M, N, rows, cols, vals, field="real", symmetry="general", noise=True):
    rng = np.random.default_rng(1)
    with open(path, "w") as f:
        f.write(f"%%MatrixMarket matrix coordinate {field} {symmetry}\n% generated\n\n")
        f.write(f"{M} {N} {rows.size}\n")
        lines = []
        for i, (r, c) in enumerate(zip(rows + 1, cols + 1)):
            if field == "pattern":
                lines.append(f"{r} {c}\n")
            elif field == "integer":
                lines.append(f"{r} {c} {int(vals[i])}\n")
            else:
                lines.append(f"{r} {c} {vals[i]:.9g}\n")
            if noise and rng.random() < 0.001:
                lines.append("% a comment between entries\n" if rng.random() < 0.5 else "   \t\r\n")
        f.write("".join(lines))


def random_entries(M, N, n, seed, lower=False):
    rng = np.random.default_rng(seed)
    key = rng.choice(M * N, size=n, replace=False)
    rows, cols = (key // N).astype(np.int64), (key % N).astype(np.int64)
    if lower:
        keep = rows > cols  # strictly lower: no diagonal, no mirrored duplicates
        rows, cols = rows[keep], cols[keep]
    vals = rng.uniform(-1, 1, rows.size).astype(np.float32)
    return rows, cols, vals


def compare_with_reference(path, A):
    if not ob.ref_available():
        return
    ref = ob.ref_read_mtx(path)
    assert (A.M, A.N) == ref[:2]
    for a, b in zip(A.arrays(), ref[2:]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("field", ["real", "integer", "pattern"])
def test_large_general_file_matches_reference(tmp_path, field):
    M, N = 40000, 30000
    rows, cols, vals = random_entries(M, N, 400_000, seed=2)
    if field == "integer":
        vals = np.round(vals * 100).astype(np.float32)
    if field == "pattern":
        vals = np.ones_like(vals)
    path = str(tmp_path / "a.mtx")
    write_mtx(path, M, N, rows, cols, vals, field=field)
    A = vm.read_matrix_market(path)
    rp, col, val = csr_from_coo_np(M, rows, cols, vals)
    got = A.arrays()
    assert np.array_equal(got[0], rp) and np.array_equal(got[1], col)
    # values went through text with 9 significant digits: exact for fp32
    assert np.array_equal(got[2], val)
    compare_with_reference(path, A)


@pytest.mark.parametrize("symmetry", ["symmetric", "skew-symmetric"])
def test_large_symmetric_file_expands_like_reference(tmp_path, symmetry):
    M = 50000
    rows, cols, vals = random_entries(M, M, 300_000, seed=3, lower=True)
    path = str(tmp_path / "s.mtx")
    write_mtx(path, M, M, rows, cols, vals, symmetry=symmetry)
    A = vm.read_matrix_market(path)
    mv = -vals if symmetry == "skew-symmetric" else vals
    r2, c2, v2 = np.concatenate([rows, cols]), np.concatenate([cols, rows]), np.concatenate([vals, mv])
    rp, col, val = csr_from_coo_np(M, r2, c2, v2)
    got = A.arrays()
    for a, b in zip(got, (rp, col, val)):
        assert np.array_equal(a, b)
    compare_with_reference(path, A)


@pytest.mark.parametrize("where", ["bad_late", "range_late", "truncated", "extra", "nonfinite_late"])
def test_large_file_errors_match_the_sequential_reader(tmp_path, where):
    M, N = 20000, 20000
    rows, cols, vals = random_entries(M, N, 200_000, seed=4)
    path = str(tmp_path / "e.mtx")
    write_mtx(path, M, N, rows, cols, vals, noise=False)
    with open(path) as f:
        lines = f.read().split("\n")
    head = 4  # banner, comment, blank, dimensions
    k = 150_001  # an entry in a late chunk
    if where == "bad_late":
        lines[head + k] = "12 x 1.0"
    elif where == "range_late":
        lines[head + k] = f"{M + 1} 3 1.0"
    elif where == "nonfinite_late":
        lines[head + k] = "3 3 1e39"
    elif where == "truncated":
        lines = lines[: head + 199_990]
    elif where == "extra":
        lines.insert(len(lines) - 1, "1 1 1.0")
    with open(path, "w") as f:
        f.write("\n".join(lines))
    with pytest.raises(vm.VcsrmcError) as e:
        vm.read_matrix_market(path)
    assert e.value.status == 6
    msg = str(e.value)
    expect = {"bad_late": f"Bad MTX entry at index {k}", "range_late": "MTX row/column index out of range",
              "nonfinite_late": "MTX value is not finite FP32", "truncated": "Truncated MTX data",
              "extra": "Extra entries after declared MTX nnz"}[where]
    assert expect in msg
    if ob.ref_available():
        with pytest.raises(ob.RefError) as r:
            ob.ref_read_mtx(path)
        assert expect in str(r.value)


def test_parallel_coo_to_csr_matches_numpy():
    M, N = 300_000, 200_000
    rows, cols, vals = random_entries(M, N, 1_500_000, seed=5)
    perm = np.random.default_rng(6).permutation(rows.size)
    A = vm.coo_to_csr(M, N, rows[perm], cols[perm], vals[perm])
    rp, col, val = csr_from_coo_np(M, rows, cols, vals)
    for a, b in zip(A.arrays(), (rp, col, val)):
        assert np.array_equal(a, b)
    dup_r, dup_c = np.append(rows, rows[10]), np.append(cols, cols[10])
    with pytest.raises(vm.VcsrmcError) as e:
        vm.coo_to_csr(M, N, dup_r, dup_c, np.append(vals, 1.0).astype(np.float32))
    assert e.value.status == 6 and "Duplicate" in str(e.value)


def test_binary_cache_round_trip_and_corruption(tmp_path):
    A = vm.CSR.generate(vm.GEN_ZIPF, 1 << 15, seed=2)
    path = str(tmp_path / "a.csr")
    A.save(path)
    B = vm.load_csr(path)
    assert (B.M, B.N, B.nnz) == (A.M, A.N, A.nnz)
    for a, b in zip(A.arrays(), B.arrays()):
        assert np.array_equal(a, b)
    raw = open(path, "rb").read()
    bad = str(tmp_path / "bad.csr")
    for blob in (raw[:-4], b"NOTACSR!" + raw[8:], raw[:32] + b"\xff\xff\xff\x7f" + raw[36:]):
        open(bad, "wb").write(blob)
        with pytest.raises(vm.VcsrmcError) as e:
            vm.load_csr(bad)
        assert e.value.status == 6
    with pytest.raises(vm.VcsrmcError) as e:
        vm.load_csr(str(tmp_path / "missing.csr"))
    assert e.value.status == 5
