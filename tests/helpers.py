"""Shared test helpers: problem construction and the tolerance checks used by every SpMM test.

Tolerances (fp64 oracle = restatement of src/main.cpp:202-207 on the same inputs):
  * FP32 path: norm-wise relative L2 error <= 1e-5, and element-wise
    |C - ref| <= 1e-4 * sum_p |a_ip b_pj| + 1e-30 (fp32 accumulation over at most a few
    thousand terms stays far below this).
  * FP16 path (fp16 A values and B, fp32 accumulation): element-wise
    |C - ref| <= 2e-2 * sum_p |a_ip b_pj|, plus the reference's own acceptance bounds
    (src/main.cpp:281,286): ||C - ref|| <= 3e-3 ||ref|| + 1e-5 sqrt(numel) and rel-L2 <= 1e-1.
"""
from __future__ import annotations

import numpy as np

FP32_REL_L2 = 1e-5
FP32_ELEM = 1e-4
FP16_ELEM = 2e-2


def rel_l2(C: np.ndarray, ref: np.ndarray) -> float:
    num = float(np.linalg.norm((C.astype(np.float64) - ref).ravel()))
    den = float(np.linalg.norm(ref.ravel()))
    return num / den if den > 0 else num


def check_fp32(C: np.ndarray, ref: np.ndarray, absref: np.ndarray) -> dict:
    err = np.abs(C.astype(np.float64) - ref)
    r = rel_l2(C, ref)
    assert np.all(np.isfinite(C)), "non-finite output"
    assert r <= FP32_REL_L2, f"FP32 rel-L2 {r:.3e} > {FP32_REL_L2}"
    worst = float(np.max(err - FP32_ELEM * absref)) if err.size else 0.0
    assert worst <= 1e-30, f"FP32 element bound exceeded by {worst:.3e}"
    return {"rel_l2": r, "max_abs": float(err.max()) if err.size else 0.0}


def check_fp16(C: np.ndarray, ref: np.ndarray, absref: np.ndarray) -> dict:
    err = np.abs(C.astype(np.float64) - ref)
    assert np.all(np.isfinite(C)), "non-finite output"
    worst = float(np.max(err - FP16_ELEM * absref - 1e-30)) if err.size else 0.0
    assert worst <= 0.0, f"FP16 element bound exceeded by {worst:.3e}"
    norm = float(np.linalg.norm(ref.ravel()))
    e = float(np.linalg.norm((C.astype(np.float64) - ref).ravel()))
    assert e <= 3e-3 * norm + 1e-5 * np.sqrt(ref.size), "reference's FP16 norm bound failed"
    r = rel_l2(C, ref)
    assert r <= 1e-1, f"rel-L2 {r:.3e} > 0.1"
    return {"rel_l2": r, "max_abs": float(err.max()) if err.size else 0.0}


def random_csr(M: int, N: int, density: float, seed: int, empty_rows: bool = False, scale: float = 1.0):
    """Small seeded CSR (numpy) with distinct sorted columns per row."""
    rng = np.random.default_rng(seed)
    rows, cols = [], []
    for r in range(M):
        if empty_rows and r % 3 == 1:
            continue
        k = rng.binomial(N, density)
        if k:
            c = np.sort(rng.choice(N, size=k, replace=False))
            rows.append(np.full(k, r, dtype=np.int32))
            cols.append(c.astype(np.int32))
    if rows:
        row = np.concatenate(rows)
        col = np.concatenate(cols)
    else:
        row = np.zeros(0, np.int32)
        col = np.zeros(0, np.int32)
    row_ptr = np.zeros(M + 1, dtype=np.int32)
    np.add.at(row_ptr, row + 1, 1)
    row_ptr = np.cumsum(row_ptr).astype(np.int32)
    val = (rng.uniform(-1, 1, size=col.size) * scale).astype(np.float32)
    return row_ptr, col, val
