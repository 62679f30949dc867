"""Generates tests/golden/golden.npz: small inputs with the outputs of the reference itself.

The outputs come from the reference implementation compiled from its own sources
(oracle/_ref/libvcsr_ref.so, built by oracle/Makefile where the reference checkout exists):
  * csr_to_vcsr_mc arrays (src/vcsr_mc.cu:25-123) for segw 16/32/48/64, FP16 and FP32 formats,
  * half_scale (src/vcsr_mc.cu:14-22),
  * rcm_column_order (include/reorder.hpp:17-77),
  * the fp64 CPU SpMM loop (src/main.cpp:202-207).
The inputs are built here with numpy's PCG64 from fixed seeds and stored in the file, so the
tests never need to regenerate them. Run from the repository root:
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import bind as ob  # noqa: E402


def csr_from_rows(M, N, rows_cols, vals):
    rp = np.zeros(M + 1, dtype=np.int32)
    for r, c in enumerate(rows_cols):
        rp[r + 1] = rp[r] + len(c)
    col = np.concatenate([np.asarray(c, dtype=np.int32) for c in rows_cols]) if rp[-1] else np.zeros(0, np.int32)
    return rp, col, np.asarray(vals, dtype=np.float32)


def random_case(seed, M, N, mean, empty_frac=0.0, scale=1.0, zipf=False):
    rng = np.random.default_rng(seed)
    rows = []
    for _ in range(M):
        if rng.random() < empty_frac:
            rows.append([])
            continue
        k = int(min(N, (rng.zipf(1.8) if zipf else rng.poisson(mean))))
        rows.append(np.sort(rng.choice(N, size=k, replace=False)))
    nnz = sum(len(r) for r in rows)
    vals = rng.uniform(-1, 1, size=nnz) * scale
    return csr_from_rows(M, N, rows, vals) + (M, N)


def stencil2d(n):
    rows = []
    for i in range(n * n):
        x, y = i % n, i // n
        r = []
        for dy in (-1, 0, 1):
            for dx in (-1, 0, 1):
                if 0 <= x + dx < n and 0 <= y + dy < n:
                    r.append((y + dy) * n + x + dx)
        rows.append(sorted(r))
    nnz = sum(len(r) for r in rows)
    vals = np.where(np.arange(nnz) % 9 == 4, 8.0, -1.0)
    return csr_from_rows(n * n, n * n, rows, vals) + (n * n, n * n)


CASES = {
    "uniform_300": lambda: random_case(1, 300, 300, 6.0),
    "rect_200x900": lambda: random_case(2, 200, 900, 12.0, empty_frac=0.2),
    "zipf_512": lambda: random_case(3, 512, 512, 0.0, zipf=True),
    "tiny_5x7": lambda: random_case(4, 5, 7, 3.0),
    "large_values": lambda: random_case(5, 64, 96, 5.0, scale=1e6),
    "tiny_values": lambda: random_case(6, 64, 96, 5.0, scale=1e-6),
    "stencil2d_20": lambda: stencil2d(20),
}


def main():
    if not ob.ref_available():
        raise SystemExit("oracle/_ref/libvcsr_ref.so is needed (make -C oracle where the reference exists)")
    out = {}
    rng = np.random.default_rng(99)
    for name, make in CASES.items():
        rp, col, val, M, N = make()
        out[f"{name}/row_ptr"], out[f"{name}/col"], out[f"{name}/val"] = rp, col, val
        out[f"{name}/shape"] = np.array([M, N], dtype=np.int64)
        out[f"{name}/half_scale"] = np.array([ob.ref_half_scale(val)], dtype=np.float32)
        for segw in (16, 32, 48, 64):
            for fp32 in (0, 1):
                f = ob.ref_build_vcsr(M, N, rp, col, val, bool(fp32), segw)
                for k in ob.VCSR_ARRAYS:
                    out[f"{name}/vcsr_s{segw}_f{fp32}/{k}"] = f[k]
                out[f"{name}/vcsr_s{segw}_f{fp32}/meta"] = np.array(
                    [f["num_segments"], f["bundle"], f["scale"]], dtype=np.float64)
        if M == N:
            out[f"{name}/rcm"] = ob.ref_rcm_column_order(M, N, rp, col)
        B = rng.uniform(-1, 1, size=(N, 16)).astype(np.float32)
        out[f"{name}/B"] = B
        ref = np.empty((M, 16), dtype=np.float64)
        runner = ob.RefSpmm(rp, col, val, B, nslices=1)
        runner.run(ref)
        runner.close()
        out[f"{name}/spmm_fp64"] = ref
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
