"""numpy mirror of the counter-based streams in csrc/common/vrng.h (bit-identical draws).

Used where host code needs a few rows of the dense B without generating all of it (the CPU
baseline sample, golden fixtures).
"""
from __future__ import annotations

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
STREAM_ROWLEN, STREAM_COLS, STREAM_VALS, STREAM_DENSE, STREAM_RMAT, STREAM_LINKS = 1, 2, 3, 4, 5, 6


def mix64(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = z ^ (z >> np.uint64(30))
        z = z * np.uint64(0xBF58476D1CE4E5B9)
        z = z ^ (z >> np.uint64(27))
        z = z * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def key(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        inner = mix64(np.uint64(stream) * GAMMA + np.uint64(0xD1B54A32D192ED03))
    return np.uint64(mix64(np.uint64(seed) ^ inner))


def at(k, i):
    i = np.asarray(i, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return mix64(np.uint64(k) + (i + np.uint64(1)) * GAMMA)


def u01(x):
    return (np.asarray(x, dtype=np.uint64) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def sym(x):
    d = (np.asarray(x, dtype=np.uint64) >> np.uint64(11)).astype(np.float64) * (1.0 / 4503599627370496.0) - 1.0
    return d.astype(np.float32)


def dense_rows(rows, cols: int, seed: int) -> np.ndarray:
    """Rows `rows` of the dense U(-1,1) matrix (element (i, j) = draw i*cols + j), fp32."""
    r = np.asarray(rows, dtype=np.uint64).reshape(-1, 1)
    idx = r * np.uint64(cols) + np.arange(cols, dtype=np.uint64).reshape(1, -1)
    return sym(at(key(seed, STREAM_DENSE), idx))
