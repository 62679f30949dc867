"""TEST INFRASTRUCTURE — ORACLE ONLY.

ctypes bindings of
  * oracle/liboracle.so         the plain-C restatement (oracle.c), and
  * oracle/_ref/libvcsr_ref.so  the reference's own host code compiled from its sources
                                (ref_shim.cpp; built only where the reference checkout exists,
                                then shipped as a prebuilt file).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import this
module, and only to check or to time the CPU baseline; the product never does.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libvcsr_ref.so")

VCSR_ARRAYS = ("group_ptr", "group_depth", "group_seg_base", "group_rows", "lcol", "val", "item_gbeg", "item_gend")

_p = ctypes.c_void_p
_i32, _i64 = ctypes.c_int32, ctypes.c_int64
_pi32 = ctypes.POINTER(ctypes.c_int32)
_pf32 = ctypes.POINTER(ctypes.c_float)


class _VcsrView(ctypes.Structure):
    _fields_ = [
        ("M", _i32), ("N", _i32), ("segw", _i32), ("bundle", _i32), ("num_segments", _i32), ("fp32", _i32),
        ("scale", ctypes.c_float), ("n_groups", _i64), ("n_slots", _i64), ("n_items", _i64),
        ("group_ptr", _pi32), ("group_depth", _pi32), ("group_seg_base", _pi32), ("group_rows", _pi32),
        ("lcol", _pi32), ("val", _pf32), ("item_gbeg", _pi32), ("item_gend", _pi32),
    ]


class _RefVcsrView(ctypes.Structure):
    _fields_ = _VcsrView._fields_ + [("impl", _p)]


class _RefCsrView(ctypes.Structure):
    _fields_ = [("M", _i32), ("N", _i32), ("nnz", _i64), ("row_ptr", _pi32), ("col", _pi32), ("val", _pf32),
                ("impl", _p)]


def _np(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a: Optional[np.ndarray]):
    return ctypes.c_void_p(a.ctypes.data) if a is not None and a.size else ctypes.c_void_p(0)


def _arr(ptr, n, dtype):
    if n == 0:
        return np.zeros(0, dtype=dtype)
    return np.ctypeslib.as_array(ptr, shape=(n,)).copy()


def _view_to_dict(v) -> dict:
    sizes = {"group_ptr": v.n_groups + 1, "group_depth": v.n_groups, "group_seg_base": v.n_groups,
             "group_rows": 16 * v.n_groups, "lcol": v.n_slots, "val": v.n_slots, "item_gbeg": v.n_items,
             "item_gend": v.n_items}
    out = {k: _arr(getattr(v, k), sizes[k], np.float32 if k == "val" else np.int32) for k in VCSR_ARRAYS}
    out.update(M=v.M, N=v.N, segw=v.segw, bundle=v.bundle, num_segments=v.num_segments, fp32=bool(v.fp32),
               scale=float(v.scale))
    return out


# ---- the C restatement --------------------------------------------------------------------------
_oracle = None


def oracle():
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            raise ImportError(f"{ORACLE_SO} missing: run `make -C oracle`")
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_spmm_fp64.argtypes = [_i32, _p, _p, _p, _p, _i32, _p, _p, ctypes.c_int]
        L.oracle_spmm_fp64.restype = None
        L.oracle_spmm_fp64_rows.argtypes = [_p, _p, _p, _p, _i32, _p, _i32, _p, _p]
        L.oracle_spmm_fp64_rows.restype = None
        L.oracle_half_scale.argtypes = [_i64, _p]
        L.oracle_half_scale.restype = ctypes.c_float
        L.oracle_build_vcsr.argtypes = [_i32, _i32, _p, _p, _p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_VcsrView)]
        L.oracle_build_vcsr.restype = ctypes.c_int
        L.oracle_vcsr_free.argtypes = [ctypes.POINTER(_VcsrView)]
        L.oracle_vcsr_free.restype = None
        L.oracle_canonicalize_vcsr.argtypes = [_i64, _i32, _p, _p, _p, _p, _p, _p]
        L.oracle_canonicalize_vcsr.restype = None
        L.oracle_rcm_column_order.argtypes = [_i32, _i32, _p, _p, _p]
        L.oracle_rcm_column_order.restype = None
        L.oracle_apply_column_permutation.argtypes = [_i32, _i32, _p, _p, _p, _p, _i32, _p]
        L.oracle_apply_column_permutation.restype = None
        _oracle = L
    return _oracle


def spmm_fp64(row_ptr, col, val, B, nthreads: int = 8, with_abs: bool = False):
    """fp64 CSR SpMM (src/main.cpp:202-207); B is N x O (converted to fp32 exactly)."""
    rp, c, v = _np(row_ptr, np.int32), _np(col, np.int32), _np(val, np.float32)
    Bf = _np(B, np.float32)
    M, O = rp.size - 1, Bf.shape[1]
    out = np.empty((M, O), dtype=np.float64)
    ab = np.empty((M, O), dtype=np.float64) if with_abs else None
    oracle().oracle_spmm_fp64(M, _ptr(rp), _ptr(c), _ptr(v), _ptr(Bf), O, _ptr(out), _ptr(ab), nthreads)
    return (out, ab) if with_abs else out


def spmm_fp64_rows(row_ptr, col, val, B, rows, with_abs: bool = False):
    rp, c, v = _np(row_ptr, np.int32), _np(col, np.int32), _np(val, np.float32)
    Bf, r = _np(B, np.float32), _np(rows, np.int32)
    O = Bf.shape[1]
    out = np.empty((r.size, O), dtype=np.float64)
    ab = np.empty((r.size, O), dtype=np.float64) if with_abs else None
    oracle().oracle_spmm_fp64_rows(_ptr(rp), _ptr(c), _ptr(v), _ptr(Bf), O, _ptr(r), r.size, _ptr(out), _ptr(ab))
    return (out, ab) if with_abs else out


def half_scale(val) -> float:
    v = _np(val, np.float32)
    return float(oracle().oracle_half_scale(v.size, _ptr(v)))


def build_vcsr(M, N, row_ptr, col, val, fp32: bool, segw: int) -> dict:
    rp, c, v = _np(row_ptr, np.int32), _np(col, np.int32), _np(val, np.float32)
    view = _VcsrView()
    rc = oracle().oracle_build_vcsr(M, N, _ptr(rp), _ptr(c), _ptr(v), 1 if fp32 else 0, segw, ctypes.byref(view))
    if rc != 0:
        raise ValueError(f"oracle: unsupported segw {segw}")
    try:
        return _view_to_dict(view)
    finally:
        oracle().oracle_vcsr_free(ctypes.byref(view))


def canonicalize(fmt: dict) -> dict:
    """Copy of a VCSR dict with rows of equal per-segment count in ascending row order."""
    out = {k: (np.array(v, copy=True) if isinstance(v, np.ndarray) else v) for k, v in fmt.items()}
    gp, gd, gs = (_np(out[k], np.int32) for k in ("group_ptr", "group_depth", "group_seg_base"))
    gr, lc, vv = _np(out["group_rows"], np.int32), _np(out["lcol"], np.int32), _np(out["val"], np.float32)
    oracle().oracle_canonicalize_vcsr(gd.size, int(out["segw"]), _ptr(gp), _ptr(gd), _ptr(gs), _ptr(gr), _ptr(lc),
                                      _ptr(vv))
    out["group_rows"], out["lcol"], out["val"] = gr, lc, vv
    return out


def rcm_column_order(M, N, row_ptr, col) -> np.ndarray:
    rp, c = _np(row_ptr, np.int32), _np(col, np.int32)
    pos = np.empty(N, dtype=np.int32)
    oracle().oracle_rcm_column_order(M, N, _ptr(rp), _ptr(c), _ptr(pos))
    return pos


def apply_column_permutation(M, N, row_ptr, col, val, B, position):
    rp = _np(row_ptr, np.int32)
    c, v = np.array(col, dtype=np.int32, copy=True), np.array(val, dtype=np.float32, copy=True)
    Bc = None if B is None else np.array(B, dtype=np.float32, copy=True, order="C")
    O = 0 if Bc is None else Bc.shape[1]
    oracle().oracle_apply_column_permutation(M, N, _ptr(rp), _ptr(c), _ptr(v), _ptr(Bc), O,
                                             _ptr(_np(position, np.int32)))
    return c, v, Bc


# ---- the reference itself (oracle/_ref) ---------------------------------------------------------
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise ImportError(f"{REF_SO} missing: build it with `make -C oracle` where the reference exists")
        L = ctypes.CDLL(REF_SO)
        L.ref_build_vcsr.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _p, _p, _p, ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(_RefVcsrView), ctypes.c_char_p, ctypes.c_size_t]
        L.ref_build_vcsr.restype = ctypes.c_int
        L.ref_vcsr_free.argtypes = [ctypes.POINTER(_RefVcsrView)]
        L.ref_vcsr_free.restype = None
        L.ref_half_scale.argtypes = [_i64, _p]
        L.ref_half_scale.restype = ctypes.c_float
        L.ref_read_mtx.argtypes = [ctypes.c_char_p, ctypes.POINTER(_RefCsrView), ctypes.c_char_p, ctypes.c_size_t]
        L.ref_read_mtx.restype = ctypes.c_int
        L.ref_coo_to_csr.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _p, _p, _p, ctypes.POINTER(_RefCsrView),
                                     ctypes.c_char_p, ctypes.c_size_t]
        L.ref_coo_to_csr.restype = ctypes.c_int
        L.ref_csr_free.argtypes = [ctypes.POINTER(_RefCsrView)]
        L.ref_csr_free.restype = None
        L.ref_rcm_column_order.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _p, _p, _p]
        L.ref_rcm_column_order.restype = ctypes.c_int
        L.ref_apply_column_permutation.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _p, _p, _p, _p, ctypes.c_int, _p]
        L.ref_apply_column_permutation.restype = ctypes.c_int
        L.ref_spmm_ctx_create.argtypes = [ctypes.c_int, ctypes.c_int, _i64, _p, _p, _p, _p, ctypes.c_int,
                                          ctypes.c_int]
        L.ref_spmm_ctx_create.restype = ctypes.c_void_p
        L.ref_spmm_ctx_run.argtypes = [ctypes.c_void_p, _p]
        L.ref_spmm_ctx_run.restype = None
        L.ref_spmm_ctx_free.argtypes = [ctypes.c_void_p]
        L.ref_spmm_ctx_free.restype = None
        _ref = L
    return _ref


class RefError(RuntimeError):
    pass


def ref_build_vcsr(M, N, row_ptr, col, val, fp32: bool, segw: int) -> dict:
    rp, c, v = _np(row_ptr, np.int32), _np(col, np.int32), _np(val, np.float32)
    view = _RefVcsrView()
    err = ctypes.create_string_buffer(512)
    rc = ref().ref_build_vcsr(M, N, c.size, _ptr(rp), _ptr(c), _ptr(v), 1 if fp32 else 0, segw,
                              ctypes.byref(view), err, 512)
    if rc != 0:
        raise RefError(err.value.decode())
    try:
        return _view_to_dict(view)
    finally:
        ref().ref_vcsr_free(ctypes.byref(view))


def ref_half_scale(val) -> float:
    v = _np(val, np.float32)
    return float(ref().ref_half_scale(v.size, _ptr(v)))


def _ref_csr(view) -> tuple:
    out = (view.M, view.N, _arr(view.row_ptr, view.M + 1, np.int32), _arr(view.col, view.nnz, np.int32),
           _arr(view.val, view.nnz, np.float32))
    ref().ref_csr_free(ctypes.byref(view))
    return out


def ref_read_mtx(path: str) -> tuple:
    view = _RefCsrView()
    err = ctypes.create_string_buffer(512)
    if ref().ref_read_mtx(path.encode(), ctypes.byref(view), err, 512) != 0:
        raise RefError(err.value.decode())
    return _ref_csr(view)


def ref_coo_to_csr(M, N, rows, cols, vals) -> tuple:
    r, c, v = _np(rows, np.int32), _np(cols, np.int32), _np(vals, np.float32)
    view = _RefCsrView()
    err = ctypes.create_string_buffer(512)
    if ref().ref_coo_to_csr(M, N, v.size, _ptr(r), _ptr(c), _ptr(v), ctypes.byref(view), err, 512) != 0:
        raise RefError(err.value.decode())
    return _ref_csr(view)


def ref_rcm_column_order(M, N, row_ptr, col) -> np.ndarray:
    rp, c = _np(row_ptr, np.int32), _np(col, np.int32)
    pos = np.empty(N, dtype=np.int32)
    ref().ref_rcm_column_order(M, N, c.size, _ptr(rp), _ptr(c), _ptr(pos))
    return pos


def ref_apply_column_permutation(M, N, row_ptr, col, val, B, position):
    rp = _np(row_ptr, np.int32)
    c, v = np.array(col, dtype=np.int32, copy=True), np.array(val, dtype=np.float32, copy=True)
    Bc = None if B is None else np.array(B, dtype=np.float32, copy=True, order="C")
    O = 0 if Bc is None else Bc.shape[1]
    ref().ref_apply_column_permutation(M, N, c.size, _ptr(rp), _ptr(c), _ptr(v), _ptr(Bc), O,
                                       _ptr(_np(position, np.int32)))
    return c, v, Bc


class RefSpmm:
    """The reference's fp64 CPU SpMM loop over `nslices` row blocks (one thread each)."""

    def __init__(self, row_ptr, col, val, B, nslices: int = 1):
        self.rp, self.c, self.v = _np(row_ptr, np.int32), _np(col, np.int32), _np(val, np.float32)
        self.B = _np(B, np.float32)
        self.M, self.O = self.rp.size - 1, self.B.shape[1]
        self.ctx = ref().ref_spmm_ctx_create(self.M, self.B.shape[0], self.c.size, _ptr(self.rp), _ptr(self.c),
                                             _ptr(self.v), _ptr(self.B), self.O, nslices)

    def run(self, out: Optional[np.ndarray] = None) -> None:
        ref().ref_spmm_ctx_run(self.ctx, _ptr(out))

    def close(self) -> None:
        if self.ctx:
            ref().ref_spmm_ctx_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
