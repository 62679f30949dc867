"""ctypes binding of libvcsrmc.so (the C ABI declared in include/vcsrmc.h).

The library is built in-tree (``make -C vcsr_mc_b200/csrc`` or ``__graft_entry__.build()``).
There is no fallback: if the shared object is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvcsrmc.so")

# status codes (vcsrmc.h)
OK, INVALID_ARG, CUDA_ERR, OOM, TIMEOUT, IO_ERR, FORMAT_ERR, INTERNAL = range(8)
F32, F16 = 0, 1
GEN_UNIFORM_POISSON, GEN_ZIPF, GEN_STENCIL27, GEN_RMAT, GEN_STENCIL27_LINKS = 1, 2, 3, 4, 5
PLAN_AUTO, PLAN_SEGMENT, PLAN_ROWS, PLAN_BAND, PLAN_HYBRID = 0, 1, 2, 3, 4

_STATUS_NAMES = {
    OK: "OK", INVALID_ARG: "INVALID_ARG", CUDA_ERR: "CUDA_ERR", OOM: "OOM", TIMEOUT: "TIMEOUT",
    IO_ERR: "IO_ERR", FORMAT_ERR: "FORMAT_ERR", INTERNAL: "INTERNAL",
}


class VcsrmcError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")


class DeviceInfo(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("segw", ctypes.c_int32),
                ("fp32", ctypes.c_int32), ("scale", ctypes.c_float), ("plans", ctypes.c_int32),
                ("n_groups", ctypes.c_int64), ("n_slots", ctypes.c_int64), ("n_items", ctypes.c_int64),
                ("n_units", ctypes.c_int64), ("rows_unit_nnz", ctypes.c_int32), ("n_split_rows", ctypes.c_int32),
                ("band_rows", ctypes.c_int32), ("n_bands", ctypes.c_int32),
                ("n_tiles", ctypes.c_int64), ("band_cols", ctypes.c_int32), ("n_hot", ctypes.c_int32),
                ("hybrid_band_rows", ctypes.c_int32), ("reserved2", ctypes.c_int32), ("hybrid_tiles", ctypes.c_int64),
                ("hybrid_band_nnz", ctypes.c_int64), ("hybrid_rows_nnz", ctypes.c_int64)]


class UploadOptions(ctypes.Structure):
    _fields_ = [("plans", ctypes.c_int32), ("rows_unit_nnz", ctypes.c_int32), ("band_rows", ctypes.c_int32),
                ("hot_rows", ctypes.c_int32), ("hot_budget_mib", ctypes.c_int32), ("hot_persist", ctypes.c_int32),
                ("hot_evict_first", ctypes.c_int32), ("reserved", ctypes.c_int32 * 1)]


class CsrView(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("nnz", ctypes.c_int64),
        ("row_ptr", ctypes.POINTER(ctypes.c_int32)), ("col", ctypes.POINTER(ctypes.c_int32)),
        ("val", ctypes.POINTER(ctypes.c_float)),
    ]


class FormatView(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("segw", ctypes.c_int32), ("bundle", ctypes.c_int32),
        ("num_segments", ctypes.c_int32), ("fp32", ctypes.c_int32), ("scale", ctypes.c_float),
        ("n_groups", ctypes.c_int64), ("n_slots", ctypes.c_int64), ("n_items", ctypes.c_int64),
        ("group_ptr", ctypes.POINTER(ctypes.c_int32)), ("group_depth", ctypes.POINTER(ctypes.c_int32)),
        ("group_seg_base", ctypes.POINTER(ctypes.c_int32)), ("group_rows", ctypes.POINTER(ctypes.c_int32)),
        ("lcol", ctypes.POINTER(ctypes.c_int32)), ("val", ctypes.POINTER(ctypes.c_float)),
        ("item_gbeg", ctypes.POINTER(ctypes.c_int32)), ("item_gend", ctypes.POINTER(ctypes.c_int32)),
    ]


_p = ctypes.c_void_p
_i32, _i64, _u64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
_int = ctypes.c_int
_pi32 = ctypes.POINTER(ctypes.c_int32)
_pf32 = ctypes.POINTER(ctypes.c_float)
_pp = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); every function of include/vcsrmc.h
PROTOTYPES = {
    "vcsrmc_version": (_int, []),
    "vcsrmc_last_error": (_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "vcsrmc_csr_read_mtx": (_int, [ctypes.c_char_p, _pp]),
    "vcsrmc_csr_from_coo": (_int, [_i32, _i32, _i64, _p, _p, _p, _pp]),
    "vcsrmc_csr_from_arrays": (_int, [_i32, _i32, _i64, _p, _p, _p, _pp]),
    "vcsrmc_csr_view_get": (_int, [_p, ctypes.POINTER(CsrView)]),
    "vcsrmc_csr_row_slice": (_int, [_p, _i32, _i32, _pp]),
    "vcsrmc_csr_free": (None, [_p]),
    "vcsrmc_csr_save": (_int, [_p, ctypes.c_char_p]),
    "vcsrmc_csr_load": (_int, [ctypes.c_char_p, _pp]),
    "vcsrmc_rcm_column_order": (_int, [_p, _p]),
    "vcsrmc_apply_column_permutation": (_int, [_p, _p, _i32, _p]),
    "vcsrmc_half_scale": (_int, [_p, _pf32]),
    "vcsrmc_build_host": (_int, [_p, _int, _int, _int, _pp]),
    "vcsrmc_format_view_get": (_int, [_p, ctypes.POINTER(FormatView)]),
    "vcsrmc_format_free": (None, [_p]),
    "vcsrmc_format_from_view": (_int, [ctypes.POINTER(FormatView), _pp]),
    "vcsrmc_upload": (_int, [_p, _int, _p, _pp]),
    "vcsrmc_upload_ex": (_int, [_p, _int, _int, _p, _pp]),
    "vcsrmc_upload_opts": (_int, [_p, _int, ctypes.POINTER(UploadOptions), _p, _pp]),
    "vcsrmc_build_device": (_int, [_i32, _i32, _i64, _p, _p, _p, _int, _int, _int, ctypes.POINTER(UploadOptions), _p,
                                   _pp]),
    "vcsrmc_device_download": (_int, [_p, _pp]),
    "vcsrmc_half_scale_device": (_int, [_p, _i64, _p, ctypes.POINTER(ctypes.c_float)]),
    "vcsrmc_device_wait_check": (_int, [_p, _i64, _p, ctypes.POINTER(ctypes.c_int)]),
    "vcsrmc_device_info_get": (_int, [_p, ctypes.POINTER(DeviceInfo)]),
    "vcsrmc_device_free": (_int, [_p]),
    "vcsrmc_device_status": (_int, [_p, ctypes.POINTER(ctypes.c_uint32), _int]),
    "vcsrmc_spmm": (_int, [_p, _p, _int, _i64, _i32, _i32, _p, _i64, _int, _p]),
    "vcsrmc_spmm_ex": (_int, [_p, _p, _int, _i64, _i32, _i32, _p, _i64, _int, _int, _p]),
    "vcsrmc_spmm_timed": (_int, [_p, _p, _int, _i64, _i32, _i32, _p, _i64, _int, _p, _pf32]),
    "vcsrmc_gen_csr": (_int, [_int, _i32, _u64, _int, _pp]),
    "vcsrmc_gen_dense_host": (_int, [_i64, _i32, _u64, _p, _int]),
    "vcsrmc_gen_dense_device": (_int, [_i64, _i32, _u64, _int, _p, _i64, _p]),
    "vcsrmc_partition_rows": (_int, [_p, _i32, _i32, _p]),
    "vcsrmc_partition_rows_weighted": (_int, [_p, _i32, _i32, ctypes.c_double, _p]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once). Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is not built; run `make -C vcsr_mc_b200/csrc` "
                    "(or __graft_entry__.build()). There is no CPU fallback.")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int) -> None:
    if status != OK:
        buf = ctypes.create_string_buffer(1024)
        lib().vcsrmc_last_error(buf, len(buf))
        raise VcsrmcError(status, buf.value.decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
