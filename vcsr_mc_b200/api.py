"""Python mirror of the reference's host interface, over the C ABI (include/vcsrmc.h).

Names follow the reference (MuuSeoTia/VCSR_MC):
  read_matrix_market / coo_to_csr        include/mmio.hpp:19, include/csr.hpp:16
  rcm_column_order / apply_column_permutation   include/reorder.hpp:17, :82
  half_scale / csr_to_vcsr_mc            src/vcsr_mc.cu:14, :25
  upload_vcsr_mc_device                  src/vcsr_mc.cu:332
  run_vcsr_mc_spmm_gpu                   src/vcsr_mc.cu:352 (blocking, returns ms)
  destroy_vcsr_mc_device                 src/vcsr_mc.cu:397
Errors raise VcsrmcError (the reference throws std::runtime_error or exits).

Device buffers are torch CUDA tensors (torch is used for device memory and streams only);
every computation runs in libvcsrmc.so.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from ._lib import F16, F32, PLAN_AUTO, PLAN_BAND, PLAN_HYBRID, PLAN_ROWS, PLAN_SEGMENT, VcsrmcError, call


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data) if a.size else ctypes.c_void_p(0)


def _as_np(ptr, n: int, dtype) -> np.ndarray:
    if n == 0:
        return np.zeros(0, dtype=dtype)
    return np.ctypeslib.as_array(ptr, shape=(n,))


class CSR:
    """Host CSR owned by the library (fields of include/csr.hpp:8-13)."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib._lib is not None:
            _lib.lib().vcsrmc_csr_free(h)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def _view(self) -> _lib.CsrView:
        v = _lib.CsrView()
        call("vcsrmc_csr_view_get", self._h, ctypes.byref(v))
        return v

    @property
    def M(self) -> int:
        return self._view().M

    @property
    def N(self) -> int:
        return self._view().N

    @property
    def nnz(self) -> int:
        return self._view().nnz

    def arrays(self, copy: bool = True):
        """(row_ptr, col, val) as numpy arrays (views valid while this object lives if copy=False)."""
        v = self._view()
        rp = _as_np(v.row_ptr, v.M + 1, np.int32)
        col = _as_np(v.col, v.nnz, np.int32)
        val = _as_np(v.val, v.nnz, np.float32)
        if copy:
            return rp.copy(), col.copy(), val.copy()
        return rp, col, val

    def row_slice(self, r0: int, r1: int) -> "CSR":
        h = ctypes.c_void_p()
        call("vcsrmc_csr_row_slice", self._h, r0, r1, ctypes.byref(h))
        return CSR(h)

    def save(self, path: str) -> None:
        """Binary cache of this CSR (vcsrmc_csr_save); load it with load_csr."""
        call("vcsrmc_csr_save", self.handle, path.encode())

    @staticmethod
    def from_arrays(M: int, N: int, row_ptr, col, val) -> "CSR":
        rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
        c = np.ascontiguousarray(col, dtype=np.int32)
        v = np.ascontiguousarray(val, dtype=np.float32)
        h = ctypes.c_void_p()
        call("vcsrmc_csr_from_arrays", M, N, int(c.size), _ptr(rp), _ptr(c), _ptr(v), ctypes.byref(h))
        return CSR(h)

    @staticmethod
    def generate(kind: int, param: int, seed: int = 0, nthreads: int = 0) -> "CSR":
        h = ctypes.c_void_p()
        call("vcsrmc_gen_csr", kind, param, seed, nthreads, ctypes.byref(h))
        return CSR(h)


def load_csr(path: str) -> CSR:
    """A CSR saved by CSR.save (binary cache; vcsrmc_csr_load)."""
    h = ctypes.c_void_p()
    call("vcsrmc_csr_load", path.encode(), ctypes.byref(h))
    return CSR(h)


def read_matrix_market(path: str) -> CSR:
    """read_matrix_market_coo + coo_to_csr (include/mmio.hpp:19-75, include/csr.hpp:16-41)."""
    h = ctypes.c_void_p()
    call("vcsrmc_csr_read_mtx", path.encode(), ctypes.byref(h))
    return CSR(h)


def coo_to_csr(M: int, N: int, rows, cols, vals) -> CSR:
    r = np.ascontiguousarray(rows, dtype=np.int32)
    c = np.ascontiguousarray(cols, dtype=np.int32)
    v = np.ascontiguousarray(vals, dtype=np.float32)
    h = ctypes.c_void_p()
    call("vcsrmc_csr_from_coo", M, N, int(v.size), _ptr(r), _ptr(c), _ptr(v), ctypes.byref(h))
    return CSR(h)


def rcm_column_order(csr: CSR) -> np.ndarray:
    pos = np.empty(csr.N, dtype=np.int32)
    call("vcsrmc_rcm_column_order", csr.handle, _ptr(pos))
    return pos


def apply_column_permutation(csr: CSR, B: Optional[np.ndarray], position: np.ndarray) -> Optional[np.ndarray]:
    """Relabels csr's columns in place; returns B (N x O fp32) with its rows permuted."""
    pos = np.ascontiguousarray(position, dtype=np.int32)
    if B is None:
        call("vcsrmc_apply_column_permutation", csr.handle, ctypes.c_void_p(0), 0, _ptr(pos))
        return None
    Bc = np.array(B, dtype=np.float32, order="C", copy=True)
    call("vcsrmc_apply_column_permutation", csr.handle, _ptr(Bc), int(Bc.shape[1]), _ptr(pos))
    return Bc


def half_scale(csr: CSR) -> float:
    s = ctypes.c_float()
    call("vcsrmc_half_scale", csr.handle, ctypes.byref(s))
    return s.value


class VCSRMC:
    """Host VCSR-MC format (struct VCSRMC, include/vcsr_formats.hpp:14-21)."""

    ARRAYS = ("group_ptr", "group_depth", "group_seg_base", "group_rows", "lcol", "val", "item_gbeg", "item_gend")

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle
        v = _lib.FormatView()
        call("vcsrmc_format_view_get", handle, ctypes.byref(v))
        self._v = v
        self.M, self.N, self.segw, self.bundle = v.M, v.N, v.segw, v.bundle
        self.num_segments, self.fp32, self.scale = v.num_segments, bool(v.fp32), v.scale
        self.n_groups, self.n_slots, self.n_items = v.n_groups, v.n_slots, v.n_items

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib._lib is not None:
            _lib.lib().vcsrmc_format_free(h)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def array(self, name: str, copy: bool = True) -> np.ndarray:
        v = self._v
        n = {"group_ptr": v.n_groups + 1, "group_depth": v.n_groups, "group_seg_base": v.n_groups,
             "group_rows": 16 * v.n_groups, "lcol": v.n_slots, "val": v.n_slots,
             "item_gbeg": v.n_items, "item_gend": v.n_items}[name]
        a = _as_np(getattr(v, name), n, np.float32 if name == "val" else np.int32)
        return a.copy() if copy else a

    def arrays(self, copy: bool = True) -> dict:
        return {k: self.array(k, copy) for k in self.ARRAYS}


def csr_to_vcsr_mc(csr: CSR, fp32: bool = False, segw: int = 16, nthreads: int = 0) -> VCSRMC:
    h = ctypes.c_void_p()
    call("vcsrmc_build_host", csr.handle, 1 if fp32 else 0, segw, nthreads, ctypes.byref(h))
    return VCSRMC(h)


def _stream_handle(stream) -> ctypes.c_void_p:
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream))


class DeviceVCSRMC:
    """A VCSR-MC format resident on one GPU (replaces src/vcsr_mc.cu:126-131's statics)."""

    def __init__(self, handle: ctypes.c_void_p, host: Optional[VCSRMC], device: int, **shape):
        self._h = handle
        self.device = device
        if host is not None:
            shape = dict(M=host.M, N=host.N, fp32=host.fp32, scale=host.scale, segw=host.segw)
        self.M, self.N, self.fp32, self.scale, self.segw = (shape[k] for k in ("M", "N", "fp32", "scale", "segw"))

    def info(self) -> dict:
        """Shape and resident layouts (vcsrmc_device_info_get); plans is a list of PLAN_* values."""
        i = _lib.DeviceInfo()
        call("vcsrmc_device_info_get", self._h, ctypes.byref(i))
        out = {k: getattr(i, k) for k, _ in _lib.DeviceInfo._fields_}
        out["plans"] = [p for p in (PLAN_SEGMENT, PLAN_ROWS, PLAN_BAND, PLAN_HYBRID) if i.plans & (1 << p)]
        return out

    def download(self) -> VCSRMC:
        """The SEGMENT arrays back on the host (FP16 formats: values as stored, rounded to fp16)."""
        h = ctypes.c_void_p()
        call("vcsrmc_device_download", self._h, ctypes.byref(h))
        return VCSRMC(h)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def free(self) -> None:
        h, self._h = self._h, None
        if h:
            call("vcsrmc_device_free", h)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def status(self, clear: bool = False) -> int:
        f = ctypes.c_uint32()
        call("vcsrmc_device_status", self._h, ctypes.byref(f), 1 if clear else 0)
        return f.value


def _upload_options(plans, rows_unit_nnz: int, band_rows: int, hot_rows: int, hot_budget_mib: int,
                    hot_persist: int, hot_evict_first: int) -> "_lib.UploadOptions":
    opts = _lib.UploadOptions()
    opts.plans = 0 if plans is None else sum(1 << p for p in set(plans))
    opts.rows_unit_nnz = rows_unit_nnz
    opts.band_rows = band_rows
    opts.hot_rows = hot_rows
    opts.hot_budget_mib = hot_budget_mib
    opts.hot_persist = hot_persist
    opts.hot_evict_first = hot_evict_first
    return opts


def upload_vcsr_mc_device(V: VCSRMC, device: int = 0, stream=None, plans=None,
                          rows_unit_nnz: int = 0, band_rows: int = 0, hot_rows: int = 0, hot_budget_mib: int = 0,
                          hot_persist: int = 0, hot_evict_first: int = 0) -> DeviceVCSRMC:
    """Copies the format to `device`. plans: iterable of PLAN_SEGMENT / PLAN_ROWS / PLAN_BAND /
    PLAN_HYBRID layouts to make resident (default: SEGMENT and ROWS, plus BAND for FP16 formats whose
    column tiles are dense enough; BAND and HYBRID need the FP16 format). rows_unit_nnz: entries per ROWS-plan work unit (0 = the library's
    choice for this matrix). band_rows: rows per BAND-plan band, 1 .. 128 (0 = chosen).
    hot_rows / hot_budget_mib / hot_persist / hot_evict_first: the ROWS plan's hot columns, off by
    default (vcsrmc_upload_options)."""
    opts = _upload_options(plans, rows_unit_nnz, band_rows, hot_rows, hot_budget_mib, hot_persist, hot_evict_first)
    h = ctypes.c_void_p()
    call("vcsrmc_upload_opts", V.handle, device, ctypes.byref(opts), _stream_handle(stream), ctypes.byref(h))
    return DeviceVCSRMC(h, V, device)


def build_vcsr_mc_device(row_ptr, col, val, M: int, N: int, fp32: bool = False, segw: int = 16, device: int = 0,
                         stream=None, plans=None, rows_unit_nnz: int = 0, band_rows: int = 0, hot_rows: int = 0,
                         hot_budget_mib: int = 0, hot_persist: int = 0, hot_evict_first: int = 0) -> DeviceVCSRMC:
    """Builds the format on the GPU from a CSR already in device memory (torch tensors: int32
    row_ptr[M+1], int32 col[nnz], float32 val[nnz], rows with strictly ascending columns) and
    keeps its plan layouts resident there. Equal-count rows of a segment come in ascending row
    order (see vcsrmc_build_device)."""
    import torch
    for t, dt in ((row_ptr, torch.int32), (col, torch.int32), (val, torch.float32)):
        if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == dt and t.is_contiguous()):
            raise VcsrmcError(_lib.INVALID_ARG, "row_ptr/col/val must be contiguous CUDA tensors (int32, int32, float32)")
    opts = _upload_options(plans, rows_unit_nnz, band_rows, hot_rows, hot_budget_mib, hot_persist, hot_evict_first)
    h = ctypes.c_void_p()
    call("vcsrmc_build_device", M, N, int(col.numel()), ctypes.c_void_p(row_ptr.data_ptr()),
         ctypes.c_void_p(col.data_ptr()), ctypes.c_void_p(val.data_ptr()), 1 if fp32 else 0, segw, device,
         ctypes.byref(opts), _stream_handle(stream), ctypes.byref(h))
    info = _lib.DeviceInfo()
    call("vcsrmc_device_info_get", h, ctypes.byref(info))
    return DeviceVCSRMC(h, None, device, M=M, N=N, fp32=fp32, scale=float(info.scale), segw=segw)


def destroy_vcsr_mc_device(dV: DeviceVCSRMC) -> None:
    dV.free()


def _b_args(B):
    import torch
    if B.dtype == torch.float16:
        return F16
    if B.dtype == torch.float32:
        return F32
    raise VcsrmcError(_lib.INVALID_ARG, f"B must be float16 or float32, got {B.dtype}")


def _check_dense(B, C, O):
    import torch
    if not (B.is_cuda and C.is_cuda) or C.dtype != torch.float32:
        raise VcsrmcError(_lib.INVALID_ARG, "B and C must be CUDA tensors, C float32")
    if B.dim() != 2 or C.dim() != 2 or B.stride(1) != 1 or C.stride(1) != 1 or B.shape[1] < O or C.shape[1] < O:
        raise VcsrmcError(_lib.INVALID_ARG, "B and C must be 2-D row-major with >= O columns")


def spmm(dV: DeviceVCSRMC, B, C, tileK: int = 128, accumulate: bool = False, stream=None, O: Optional[int] = None,
         plan: int = PLAN_AUTO):
    """C[:, :O] (+)= A * B[:, :O] on the GPU, asynchronous on `stream` (default: torch's current)."""
    O = int(B.shape[1]) if O is None else O
    _check_dense(B, C, O)
    call("vcsrmc_spmm_ex", dV.handle, ctypes.c_void_p(B.data_ptr()), _b_args(B), B.stride(0), O, tileK,
         ctypes.c_void_p(C.data_ptr()), C.stride(0), 1 if accumulate else 0, plan, _stream_handle(stream))
    return C


def run_vcsr_mc_spmm_gpu(dV: DeviceVCSRMC, B, O: int, tileK: int, C, stream=None, accumulate: bool = True) -> float:
    """Blocking, event-timed launch with the reference's C += A*B contract; returns ms."""
    _check_dense(B, C, O)
    ms = ctypes.c_float()
    call("vcsrmc_spmm_timed", dV.handle, ctypes.c_void_p(B.data_ptr()), _b_args(B), B.stride(0), O, tileK,
         ctypes.c_void_p(C.data_ptr()), C.stride(0), 1 if accumulate else 0, _stream_handle(stream),
         ctypes.byref(ms))
    return ms.value


def gen_dense_host(rows: int, cols: int, seed: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.float32)
    call("vcsrmc_gen_dense_host", rows, cols, seed, _ptr(out), nthreads)
    return out


def gen_dense_device(out, seed: int, stream=None):
    """Fills a 2-D CUDA tensor (float32 or float16) with the dense U(-1,1) stream."""
    dt = _b_args(out)
    call("vcsrmc_gen_dense_device", int(out.shape[0]), int(out.shape[1]), seed, dt,
         ctypes.c_void_p(out.data_ptr()), out.stride(0), _stream_handle(stream))
    return out


# Row weight of the multi-GPU partition that the benchmark and the sharded path use: a block's
# cost is nnz + SHARD_ROW_WEIGHT * rows. It is the ratio of the per-row to the per-entry cost of the
# ROWS plan fitted (least squares) to 56 measured shard times of the 2^24-row R-MAT: 0.118 ns per row
# (the C row store and the row bookkeeping) against 0.0312 ns per entry.
SHARD_ROW_WEIGHT = 3.8


def partition_rows(row_ptr: np.ndarray, parts: int, row_weight: float = 0.0) -> np.ndarray:
    """parts+1 row cuts balancing nnz + row_weight * rows per block (0: pure nnz balance)."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int32)
    cuts = np.empty(parts + 1, dtype=np.int32)
    if row_weight == 0.0:
        call("vcsrmc_partition_rows", _ptr(rp), int(rp.size - 1), parts, _ptr(cuts))
    else:
        call("vcsrmc_partition_rows_weighted", _ptr(rp), int(rp.size - 1), parts, float(row_weight), _ptr(cuts))
    return cuts
