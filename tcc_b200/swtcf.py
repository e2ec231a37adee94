"""SWTCF (super-window tensor-core format) conversion and SpMM on torch tensors.

Mirrors the reference's C++ SWTCF interface (include/swtcf_convert.cuh:74-78,
include/swtcf_spmm.cuh:10-26) over the C ABI of include/tcc_b200.h; the
reference names are kept as aliases (allocateDeviceSWTCF, convertCOOToSWTCF,
launchSWTCFSpMM ...).  Everything runs on the current CUDA device and torch's
current stream; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L

DEFAULT_TC_THRESHOLD = 12
FEATURE_DIM = 128


def _stream(stream=None):
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return C.c_void_p(t.data_ptr())


def _check_f32(t, name):
    if t.dtype != torch.float32 or not t.is_cuda:
        raise TypeError(f"{name} must be a float32 CUDA tensor")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with unit column stride")


class _DeviceView:
    """__cuda_array_interface__ over a raw device pointer (no copy)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (int(ptr or 0), False), "version": 3}


def device_array(ptr: int, n: int, dtype) -> torch.Tensor:
    """A torch view of n elements of a device array (uint32 -> int32, uint64 -> int64)."""
    dt = np.dtype(dtype)
    typestr = {1: "|u1", 4: "<i4", 8: "<i8"}[dt.itemsize]
    if n == 0:
        return torch.empty(0, dtype={1: torch.uint8, 4: torch.int32, 8: torch.int64}[dt.itemsize],
                           device="cuda")
    return torch.as_tensor(_DeviceView(ptr, n, typestr), device="cuda")


class SWTCFMatrix:
    """Owning handle of a device SWTCF matrix (the reference DeviceSWTCFMatrix,
    include/swtcf_convert.cuh:13-35); arrays are sized by nnz like the
    reference's allocateDeviceSWTCF (src/swtcf_convert.cu:1113-1263)."""

    def __init__(self, rows: int, cols: int, nnz: int, super_window_size: int = 16):
        self.c = L.Swtcf()
        self._device = torch.cuda.current_device()
        L.call("tcc_swtcf_alloc", C.byref(self.c), rows, cols, nnz, super_window_size)
        self._live = True

    def free(self):
        if getattr(self, "_live", False):
            with torch.cuda.device(self._device):
                L.call("tcc_swtcf_free", C.byref(self.c))
            self._live = False

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def rows(self):
        return self.c.rows

    @property
    def cols(self):
        return self.c.cols

    @property
    def num_col_windows(self):
        return self.c.numColWindows

    @property
    def num_super_windows(self):
        return self.c.numSuperWindows

    def sizes(self, stream=None):
        """(T, R): tiles and super-window rows (synchronises)."""
        t, r = C.c_uint64(), C.c_uint64()
        L.call("tcc_swtcf_sizes", C.byref(self.c), _stream(stream), C.byref(t), C.byref(r))
        return t.value, r.value

    def to_host(self, stream=None) -> dict:
        """All arrays as numpy, trimmed to T / R (the compared extents)."""
        T, R = self.sizes(stream)
        W, SW = self.c.numColWindows, self.c.numSuperWindows

        def dl(ptr, n, dtype):
            return device_array(ptr, n, dtype).cpu().numpy().view(dtype)

        c = self.c
        return dict(
            rows=c.rows, cols=c.cols, S=c.superWindowSize, numColWindows=W, numSuperWindows=SW,
            T=T, R=R,
            colWindowOffset=dl(c.colWindowOffset, W + 1, np.uint32),
            tileLocalBit=dl(c.tileLocalBit, T, np.uint64),
            tileRowSlot=dl(c.tileRowSlot, 8 * T, np.uint32),
            superWindowRowOffset=dl(c.superWindowRowOffset, SW + 1, np.uint32),
            superWindowRows=dl(c.superWindowRows, R, np.uint32),
            superWindowRowCacheSlot=dl(c.superWindowRowCacheSlot, R, np.uint8),
            superWindowCachedRowSlot=dl(c.superWindowCachedRowSlot, 32 * SW, np.uint32),
            superWindowCachedCount=dl(c.superWindowCachedCount, SW, np.uint8))


class SWTCFConvertWorkspace:
    """The converter's scratch (reference SWTCFConvertWorkspace,
    src/swtcf_convert.cu:1306-1655)."""

    def __init__(self, edge_capacity: int, num_src: int, super_window_size: int = 16):
        self.h = C.c_void_p()
        self._device = torch.cuda.current_device()
        L.call("tcc_swtcf_workspace_create", C.byref(self.h), edge_capacity, num_src,
               super_window_size)

    def free(self):
        if self.h:
            with torch.cuda.device(self._device):
                L.call("tcc_swtcf_workspace_destroy", self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def device_error(self, stream=None) -> int:
        code = C.c_uint32()
        L.call("tcc_swtcf_workspace_device_error", self.h, _stream(stream), C.byref(code))
        return code.value


def convert_coo(dst: torch.Tensor, src: torch.Tensor, m: SWTCFMatrix, ws: SWTCFConvertWorkspace,
                stream=None):
    """convertCOOToSWTCF (src/swtcf_convert.cu:1754-2342): canonical tiles of the
    COO (dst[e], src[e]) (int32/uint32 CUDA tensors)."""
    if dst.numel() != src.numel():
        raise ValueError("dst and src differ in length")
    for t in (dst, src):
        if t.element_size() != 4 or not t.is_contiguous():
            raise TypeError("dst/src must be contiguous 32-bit CUDA tensors")
    L.call("tcc_swtcf_convert_coo", _ptr(dst), _ptr(src), dst.numel(), C.byref(m.c), ws.h,
           _stream(stream))


def convert_csr(rowptr: torch.Tensor, col: torch.Tensor, m: SWTCFMatrix,
                ws: SWTCFConvertWorkspace, stream=None):
    """CSR entry of the conversion (rowptr int64, col int32; row = dst)."""
    if rowptr.dtype != torch.int64 or col.element_size() != 4:
        raise TypeError("rowptr must be int64 and col 32-bit")
    L.call("tcc_swtcf_convert_csr", _ptr(rowptr), _ptr(col), rowptr.numel() - 1, col.numel(),
           C.byref(m.c), ws.h, _stream(stream))


def prepare_pull(m: SWTCFMatrix, stream=None):
    """Build the converted matrix's row-window tiling (no reference
    counterpart; allocates, synchronises).  Until the next conversion,
    ``spmm`` and ``spmm_ex`` run the forward product as a pull over row windows
    instead of the push over column windows."""
    L.call("tcc_swtcf_prepare_pull", C.byref(m.c), _stream(stream))


def spmm(m: SWTCFMatrix, X: torch.Tensor, Y: torch.Tensor,
         tc_threshold: int = DEFAULT_TC_THRESHOLD, stream=None):
    """launchSWTCFSpMM (src/swtcf_spmm.cu:437-466): Y[rows x 128] += A X[cols x 128]."""
    for t, nm in ((X, "X"), (Y, "Y")):
        _check_f32(t, nm)
        if t.shape[1] != FEATURE_DIM or t.stride(0) != FEATURE_DIM:
            raise ValueError(f"{nm} must be contiguous with {FEATURE_DIM} columns")
    L.call("tcc_swtcf_spmm", C.byref(m.c), _ptr(X), _ptr(Y), tc_threshold, _stream(stream))


def spmm_quantized(m: SWTCFMatrix, q_x: torch.Tensor, scales: torch.Tensor, src_global, Y: torch.Tensor,
                   tc_threshold: int = DEFAULT_TC_THRESHOLD, stream=None):
    """launchSWTCFSpMMQuantized (src/swtcf_spmm.cu:268-432, 469-502): Y += A Xq
    with source column c reading int8 row q_x[src_global[c]] times
    scales[src_global[c]] (src_global None: identity)."""
    if q_x.dtype != torch.int8 or not q_x.is_cuda or q_x.shape[1] != FEATURE_DIM or \
            q_x.stride(0) != FEATURE_DIM:
        raise ValueError(f"q_x must be a contiguous CUDA int8 tensor with {FEATURE_DIM} columns")
    if scales.dtype != torch.float32 or not scales.is_cuda or scales.dim() != 1 or \
            not scales.is_contiguous() or scales.numel() < q_x.shape[0]:
        raise ValueError("scales must be a contiguous CUDA float32 vector with one entry per q_x row")
    _check_f32(Y, "Y")
    if Y.shape[1] != FEATURE_DIM or Y.stride(0) != FEATURE_DIM:
        raise ValueError(f"Y must be contiguous with {FEATURE_DIM} columns")
    sg = None if src_global is None else src_global
    if sg is not None and (sg.dtype != torch.int32 or not sg.is_cuda):
        raise ValueError("src_global must be a CUDA int32 (uint32 bits) tensor")
    L.call("tcc_swtcf_spmm_quantized", C.byref(m.c), _ptr(q_x), _ptr(scales), _ptr(sg), _ptr(Y),
           tc_threshold, _stream(stream))


# the reference's name
launchSWTCFSpMMQuantized = spmm_quantized


def spmm_ex(m: SWTCFMatrix, X: torch.Tensor, Y: torch.Tensor | None = None,
            tc_threshold: int = DEFAULT_TC_THRESHOLD, row_scale=None, col_scale=None,
            accumulate: bool = False, stream=None) -> torch.Tensor:
    """Y = diag(row_scale) A diag(col_scale) X for any F (multiple of 4)."""
    _check_f32(X, "X")
    F = X.shape[1]
    if Y is None:
        Y = torch.empty((m.rows, F), dtype=torch.float32, device=X.device)
        accumulate = False
    _check_f32(Y, "Y")
    L.call("tcc_swtcf_spmm_ex", C.byref(m.c), _ptr(X), X.stride(0), _ptr(Y), Y.stride(0), F,
           tc_threshold, _ptr(row_scale), _ptr(col_scale), int(accumulate), _stream(stream))
    return Y


def spmm_t(m: SWTCFMatrix, G: torch.Tensor, Z: torch.Tensor | None = None,
           tc_threshold: int = DEFAULT_TC_THRESHOLD, row_scale=None, col_scale=None,
           accumulate: bool = False, stream=None) -> torch.Tensor:
    """Z = diag(col_scale) A^T diag(row_scale) G over the same tiles."""
    _check_f32(G, "G")
    F = G.shape[1]
    if Z is None:
        Z = torch.empty((m.cols, F), dtype=torch.float32, device=G.device)
        accumulate = False
    _check_f32(Z, "Z")
    L.call("tcc_swtcf_spmm_t", C.byref(m.c), _ptr(G), G.stride(0), _ptr(Z), Z.stride(0), F,
           tc_threshold, _ptr(row_scale), _ptr(col_scale), int(accumulate), _stream(stream))
    return Z


# reference names (include/swtcf_convert.cuh:74-78, include/swtcf_spmm.cuh:10-16)
allocateDeviceSWTCF = SWTCFMatrix
allocateSWTCFConvertWorkspace = SWTCFConvertWorkspace
convertCOOToSWTCF = convert_coo
launchSWTCFSpMM = spmm
