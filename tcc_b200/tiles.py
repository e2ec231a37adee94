"""BCSR / BCSC window tiles (the spmm_cnic formats) on torch tensors.

The tiles mirror BCSR<float> / BCSC<float> (cnic/include/class.h:20-57, where
cnic/ is TAC_training_backend/spmm_cnic/): 8-row (BCSR) or 8-column (BCSC)
windows whose distinct columns / rows are condensed in ascending order into 8x8
tiles with a 64-bit bitmap each.  Index arrays are held as int32 tensors with
the reference's uint32 bit patterns (padding 0xFFFFFFFF reads as -1), bitmaps as
int64.  Conversion and SpMM run through the C ABI (include/tcc_b200.h).
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import torch

from . import _lib as L
from .swtcf import _ptr, _stream, _check_f32

DEFAULT_TC_THRESHOLD = 12


@dataclasses.dataclass
class Tiles:
    """One BCSR (kind 'bcsr') or BCSC (kind 'bcsc') tiling of an A[num_rows x num_cols]."""
    kind: str
    num_rows: int
    num_cols: int
    nnz: int
    num_TCBlocks: int
    num_windows: int
    windowOffset: torch.Tensor   # rowWindowOffset / colWindowOffset, int32 [W+1]
    tcOffset: torch.Tensor       # int32 [T+1]
    sparseIdx: torch.Tensor      # sparseA2B / sparseA2C, int32 [8T]
    tcLocalBit: torch.Tensor     # int64 [T]
    _scratch: torch.Tensor | None = None
    _plan_ready: bool = False

    # reference field names
    @property
    def num_rowWindows(self):
        return self.num_windows

    @property
    def num_colWindows(self):
        return self.num_windows

    @property
    def rowWindowOffset(self):
        return self.windowOffset

    @property
    def colWindowOffset(self):
        return self.windowOffset

    @property
    def sparseA2B(self):
        return self.sparseIdx

    @property
    def sparseA2C(self):
        return self.sparseIdx

    def struct(self):
        if self.kind == "bcsr":
            s = L.Bcsr()
            s.num_rowWindows = self.num_windows
            s.rowWindowOffset = self.windowOffset.data_ptr()
            s.sparseA2B = self.sparseIdx.data_ptr()
        else:
            s = L.Bcsc()
            s.num_colWindows = self.num_windows
            s.colWindowOffset = self.windowOffset.data_ptr()
            s.sparseA2C = self.sparseIdx.data_ptr()
        s.num_rows, s.num_cols, s.nnz = self.num_rows, self.num_cols, self.nnz
        s.num_TCBlocks = self.num_TCBlocks
        s.tcOffset = self.tcOffset.data_ptr()
        s.tcLocalBit = self.tcLocalBit.data_ptr()
        return s

    def scratch(self):
        """Pull-plan scratch owned by this tiling (built on first use)."""
        if self._scratch is None:
            n = L.lib().tcc_pull_scratch_bytes(self.num_windows, self.num_TCBlocks)
            self._scratch = torch.empty(n, dtype=torch.uint8, device=self.windowOffset.device)
            self._plan_ready = False
        return self._scratch

    def to_host(self) -> dict:
        """numpy views with the reference dtypes (uint32 / uint64)."""
        import numpy as np
        key_off = "rowWindowOffset" if self.kind == "bcsr" else "colWindowOffset"
        key_idx = "sparseA2B" if self.kind == "bcsr" else "sparseA2C"
        key_w = "num_rowWindows" if self.kind == "bcsr" else "num_colWindows"
        return {
            "num_rows": self.num_rows, "num_cols": self.num_cols, "nnz": self.nnz,
            "num_TCBlocks": self.num_TCBlocks, key_w: self.num_windows,
            key_off: self.windowOffset.cpu().numpy().view(np.uint32),
            "tcOffset": self.tcOffset.cpu().numpy().view(np.uint32),
            key_idx: self.sparseIdx.cpu().numpy().view(np.uint32),
            "tcLocalBit": self.tcLocalBit.cpu().numpy().view(np.uint64),
        }


class TilesWorkspace:
    """Scratch of the CSR -> BCSR/BCSC conversion (sort + group buffers)."""

    def __init__(self, nnz_capacity: int, rows: int, cols: int):
        self.h = C.c_void_p()
        self._device = torch.cuda.current_device()
        L.call("tcc_tiles_workspace_create", C.byref(self.h), nnz_capacity, rows, cols)
        self.nnz_capacity, self.rows, self.cols = nnz_capacity, rows, cols

    def free(self):
        if self.h:
            with torch.cuda.device(self._device):
                L.call("tcc_tiles_workspace_destroy", self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def from_csr(rowptr: torch.Tensor, col: torch.Tensor, num_rows: int, num_cols: int,
             kind: str = "bcsr", ws: TilesWorkspace | None = None, stream=None) -> Tiles:
    """Canonical BCSR or BCSC tiles of a CSR (rowptr int64 [rows+1], col int32 [nnz])."""
    if rowptr.dtype != torch.int64 or col.element_size() != 4:
        raise TypeError("rowptr must be int64 and col 32-bit")
    if not (rowptr.is_cuda and col.is_cuda):
        raise ValueError("CSR must be on the GPU")
    nnz = col.numel()
    own = ws is None
    if own:
        ws = TilesWorkspace(max(nnz, 1), num_rows, num_cols)
    k = L.TILES_BCSR if kind == "bcsr" else L.TILES_BCSC
    T = C.c_uint64()
    L.call("tcc_tiles_prepare_csr", ws.h, k, _ptr(rowptr), _ptr(col) if nnz else None, num_rows,
           num_cols, nnz, _stream(stream), C.byref(T))
    T = T.value
    W = (num_rows + 7) // 8 if kind == "bcsr" else (num_cols + 7) // 8
    dev = rowptr.device
    t = Tiles(kind, num_rows, num_cols, nnz, T, W,
              torch.empty(W + 1, dtype=torch.int32, device=dev),
              torch.empty(T + 1, dtype=torch.int32, device=dev),
              torch.empty(max(8 * T, 1), dtype=torch.int32, device=dev),
              torch.empty(max(T, 1), dtype=torch.int64, device=dev))
    s = t.struct()
    L.call("tcc_tiles_fill_bcsr" if kind == "bcsr" else "tcc_tiles_fill_bcsc", ws.h, C.byref(s),
           _stream(stream))
    if own:
        torch.cuda.current_stream().synchronize()
        ws.free()
    return t


def from_arrays(kind: str, num_rows: int, num_cols: int, nnz: int, num_TCBlocks: int,
                num_windows: int, windowOffset, tcOffset, sparseIdx, tcLocalBit) -> Tiles:
    """Wrap caller-provided tile tensors (e.g. the reference's sampler output)."""
    def i32(x):
        return x if x.dtype == torch.int32 else x.view(torch.int32) if x.element_size() == 4 \
            else x.to(torch.int32)
    return Tiles(kind, int(num_rows), int(num_cols), int(nnz), int(num_TCBlocks),
                 int(num_windows), i32(windowOffset).contiguous(), i32(tcOffset).contiguous(),
                 i32(sparseIdx).contiguous(), tcLocalBit.view(torch.int64).contiguous())


def bcsr_spmm(a: Tiles, B: torch.Tensor, C_out: torch.Tensor | None = None,
              tc_threshold: int = DEFAULT_TC_THRESHOLD, rs=None, cs=None,
              accumulate: bool = False, stream=None) -> torch.Tensor:
    """C = diag(rs) A diag(cs) B with A as BCSR tiles (pull, owner-computes)."""
    assert a.kind == "bcsr"
    _check_f32(B, "B")
    F = B.shape[1]
    if C_out is None:
        C_out = torch.empty((a.num_rows, F), dtype=torch.float32, device=B.device)
        accumulate = False
    _check_f32(C_out, "C")
    sc = a.scratch()
    s = a.struct()
    L.call("tcc_bcsr_spmm", C.byref(s), _ptr(B), B.stride(0), _ptr(C_out), C_out.stride(0), F,
           tc_threshold, _ptr(rs), _ptr(cs), int(accumulate), _ptr(sc), sc.numel(),
           int(a._plan_ready), _stream(stream))
    a._plan_ready = True
    return C_out


def pull_device_error(a: Tiles, stream=None) -> int:
    """Device error word of the tiling's pull scratch (0, or
    TCC_DEVERR_WAIT_TIMEOUT when a pull kernel gave up waiting on one of its
    TMA copies); synchronises the stream and clears the word."""
    if a._scratch is None:
        return 0
    code = C.c_int(0)
    L.call("tcc_pull_device_error", _ptr(a._scratch), C.byref(code), _stream(stream))
    return code.value


def bcsr_spmm_t(a: Tiles, G: torch.Tensor, Z: torch.Tensor,
                tc_threshold: int = DEFAULT_TC_THRESHOLD, rs=None, cs=None, stream=None):
    """Z += diag(cs) A^T diag(rs) G with A as BCSR tiles (push over row windows)."""
    assert a.kind == "bcsr"
    _check_f32(G, "G")
    _check_f32(Z, "Z")
    s = a.struct()
    L.call("tcc_bcsr_spmm_t", C.byref(s), _ptr(G), G.stride(0), _ptr(Z), Z.stride(0),
           G.shape[1], tc_threshold, _ptr(rs), _ptr(cs), _stream(stream))
    return Z


def bcsc_spmm(a: Tiles, B: torch.Tensor, C_out: torch.Tensor,
              tc_threshold: int = DEFAULT_TC_THRESHOLD, rs=None, cs=None, stream=None):
    """C += diag(rs) A diag(cs) B with A as BCSC tiles (push, vector reductions)."""
    assert a.kind == "bcsc"
    _check_f32(B, "B")
    _check_f32(C_out, "C")
    s = a.struct()
    L.call("tcc_bcsc_spmm", C.byref(s), _ptr(B), B.stride(0), _ptr(C_out), C_out.stride(0),
           B.shape[1], tc_threshold, _ptr(rs), _ptr(cs), _stream(stream))
    return C_out


def bcsc_spmm_t(a: Tiles, G: torch.Tensor, Z: torch.Tensor | None = None,
                tc_threshold: int = DEFAULT_TC_THRESHOLD, rs=None, cs=None,
                accumulate: bool = False, stream=None) -> torch.Tensor:
    """Z = diag(cs) A^T diag(rs) G with A as BCSC tiles (pull per column window)."""
    assert a.kind == "bcsc"
    _check_f32(G, "G")
    F = G.shape[1]
    if Z is None:
        Z = torch.empty((a.num_cols, F), dtype=torch.float32, device=G.device)
        accumulate = False
    _check_f32(Z, "Z")
    sc = a.scratch()
    s = a.struct()
    L.call("tcc_bcsc_spmm_t", C.byref(s), _ptr(G), G.stride(0), _ptr(Z), Z.stride(0), F,
           tc_threshold, _ptr(rs), _ptr(cs), int(accumulate), _ptr(sc), sc.numel(),
           int(a._plan_ready), _stream(stream))
    a._plan_ready = True
    return Z
