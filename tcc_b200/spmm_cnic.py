"""Drop-in for the reference's pybind module ``spmm_cnic``
(TAC_training_backend/spmm_cnic/src/bindings/module.cu:100-365).

Same function names, argument order and meaning.  Differences, all on the safe
side: the work runs on torch's current stream (the reference launches on two
private streams and never joins them back, module.cu:13-16); outputs are fresh
tensors unless a ``denseC`` buffer from :func:`space_malloc` is passed, in which
case the result is written into it and a view is returned, as the reference
does; pointer arguments the reference passes as PyCapsules are taken as plain
integers (device / unified addresses) or tensors.

forward_tensorcore_mixed with ``x`` given computes from the dense ``x`` (the
compiled reference's ``use_global_memory_access`` branch, module.cu:18-19, 94-189);
with ``x=None`` it gathers from the hot/cold feature store (the
``use_mixed_memory_access`` branch, module.cu:21-92).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from . import tiles as T

_buffers: dict = {}


def _ptr_of(v):
    if v is None:
        return None
    if isinstance(v, int):
        return C.c_void_p(v)
    if isinstance(v, torch.Tensor):
        return C.c_void_p(v.data_ptr())
    if isinstance(v, (list, tuple)):  # per-GPU feature shards -> device pointer table
        table = torch.tensor([t.data_ptr() for t in v], dtype=torch.int64,
                             device=torch.device("cuda", torch.cuda.current_device()))
        _buffers.setdefault("_tables", []).append(table)
        return C.c_void_p(table.data_ptr())
    raise TypeError(f"unsupported pointer argument {type(v)}")


def _parts(bcsr_args, bcsc_args):
    r = T.from_arrays("bcsr", *bcsr_args) if bcsr_args[3] and bcsr_args[4] else None
    c = T.from_arrays("bcsc", *bcsc_args) if bcsc_args[3] and bcsc_args[4] else None
    return r, c


def _out(num_rows, F, device, denseC):
    W = (num_rows + 7) // 8
    need = (W + 1) * 8 * F
    if denseC is not None:
        if denseC.numel() < need or denseC.dtype != torch.float32:
            raise ValueError(f"denseC holds {denseC.numel()} floats, needs {need}")
        return denseC.view(-1)[:need]
    return torch.empty(need, dtype=torch.float32, device=device)


def _scratch(parts):
    r = parts[0]
    if r is None:
        return None, 0
    n = L.lib().tcc_pull_scratch_bytes(r.num_windows, r.num_TCBlocks)
    buf = torch.empty(n, dtype=torch.uint8, device=r.windowOffset.device)
    return buf, n


def _structs(parts):
    r, c = parts
    return (C.byref(r.struct()) if r is not None else None,
            C.byref(c.struct()) if c is not None else None)


def forward_tensorcore(bcsr_num_rows, bcsr_num_cols, bcsr_nnz, bcsr_num_TCBlocks,
                       bcsr_num_rowWindows, bcsr_rowWindowOffset, bcsr_tcOffset, bcsr_sparseA2B,
                       bcsr_tcLocalBit, bcsc_num_rows, bcsc_num_cols, bcsc_nnz,
                       bcsc_num_TCBlocks, bcsc_num_colWindows, bcsc_colWindowOffset,
                       bcsc_tcOffset, bcsc_sparseA2C, bcsc_tcLocalBit, feature_dim, x,
                       device_id=None, denseC=None, tc_threshold: int = 0):
    """C = BCSR*x + BCSC*x (module.cu:192-273 -> launch_spmm_kernel,
    spmm_launcher.cu:203-271); returns the first num_rows*feature_dim floats."""
    if device_id is not None:
        torch.cuda.set_device(device_id)
    parts = _parts((bcsr_num_rows, bcsr_num_cols, bcsr_nnz, bcsr_num_TCBlocks, bcsr_num_rowWindows,
                    bcsr_rowWindowOffset, bcsr_tcOffset, bcsr_sparseA2B, bcsr_tcLocalBit),
                   (bcsc_num_rows, bcsc_num_cols, bcsc_nnz, bcsc_num_TCBlocks, bcsc_num_colWindows,
                    bcsc_colWindowOffset, bcsc_tcOffset, bcsc_sparseA2C, bcsc_tcLocalBit))
    F = int(feature_dim)
    rows = int(bcsr_num_rows)
    x = x.contiguous().view(-1, F) if x.dim() == 1 else x.contiguous()
    out = _out(rows, F, x.device, denseC)
    if parts == (None, None):
        out.zero_()
        return out[: rows * F]
    sc, n = _scratch(parts)
    pr, pc = _structs(parts)
    L.call("tcc_cnic_forward", pr, pc, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), F,
           tc_threshold, None if sc is None else C.c_void_p(sc.data_ptr()), n,
           C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return out[: rows * F]


def forward_tensorcore_mixed(bcsr_num_rows, bcsr_num_cols, bcsr_nnz, bcsr_num_TCBlocks,
                             bcsr_num_rowWindows, bcsr_rowWindowOffset, bcsr_tcOffset,
                             bcsr_sparseA2B, bcsr_tcLocalBit, bcsc_num_rows, bcsc_num_cols,
                             bcsc_nnz, bcsc_num_TCBlocks, bcsc_num_colWindows,
                             bcsc_colWindowOffset, bcsc_tcOffset, bcsc_sparseA2C,
                             bcsc_tcLocalBit, cpu_float_feature_len, gpu_node_capacity,
                             feature_dim, id_map, cpu_feature_cache_ptr, cache_search_map,
                             gpu_feature_cache_ptr, x=None, device_id=None, denseC=None,
                             tc_threshold: int = 0):
    """First-layer aggregation (module.cu:21-189): rows of condensed columns come
    from the hot/cold feature store (x=None) or from the dense x."""
    if x is not None:
        return forward_tensorcore(bcsr_num_rows, bcsr_num_cols, bcsr_nnz, bcsr_num_TCBlocks,
                                  bcsr_num_rowWindows, bcsr_rowWindowOffset, bcsr_tcOffset,
                                  bcsr_sparseA2B, bcsr_tcLocalBit, bcsc_num_rows, bcsc_num_cols,
                                  bcsc_nnz, bcsc_num_TCBlocks, bcsc_num_colWindows,
                                  bcsc_colWindowOffset, bcsc_tcOffset, bcsc_sparseA2C,
                                  bcsc_tcLocalBit, feature_dim, x, device_id, denseC,
                                  tc_threshold)
    if device_id is not None:
        torch.cuda.set_device(device_id)
    parts = _parts((bcsr_num_rows, bcsr_num_cols, bcsr_nnz, bcsr_num_TCBlocks, bcsr_num_rowWindows,
                    bcsr_rowWindowOffset, bcsr_tcOffset, bcsr_sparseA2B, bcsr_tcLocalBit),
                   (bcsc_num_rows, bcsc_num_cols, bcsc_nnz, bcsc_num_TCBlocks, bcsc_num_colWindows,
                    bcsc_colWindowOffset, bcsc_tcOffset, bcsc_sparseA2C, bcsc_tcLocalBit))
    F = int(feature_dim)
    rows = int(bcsr_num_rows)
    dev = torch.device("cuda", torch.cuda.current_device())
    out = _out(rows, F, dev, denseC)
    if parts == (None, None):
        out.zero_()
        return out[: rows * F]
    sc, n = _scratch(parts)
    pr, pc = _structs(parts)
    L.call("tcc_cnic_forward_mixed", pr, pc, _ptr_of(id_map), _ptr_of(cpu_feature_cache_ptr),
           _ptr_of(cache_search_map), _ptr_of(gpu_feature_cache_ptr), int(gpu_node_capacity),
           C.c_void_p(out.data_ptr()), F, tc_threshold,
           None if sc is None else C.c_void_p(sc.data_ptr()), n,
           C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return out[: rows * F]


def initialize(device_id):
    """module.cu:299-304 creates two streams; here work follows torch's stream."""
    torch.cuda.set_device(device_id)


def space_malloc(device_id, denseC_size):
    """Two zeroed float buffers of denseC_size (module.cu:306-327)."""
    torch.cuda.set_device(device_id)
    bufs = [torch.zeros(int(denseC_size), dtype=torch.float32, device=f"cuda:{device_id}")
            for _ in range(2)]
    _buffers.setdefault(device_id, []).extend(bufs)
    return bufs


def finalize(device_id):
    """Release what space_malloc handed out on this device (module.cu:329-341)."""
    _buffers.pop(device_id, None)
    _buffers.pop("_tables", None)


def read_cpu_feature_cache(cpu_feature_cache, cpu_feature_len):
    """Debug print of the host feature cache (module.cu:276-285)."""
    t = cpu_feature_cache if isinstance(cpu_feature_cache, torch.Tensor) else None
    if t is None:
        raise TypeError("pass the pinned host feature tensor")
    print("h_cpu_feature_cache: {", ", ".join(f"{v:f}" for v in t.view(-1)[:cpu_feature_len].tolist()), "}")


def read_gpu0_feature_cache(gpu_feature_cache):
    """Debug print of the first 100 values of GPU shard 0 (module.cu:287-297)."""
    t = gpu_feature_cache[0] if isinstance(gpu_feature_cache, (list, tuple)) else gpu_feature_cache
    print("gpu feature: {", ", ".join(f"{v:f}" for v in t.view(-1)[:100].tolist()), "}")
