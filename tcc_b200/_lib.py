"""ctypes binding of tcc_b200/libtcc_b200.so (the C ABI of include/tcc_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.  Build it with ``python -m tcc_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtcc_b200.so")

TCC_OK = 0
STATUS_NAMES = {0: "TCC_OK", 1: "TCC_ERR_INVALID_ARGUMENT", 2: "TCC_ERR_CUDA",
                3: "TCC_ERR_OUT_OF_MEMORY", 4: "TCC_ERR_UNSUPPORTED", 5: "TCC_ERR_DEVICE",
                6: "TCC_ERR_CAPACITY"}
NOALLOC_SCRATCH_BYTES = 16 << 20  # TCC_NOALLOC_SCRATCH_BYTES
TILES_BCSR = 0
TILES_BCSC = 1
DEVERR_GROUP_DEGREE = 1
DEVERR_INDEX_RANGE = 5
DEVERR_WAIT_TIMEOUT = 6
DEFAULT_WAIT_LIMIT_NS = 2_000_000_000  # TCC_DEFAULT_WAIT_LIMIT_NS


class TccError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Swtcf(C.Structure):
    """Field-for-field tcc_swtcf / the reference's DeviceSWTCFMatrix."""
    _fields_ = [("rows", C.c_uint32), ("cols", C.c_uint32), ("nnz", C.c_uint32),
                ("colWindowWidth", C.c_uint32), ("tileRows", C.c_uint32),
                ("superWindowSize", C.c_uint32), ("numColWindows", C.c_uint32),
                ("numSuperWindows", C.c_uint32),
                ("superWindowRowOffset", C.c_void_p), ("superWindowRows", C.c_void_p),
                ("superWindowRowCacheSlot", C.c_void_p), ("superWindowCachedRowSlot", C.c_void_p),
                ("superWindowCachedCount", C.c_void_p), ("colWindowOffset", C.c_void_p),
                ("tileRowSlot", C.c_void_p), ("tileLocalBit", C.c_void_p),
                ("capacity_tiles", C.c_uint64), ("capacity_rows", C.c_uint64),
                ("pull_plan", C.c_void_p), ("pull_plan_bytes", C.c_uint64),
                ("pull_plan_ready", C.c_int32), ("fwd_ready", C.c_int32),
                ("fwdRowWindowOffset", C.c_void_p), ("fwdTcOffset", C.c_void_p),
                ("fwdSparseA2B", C.c_void_p), ("fwdTcLocalBit", C.c_void_p),
                ("fwd_tiles", C.c_uint64), ("fwd_plan", C.c_void_p),
                ("fwd_plan_bytes", C.c_uint64), ("fwd_plan_ready", C.c_int32)]


PEER_MAX_RANKS = 8    # TCC_PEER_MAX_RANKS
PEER_MAX_TAGS = 4     # TCC_PEER_MAX_TAGS
PEER_FLAGS_BYTES = 4096  # TCC_PEER_FLAGS_BYTES


class IpcHandle(C.Structure):
    """tcc_ipc_handle (a cudaIpcMemHandle_t, 64 bytes)."""
    _fields_ = [("bytes", C.c_ubyte * 64)]


class HaloPushArgs(C.Structure):
    """tcc_halo_push_args."""
    _fields_ = [("x", C.c_void_p), ("ldx", C.c_uint64), ("num_rows", C.c_uint64),
                ("send_idx", C.c_void_p), ("width", C.c_uint32), ("world", C.c_uint32),
                ("rank", C.c_uint32), ("tag", C.c_uint32), ("seq", C.c_uint32),
                ("max_blocks", C.c_uint32), ("buffers", C.c_uint32),
                ("seg", C.c_uint64 * (PEER_MAX_RANKS + 1)),
                ("dst", C.c_void_p * PEER_MAX_RANKS), ("ld_dst", C.c_uint64),
                ("peer_flags", C.c_void_p * PEER_MAX_RANKS), ("flags", C.c_void_p),
                ("wait_ns", C.c_uint64)]


class DistOperand(C.Structure):
    """tcc_dist_operand."""
    _fields_ = [("push", HaloPushArgs), ("halo", C.c_void_p), ("ld_halo", C.c_uint64),
                ("y", C.c_void_p), ("ldy", C.c_uint64)]


class DistStepArgs(C.Structure):
    """tcc_dist_step_args."""
    _fields_ = [("local", C.c_void_p), ("local_scratch", C.c_void_p),
                ("local_scratch_bytes", C.c_size_t), ("local_plan_ready", C.c_int32),
                ("halo", C.c_void_p), ("halo_scratch", C.c_void_p),
                ("halo_scratch_bytes", C.c_size_t), ("halo_plan_ready", C.c_int32),
                ("rs", C.c_void_p), ("cs_local", C.c_void_p), ("cs_halo", C.c_void_p),
                ("tc_threshold", C.c_uint32), ("recv_mask", C.c_uint32),
                ("reserve_sms", C.c_uint32), ("reserve_passes", C.c_uint32),
                ("peer_flags", C.c_void_p * PEER_MAX_RANKS), ("n_ops", C.c_uint32),
                ("ops", DistOperand * 2), ("events", C.c_void_p * 6)]


class Bcsr(C.Structure):
    """Field-for-field tcc_bcsr / the reference's BCSR<float>."""
    _fields_ = [("num_rows", C.c_uint32), ("num_cols", C.c_uint32), ("nnz", C.c_uint32),
                ("num_TCBlocks", C.c_uint32), ("num_rowWindows", C.c_uint32),
                ("rowWindowOffset", C.c_void_p), ("tcOffset", C.c_void_p),
                ("sparseA2B", C.c_void_p), ("tcLocalBit", C.c_void_p)]


class Bcsc(C.Structure):
    """Field-for-field tcc_bcsc / the reference's BCSC<float>."""
    _fields_ = [("num_rows", C.c_uint32), ("num_cols", C.c_uint32), ("nnz", C.c_uint32),
                ("num_TCBlocks", C.c_uint32), ("num_colWindows", C.c_uint32),
                ("colWindowOffset", C.c_void_p), ("tcOffset", C.c_void_p),
                ("sparseA2C", C.c_void_p), ("tcLocalBit", C.c_void_p)]


# name -> (restype, argtypes); the symbols include/tcc_b200.h declares
_vp = C.c_void_p
_u32 = C.c_uint32
_u64 = C.c_uint64
_i = C.c_int
_st = C.c_int
PROTOTYPES = {
    "tcc_last_error": (C.c_char_p, []),
    "tcc_version": (C.c_char_p, []),
    "tcc_swtcf_alloc": (_st, [C.POINTER(Swtcf), _u32, _u32, _u32, _u32]),
    "tcc_swtcf_free": (_st, [C.POINTER(Swtcf)]),
    "tcc_swtcf_workspace_create": (_st, [C.POINTER(_vp), _u64, _u32, _u32]),
    "tcc_swtcf_workspace_destroy": (_st, [_vp]),
    "tcc_swtcf_convert_coo": (_st, [_vp, _vp, _u64, C.POINTER(Swtcf), _vp, _vp]),
    "tcc_swtcf_convert_csr": (_st, [_vp, _vp, _u32, _u64, C.POINTER(Swtcf), _vp, _vp]),
    "tcc_swtcf_workspace_device_error": (_st, [_vp, _vp, C.POINTER(_u32)]),
    "tcc_swtcf_sizes": (_st, [C.POINTER(Swtcf), _vp, C.POINTER(_u64), C.POINTER(_u64)]),
    "tcc_swtcf_spmm": (_st, [C.POINTER(Swtcf), _vp, _vp, _u32, _vp]),
    "tcc_swtcf_prepare_pull": (_st, [C.POINTER(Swtcf), _vp]),
    "tcc_swtcf_spmm_quantized": (_st, [C.POINTER(Swtcf), _vp, _vp, _vp, _vp, _u32, _vp]),
    "tcc_swtcf_spmm_ex": (_st, [C.POINTER(Swtcf), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp,
                                _i, _vp]),
    "tcc_swtcf_spmm_t": (_st, [C.POINTER(Swtcf), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp, _i,
                               _vp]),
    "tcc_tiles_workspace_create": (_st, [C.POINTER(_vp), _u64, _u32, _u32]),
    "tcc_tiles_workspace_destroy": (_st, [_vp]),
    "tcc_tiles_prepare_csr": (_st, [_vp, _i, _vp, _vp, _u32, _u32, _u64, _vp, C.POINTER(_u64)]),
    "tcc_tiles_fill_bcsr": (_st, [_vp, C.POINTER(Bcsr), _vp]),
    "tcc_tiles_fill_bcsc": (_st, [_vp, C.POINTER(Bcsc), _vp]),
    "tcc_pull_scratch_bytes": (C.c_size_t, [_u32, _u32]),
    "tcc_pull_device_error": (_st, [_vp, C.POINTER(_i), _vp]),
    "tcc_set_grid_reserve": (None, [_u32]),
    "tcc_get_grid_reserve": (_u32, []),
    "tcc_set_wait_limit_ns": (None, [_u64]),
    "tcc_get_wait_limit_ns": (_u64, []),
    "tcc_gather_rows": (_st, [_vp, _u64, _u64, _vp, _u64, _vp, _u64, _u32, _vp, _vp]),
    "tcc_bcsr_spmm": (_st, [C.POINTER(Bcsr), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp, _i, _vp,
                            C.c_size_t, _i, _vp]),
    "tcc_bcsr_spmm_noalloc": (_st, [C.POINTER(Bcsr), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp,
                                    _i, _vp]),
    "tcc_noalloc_device_error": (_st, [C.POINTER(_i), _vp]),
    "tcc_scatter_add_rows": (_st, [_vp, _u64, _vp, _u64, _vp, _u64, _u64, _u32, _vp, _vp]),
    "tcc_peer_alloc": (_st, [C.c_size_t, C.POINTER(_vp), C.POINTER(IpcHandle)]),
    "tcc_peer_open": (_st, [C.POINTER(IpcHandle), C.POINTER(_vp)]),
    "tcc_peer_close": (_st, [_vp]),
    "tcc_peer_free": (_st, [_vp]),
    "tcc_halo_push": (_st, [C.POINTER(HaloPushArgs), _vp]),
    "tcc_halo_wait": (_st, [_vp, _u32, _u32, _u32, _u64, _vp]),
    "tcc_halo_release": (_st, [C.POINTER(_vp), _u32, _u32, _u32, _u32, _u32, _vp]),
    "tcc_peer_device_error": (_st, [_vp, C.POINTER(_i), _vp]),
    "tcc_dist_step": (_st, [C.POINTER(DistStepArgs), _vp, _vp]),
    "tcc_relu_dropout_forward": (_st, [_vp, _vp, _u64, C.c_float, _u64, _vp]),
    "tcc_relu_dropout_backward": (_st, [_vp, _vp, _vp, _u64, C.c_float, _vp]),
    "tcc_bcsr_spmm_t": (_st, [C.POINTER(Bcsr), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp, _vp]),
    "tcc_bcsc_spmm": (_st, [C.POINTER(Bcsc), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp, _vp]),
    "tcc_bcsc_spmm_t": (_st, [C.POINTER(Bcsc), _vp, _u64, _vp, _u64, _u32, _u32, _vp, _vp, _i,
                              _vp, C.c_size_t, _i, _vp]),
    "tcc_cnic_forward": (_st, [C.POINTER(Bcsr), C.POINTER(Bcsc), _vp, _vp, _u32, _u32, _vp,
                               C.c_size_t, _vp]),
    "tcc_cnic_forward_mixed": (_st, [C.POINTER(Bcsr), C.POINTER(Bcsc), _vp, _vp, _vp, _vp,
                                     C.c_int64, _vp, _u32, _u32, _vp, C.c_size_t, _vp]),
}

_LIB = None


def lib():
    """The loaded library; raises if it is absent (no CPU fallback exists)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise TccError(-1, f"{LIB_PATH} is missing; build it with `python -m tcc_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status: int, what: str = ""):
    if status != TCC_OK:
        msg = lib().tcc_last_error().decode(errors="replace")
        raise TccError(status, f"{what}: {msg}" if what else msg)


def call(name: str, *args):
    check(getattr(lib(), name)(*args), name)
