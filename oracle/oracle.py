"""ctypes front end of the CPU oracle (oracle/liboracle.so) and of the
reference build (oracle/_ref/libtcc_ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py as the checker, never by the tcc_b200 package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

u32p = np.ctypeslib.ndpointer(np.uint32, flags="C")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C")


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        vp = C.c_void_p
        L.orc_swtcf_convert.restype = C.c_int
        L.orc_swtcf_convert.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, u32p, u32p,
                                        C.c_uint64, C.c_uint64, u32p, u64p, u32p, u32p, u32p, u8p,
                                        u32p, u8p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
        L.orc_swtcf_validate.restype = C.c_int
        L.orc_swtcf_validate.argtypes = [C.c_uint32, C.c_uint32, C.c_uint64, u32p, u32p, C.c_uint32,
                                         u32p, u64p, u32p, C.c_uint32, u32p, u32p, u8p, u32p, u8p,
                                         C.c_char_p, C.c_size_t]
        L.orc_swtcf_canonicalize.restype = C.c_int
        L.orc_swtcf_canonicalize.argtypes = [C.c_uint32, C.c_uint32, u32p, u64p, u32p, C.c_uint32,
                                             u32p, u32p, u8p, u32p, u8p]
        L.orc_swtcf_spmm.restype = None
        L.orc_swtcf_spmm.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, u32p, u64p, u32p, u32p,
                                     u32p, f32p, C.c_uint32, C.c_uint64, f32p, C.c_uint64,
                                     C.c_uint32]
        for nm in ("orc_bcsr_from_csr", "orc_bcsc_from_csr"):
            fn = getattr(L, nm)
            fn.restype = C.c_int
            fn.argtypes = [C.c_uint32, C.c_uint32, u64p, u32p, C.c_uint64, vp, vp, vp, vp,
                           C.POINTER(C.c_uint64)]
        for nm in ("orc_bcsr_spmm", "orc_bcsc_spmm"):
            fn = getattr(L, nm)
            fn.restype = None
            fn.argtypes = [C.c_uint32, C.c_uint32, u32p, u32p, u64p, f32p, C.c_uint32, C.c_uint64,
                           f32p, C.c_uint64, C.c_uint32, C.c_uint32]
        L.orc_csr_spmm.restype = None
        L.orc_csr_spmm.argtypes = [C.c_uint32, u64p, u32p, vp, vp, f32p, C.c_uint32, C.c_uint64,
                                   f32p, C.c_uint64, C.c_int]
        L.orc_csr_spmm_t.restype = None
        L.orc_csr_spmm_t.argtypes = [C.c_uint32, C.c_uint32, u64p, u32p, vp, vp, f32p, C.c_uint32,
                                     C.c_uint64, f32p, C.c_uint64, C.c_int]
        L.orc_csr_spmm_f32_omp.restype = None
        L.orc_csr_spmm_f32_omp.argtypes = [C.c_uint32, u64p, u32p, vp, vp, f32p, C.c_uint32,
                                           C.c_uint64, f32p, C.c_uint64, C.c_int]
        L.orc_kat_feature.restype = C.c_float
        L.orc_kat_feature.argtypes = [C.c_uint32, C.c_uint32]
        L.orc_tf32_rna.restype = C.c_float
        L.orc_tf32_rna.argtypes = [C.c_float]
        _LIB = L
    return _LIB


class OracleError(RuntimeError):
    def __init__(self, code, what=""):
        super().__init__(f"oracle status {code} {what}")
        self.code = code


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ------------------------------------------------------------------ SWTCF --

def swtcf_convert(rows, cols, dst, src, S=16):
    """Canonical SWTCF arrays (dict of numpy arrays, trimmed to T / R)."""
    L = lib()
    dst = np.ascontiguousarray(dst, dtype=np.uint32)
    src = np.ascontiguousarray(src, dtype=np.uint32)
    nnz = dst.size
    W = (cols + 7) // 8
    SW = (W + S - 1) // S
    cap = max(nnz, 1)
    out = dict(
        colWindowOffset=np.zeros(W + 1, np.uint32), tileLocalBit=np.zeros(cap, np.uint64),
        tileRowSlot=np.zeros(8 * cap, np.uint32), superWindowRowOffset=np.zeros(SW + 1, np.uint32),
        superWindowRows=np.zeros(cap, np.uint32), superWindowRowCacheSlot=np.zeros(cap, np.uint8),
        superWindowCachedRowSlot=np.zeros(32 * SW, np.uint32),
        superWindowCachedCount=np.zeros(SW, np.uint8))
    T = C.c_uint64()
    R = C.c_uint64()
    st = L.orc_swtcf_convert(rows, cols, S, nnz, dst, src, cap, cap, out["colWindowOffset"],
                             out["tileLocalBit"], out["tileRowSlot"], out["superWindowRowOffset"],
                             out["superWindowRows"], out["superWindowRowCacheSlot"],
                             out["superWindowCachedRowSlot"], out["superWindowCachedCount"],
                             C.byref(T), C.byref(R))
    if st != 0:
        raise OracleError(st, "swtcf_convert")
    T, R = T.value, R.value
    out["tileLocalBit"] = out["tileLocalBit"][:T].copy()
    out["tileRowSlot"] = out["tileRowSlot"][:8 * T].copy()
    out["superWindowRows"] = out["superWindowRows"][:R].copy()
    out["superWindowRowCacheSlot"] = out["superWindowRowCacheSlot"][:R].copy()
    out.update(rows=rows, cols=cols, S=S, numColWindows=W, numSuperWindows=SW, T=T, R=R)
    return out


def swtcf_validate(m, dst, src):
    """Run the restated reference validators; returns (ok, reason)."""
    L = lib()
    why = C.create_string_buffer(256)
    dst = np.ascontiguousarray(dst, dtype=np.uint32)
    src = np.ascontiguousarray(src, dtype=np.uint32)
    st = L.orc_swtcf_validate(m["cols"], m["S"], dst.size, dst, src, m["numColWindows"],
                              m["colWindowOffset"], m["tileLocalBit"], m["tileRowSlot"],
                              m["numSuperWindows"], m["superWindowRowOffset"], m["superWindowRows"],
                              m["superWindowRowCacheSlot"], m["superWindowCachedRowSlot"],
                              m["superWindowCachedCount"], why, 256)
    return st == 0, why.value.decode()


def swtcf_canonicalize(m):
    """Canonical form of a (reference) SWTCF dict, returned as a new dict."""
    L = lib()
    c = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in m.items()}
    st = L.orc_swtcf_canonicalize(c["S"], c["numColWindows"], c["colWindowOffset"],
                                  c["tileLocalBit"], c["tileRowSlot"], c["numSuperWindows"],
                                  c["superWindowRowOffset"], c["superWindowRows"],
                                  c["superWindowRowCacheSlot"], c["superWindowCachedRowSlot"],
                                  c["superWindowCachedCount"])
    if st != 0:
        raise OracleError(st, "canonicalize")
    return c


def swtcf_spmm(m, X, tc_threshold=12, Y=None):
    """Reference SWTCF arithmetic on the CPU (accumulates into Y)."""
    L = lib()
    X = np.ascontiguousarray(X, dtype=np.float32)
    F = X.shape[1]
    if Y is None:
        Y = np.zeros((m["rows"], F), np.float32)
    L.orc_swtcf_spmm(m["numColWindows"], m["S"], m["cols"], m["colWindowOffset"],
                     m["tileLocalBit"], m["tileRowSlot"], m["superWindowRowOffset"],
                     m["superWindowRows"], X, F, X.shape[1], Y, Y.shape[1], tc_threshold)
    return Y


# -------------------------------------------------------------- BCSR/BCSC --

def _tiles(fn, g, nwin):
    L = lib()
    T = C.c_uint64()
    st = getattr(L, fn)(g.rows, g.cols, g.rowptr, g.col, 0, None, None, None, None, C.byref(T))
    if st != 0:
        raise OracleError(st, fn)
    T = T.value
    off = np.zeros(nwin + 1, np.uint32)
    tco = np.zeros(T + 1, np.uint32)
    idx = np.zeros(max(8 * T, 1), np.uint32)
    bits = np.zeros(max(T, 1), np.uint64)
    st = getattr(L, fn)(g.rows, g.cols, g.rowptr, g.col, T, _ptr(off), _ptr(tco), _ptr(idx),
                        _ptr(bits), C.byref(C.c_uint64()))
    if st != 0:
        raise OracleError(st, fn)
    return off, tco, idx[:8 * T].copy(), bits[:T].copy(), T


def bcsr_from_csr(g):
    nwin = (g.rows + 7) // 8
    off, tco, idx, bits, T = _tiles("orc_bcsr_from_csr", g, nwin)
    return dict(num_rows=g.rows, num_cols=g.cols, nnz=g.nnz, num_TCBlocks=T, num_rowWindows=nwin,
                rowWindowOffset=off, tcOffset=tco, sparseA2B=idx, tcLocalBit=bits)


def bcsc_from_csr(g):
    nwin = (g.cols + 7) // 8
    off, tco, idx, bits, T = _tiles("orc_bcsc_from_csr", g, nwin)
    return dict(num_rows=g.rows, num_cols=g.cols, nnz=g.nnz, num_TCBlocks=T, num_colWindows=nwin,
                colWindowOffset=off, tcOffset=tco, sparseA2C=idx, tcLocalBit=bits)


def bcsr_spmm(b, X, tc_threshold=0, C_out=None):
    L = lib()
    X = np.ascontiguousarray(X, dtype=np.float32)
    F = X.shape[1]
    if C_out is None:
        C_out = np.zeros((b["num_rows"], F), np.float32)
    L.orc_bcsr_spmm(b["num_rowWindows"], b["num_cols"], b["rowWindowOffset"], b["sparseA2B"],
                    b["tcLocalBit"], X, F, F, C_out, F, b["num_rows"], tc_threshold)
    return C_out


def bcsc_spmm(b, X, tc_threshold=0, C_out=None):
    L = lib()
    X = np.ascontiguousarray(X, dtype=np.float32)
    F = X.shape[1]
    if C_out is None:
        C_out = np.zeros((b["num_rows"], F), np.float32)
    L.orc_bcsc_spmm(b["num_colWindows"], b["num_cols"], b["colWindowOffset"], b["sparseA2C"],
                    b["tcLocalBit"], X, F, F, C_out, F, b["num_rows"], tc_threshold)
    return C_out


# --------------------------------------------------------------- CSR SpMM --

def csr_spmm(g, X, rs=None, cs=None):
    L = lib()
    X = np.ascontiguousarray(X, dtype=np.float32)
    Y = np.zeros((g.rows, X.shape[1]), np.float32)
    L.orc_csr_spmm(g.rows, g.rowptr, g.col, _ptr(rs), _ptr(cs), X, X.shape[1], X.shape[1], Y,
                   Y.shape[1], 0)
    return Y


def csr_spmm_t(g, X, rs=None, cs=None):
    L = lib()
    X = np.ascontiguousarray(X, dtype=np.float32)
    Y = np.zeros((g.cols, X.shape[1]), np.float32)
    L.orc_csr_spmm_t(g.rows, g.cols, g.rowptr, g.col, _ptr(rs), _ptr(cs), X, X.shape[1],
                     X.shape[1], Y, Y.shape[1], 0)
    return Y


def csr_spmm_f32_omp(g, X, rs=None, cs=None, threads=0, rows=None, Y=None):
    """The CPU baseline kernel; `rows` limits it to the first rows (a sample)."""
    L = lib()
    n = g.rows if rows is None else rows
    if Y is None:
        Y = np.zeros((n, X.shape[1]), np.float32)
    L.orc_csr_spmm_f32_omp(n, g.rowptr, g.col, _ptr(rs), _ptr(cs), X, X.shape[1], X.shape[1], Y,
                           Y.shape[1], threads)
    return Y


def kat_features(n, F=128):
    """The reference's closed-form X (src/swtcf_spmm_main.cu:33-45)."""
    s = np.arange(n, dtype=np.uint32)[:, None]
    f = np.arange(F, dtype=np.uint32)[None, :]
    a = ((s * np.uint32(17) + np.uint32(13)) % np.uint32(97)).astype(np.float32) * np.float32(0.001)
    b = ((s * np.uint32(29) + np.uint32(7)) % np.uint32(89)).astype(np.float32) * np.float32(0.00001)
    return (a + b * f.astype(np.float32)).astype(np.float32)


def tf32(x):
    """Vectorised cvt.rna.tf32 restatement (same rule as orc_tf32_rna)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    finite = (u & np.uint32(0x7F800000)) != np.uint32(0x7F800000)
    r = np.where(finite, (u + np.uint32(0x1000)) & np.uint32(0xFFFFE000), u).astype(np.uint32)
    return r.view(np.float32)


def tf32_trunc(x):
    """fp32 -> TF32 by dropping the low 13 mantissa bits: how the tcgen05
    kind::tf32 tensor-core MMA reads an fp32 operand from shared memory."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


# -------------------------------------------------------------- reference --

def ref_lib():
    """oracle/_ref/libtcc_ref.so (reference sources built for sm_100a) or None."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libtcc_ref.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_cnic_last_error.restype = C.c_char_p
        L.ref_swtcf_convert.restype = C.c_int
        L.ref_swtcf_convert.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, u32p, u32p,
                                        u32p, u64p, u32p, u32p, u32p, u8p, u32p, u8p,
                                        C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                        C.POINTER(C.c_uint32)]
        L.ref_swtcf_convert_timed.restype = C.c_int
        L.ref_swtcf_convert_timed.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                              u32p, u32p, C.c_int, C.c_int,
                                              C.POINTER(C.c_float)]
        L.ref_swtcf_spmm_tiles.restype = C.c_int
        L.ref_swtcf_spmm_tiles.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                           C.c_uint32, u32p, u64p, u32p, u32p, u32p, u8p, u32p,
                                           u8p, f32p, f32p, C.c_uint32]
        L.ref_swtcf_spmm.restype = C.c_int
        L.ref_swtcf_spmm.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, u32p, u32p, f32p, f32p,
                                     C.c_uint32, C.c_int, C.c_int, C.POINTER(C.c_float)]
        L.ref_swtcf_spmm_quantized.restype = C.c_int
        L.ref_swtcf_spmm_quantized.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, u32p, u32p, i8p,
                                               f32p, C.c_uint32, u32p, f32p, C.c_uint32]
        L.ref_cnic_spmm.restype = C.c_int
        L.ref_cnic_spmm.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                    u32p, u32p, u32p, u64p, C.c_uint32, C.c_uint32, u32p, u32p,
                                    u32p, u64p, f32p, f32p, C.c_uint32, C.c_int, C.c_int,
                                    C.POINTER(C.c_float)]
        _REF = L
    return _REF


def ref_swtcf_convert(rows, cols, dst, src, S=16):
    L = ref_lib()
    dst = np.ascontiguousarray(dst, dtype=np.uint32)
    src = np.ascontiguousarray(src, dtype=np.uint32)
    nnz = dst.size
    W = (cols + 7) // 8
    SW = (W + S - 1) // S
    o = dict(colWindowOffset=np.zeros(W + 1, np.uint32), tileLocalBit=np.zeros(nnz, np.uint64),
             tileRowSlot=np.zeros(8 * nnz, np.uint32),
             superWindowRowOffset=np.zeros(SW + 1, np.uint32),
             superWindowRows=np.zeros(nnz, np.uint32),
             superWindowRowCacheSlot=np.zeros(nnz, np.uint8),
             superWindowCachedRowSlot=np.zeros(32 * SW, np.uint32),
             superWindowCachedCount=np.zeros(SW, np.uint8))
    T, R, err = C.c_uint32(), C.c_uint32(), C.c_uint32()
    rc = L.ref_swtcf_convert(rows, cols, S, nnz, dst, src, o["colWindowOffset"], o["tileLocalBit"],
                             o["tileRowSlot"], o["superWindowRowOffset"], o["superWindowRows"],
                             o["superWindowRowCacheSlot"], o["superWindowCachedRowSlot"],
                             o["superWindowCachedCount"], C.byref(T), C.byref(R), C.byref(err))
    if rc != 0:
        raise OracleError(rc, L.ref_last_error().decode())
    T, R = T.value, R.value
    o["tileLocalBit"] = o["tileLocalBit"][:T].copy()
    o["tileRowSlot"] = o["tileRowSlot"][:8 * T].copy()
    o["superWindowRows"] = o["superWindowRows"][:R].copy()
    o["superWindowRowCacheSlot"] = o["superWindowRowCacheSlot"][:R].copy()
    o.update(rows=rows, cols=cols, S=S, numColWindows=W, numSuperWindows=SW, T=T, R=R,
             device_error=err.value)
    return o


def ref_swtcf_convert_ms(rows, cols, dst, src, S=16, warmup=1, reps=5):
    """Mean ms per reference convertCOOToSWTCF call on the GPU (inputs resident)."""
    L = ref_lib()
    ms = C.c_float(0.0)
    rc = L.ref_swtcf_convert_timed(rows, cols, S, len(dst), np.ascontiguousarray(dst, np.uint32),
                                   np.ascontiguousarray(src, np.uint32), warmup, reps, C.byref(ms))
    if rc != 0:
        raise OracleError(rc, L.ref_last_error().decode())
    return ms.value


def ref_swtcf_spmm_tiles(m, X128, tc_threshold=12):
    """Reference launchSWTCFSpMM on the given SWTCF dict (e.g. the oracle's
    canonical tiling); returns Y (rows x 128)."""
    L = ref_lib()
    Y = np.zeros((m["rows"], 128), np.float32)
    rc = L.ref_swtcf_spmm_tiles(
        m["rows"], m["cols"], m["S"], m["T"], m["R"], m["colWindowOffset"],
        np.ascontiguousarray(m["tileLocalBit"]), np.ascontiguousarray(m["tileRowSlot"]),
        m["superWindowRowOffset"], np.ascontiguousarray(m["superWindowRows"]),
        np.ascontiguousarray(m["superWindowRowCacheSlot"]), m["superWindowCachedRowSlot"],
        m["superWindowCachedCount"], np.ascontiguousarray(X128, np.float32), Y, tc_threshold)
    if rc != 0:
        raise OracleError(rc, L.ref_last_error().decode())
    return Y


def ref_swtcf_spmm(rows, cols, dst, src, X128, tc_threshold=12, warmup=0, reps=0):
    """Reference convert + SpMM on the GPU; returns (Y, ms_per_launch or None)."""
    L = ref_lib()
    Y = np.zeros((rows, 128), np.float32)
    ms = C.c_float(0.0)
    rc = L.ref_swtcf_spmm(rows, cols, len(dst), np.ascontiguousarray(dst, np.uint32),
                          np.ascontiguousarray(src, np.uint32),
                          np.ascontiguousarray(X128, np.float32), Y, tc_threshold, warmup, reps,
                          C.byref(ms) if reps > 0 else None)
    if rc != 0:
        raise OracleError(rc, L.ref_last_error().decode())
    return Y, (ms.value if reps > 0 else None)


def ref_swtcf_spmm_quantized(rows, cols, dst, src, q_x, scales, src_global, tc_threshold=12):
    """Reference convert + launchSWTCFSpMMQuantized on the GPU; returns Y."""
    L = ref_lib()
    Y = np.zeros((rows, 128), np.float32)
    rc = L.ref_swtcf_spmm_quantized(rows, cols, len(dst), np.ascontiguousarray(dst, np.uint32),
                                    np.ascontiguousarray(src, np.uint32),
                                    np.ascontiguousarray(q_x, np.int8),
                                    np.ascontiguousarray(scales, np.float32), q_x.shape[0],
                                    np.ascontiguousarray(src_global, np.uint32), Y, tc_threshold)
    if rc != 0:
        raise OracleError(rc, L.ref_last_error().decode())
    return Y


def ref_cnic_spmm(num_rows, num_cols, B, bcsr=None, bcsc=None, warmup=0, reps=0):
    """Reference BCSR + BCSC kernels into one C; returns (C, ms_per_call or None)."""
    L = ref_lib()
    F = B.shape[1]
    Cm = np.zeros((num_rows, F), np.float32)
    z32 = np.zeros(1, np.uint32)
    z64 = np.zeros(1, np.uint64)
    ms = C.c_float(0.0)
    r = bcsr or {}
    c = bcsc or {}
    rc = L.ref_cnic_spmm(
        num_rows, num_cols, F,
        r.get("num_rowWindows", 0), r.get("num_TCBlocks", 0), r.get("rowWindowOffset", z32),
        r.get("tcOffset", z32), r.get("sparseA2B", z32), r.get("tcLocalBit", z64),
        c.get("num_colWindows", 0), c.get("num_TCBlocks", 0), c.get("colWindowOffset", z32),
        c.get("tcOffset", z32), c.get("sparseA2C", z32), c.get("tcLocalBit", z64),
        np.ascontiguousarray(B, np.float32), Cm, num_rows, warmup, reps,
        C.byref(ms) if reps > 0 else None)
    if rc != 0:
        raise OracleError(rc, L.ref_cnic_last_error().decode())
    return Cm, (ms.value if reps > 0 else None)
