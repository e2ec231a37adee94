"""tcc_bcsr_spmm_noalloc: the BCSR SpMM for callers that cannot allocate device
memory (code running inside an allocator's own callbacks, plug-ins of hosts that
own all device memory, real-time loops that forbid allocation after start-up).

Its work plan lives in a scratch array built into the library instead of caller
scratch.  This test calls it through the C ABI twice in a row, then on another
tiling, then on the first again, at widths that run each pull kernel, and
checks every result against tcc_bcsr_spmm (caller scratch) within the fp32
tolerance the SpMM tests use; it reads the built-in array's error word through
tcc_noalloc_device_error after each call, and checks that a tiling too large
for the built-in scratch is refused.  The file is collected last on purpose; it builds its own inputs, so it
passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import csr_dev, dense, rel_fro
from tcc_b200 import _lib as L
from tcc_b200 import graphs as G
from tcc_b200 import tiles

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5


def _noalloc(t, X, Y, thr, rs, cs, accumulate):
    s = t.struct()
    return L.lib().tcc_bcsr_spmm_noalloc(
        C.byref(s), C.c_void_p(X.data_ptr()), X.stride(0), C.c_void_p(Y.data_ptr()), Y.stride(0),
        X.shape[1], thr, C.c_void_p(rs.data_ptr()), C.c_void_p(cs.data_ptr()), accumulate,
        C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _noalloc_error():
    code = C.c_int(-1)
    st = L.lib().tcc_noalloc_device_error(C.byref(code),
                                          C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == L.TCC_OK, L.lib().tcc_last_error()
    return code.value


# F = 64 and 100 run the register-gather kernel, which reads its work plan
# (chunk descriptors, split windows) from the built-in array; F = 128 runs the
# bulk-copy kernel, which reads only the array's error word; F = 128 with
# TCC_PULL_KERNEL=ldg forces the register-gather kernel at that width too.
@pytest.mark.parametrize("F,kernel", [(64, ""), (100, ""), (128, ""), (128, "ldg")])
def test_noalloc_matches_scratch_entry_point(gpu, monkeypatch, F, kernel):
    if kernel:
        monkeypatch.setenv("TCC_PULL_KERNEL", kernel)
    else:
        monkeypatch.delenv("TCC_PULL_KERNEL", raising=False)
    # a power-law graph (heavy windows split across warps) plus a star hub
    g = G.rmat(14, 16 << 14, seed=21)
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    rs, cs = G.gcn_scales(g)
    X = dense(G.features(g.cols, F, seed=22))
    rs_d, cs_d = dense(rs), dense(cs)
    thr = 65  # fp32-accurate tiles
    ref = tiles.bcsr_spmm(t, X, tc_threshold=thr, rs=rs_d, cs=cs_d)
    for call in range(2):
        Y = torch.full((g.rows, F), float("nan"), device="cuda")
        assert _noalloc(t, X, Y, thr, rs_d, cs_d, 0) == L.TCC_OK, L.lib().tcc_last_error()
        assert _noalloc_error() == 0
        assert rel_fro(Y.cpu().numpy(), ref.cpu().numpy()) <= FP32_TOL, f"call {call}"
    # a different, smaller tiling next: the shared plan is rebuilt, not reused
    g2 = G.uniform(3000, 12, seed=23)
    rp2, col2 = csr_dev(g2)
    t2 = tiles.from_csr(rp2, col2, g2.rows, g2.cols, kind="bcsr")
    rs2, cs2 = G.gcn_scales(g2)
    X2 = dense(G.features(g2.cols, F, seed=24))
    ref2 = tiles.bcsr_spmm(t2, X2, tc_threshold=thr, rs=dense(rs2), cs=dense(cs2))
    Y2 = torch.empty((g2.rows, F), device="cuda")
    assert _noalloc(t2, X2, Y2, thr, dense(rs2), dense(cs2), 0) == L.TCC_OK
    assert _noalloc_error() == 0
    assert rel_fro(Y2.cpu().numpy(), ref2.cpu().numpy()) <= FP32_TOL
    # and back to the first, accumulating into a copy of its result
    Y3 = ref.clone()
    assert _noalloc(t, X, Y3, thr, rs_d, cs_d, 1) == L.TCC_OK
    assert _noalloc_error() == 0
    assert rel_fro(Y3.cpu().numpy(), 2 * ref.cpu().numpy()) <= FP32_TOL


def test_noalloc_refuses_oversized_tiling(gpu):
    lib = L.lib()
    rows = 8 << 20  # ~1M windows: its plan needs more than the built-in scratch
    need = lib.tcc_pull_scratch_bytes((rows + 7) // 8, 1 << 22)
    assert need > L.NOALLOC_SCRATCH_BYTES
    dummy = torch.zeros(16, dtype=torch.int64, device="cuda")
    s = L.Bcsr()
    s.num_rows, s.num_cols, s.nnz = rows, rows, 1 << 22
    s.num_TCBlocks, s.num_rowWindows = 1 << 22, (rows + 7) // 8
    s.rowWindowOffset = s.tcOffset = s.sparseA2B = s.tcLocalBit = dummy.data_ptr()
    X = torch.zeros((4, 128), device="cuda")
    st = lib.tcc_bcsr_spmm_noalloc(C.byref(s), C.c_void_p(X.data_ptr()), 128,
                                   C.c_void_p(X.data_ptr()), 128, 128, 65, None, None, 0, None)
    assert st == 6  # TCC_ERR_CAPACITY, refused before any launch
    assert b"built-in scratch" in lib.tcc_last_error()
