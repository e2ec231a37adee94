"""Bounded waits of the bulk-copy pull kernel run out without faulting the GPU.

The kernel's mbarrier waits give up after the limit of tcc_set_wait_limit_ns,
record TCC_DEVERR_WAIT_TIMEOUT in the pull scratch's error word, wait (with
their own 2 s bound) for the copies they already issued, and return.  A limit
of 1 ns (below the timer's resolution) makes every wait a single test of its
barrier, so the first wait of a warp whose copies have not landed -- X is
512 MiB here, larger than L2, so the rows come from DRAM -- gives up; every
copy still reads valid memory, so nothing faults.  The next launch with the
default limit must give the right answer on the same context.
"""
import numpy as np
import pytest
import torch

from gpu_util import rel_fro
from tcc_b200 import _lib as L
from tcc_b200 import graphs as G
from tcc_b200 import tiles

pytestmark = pytest.mark.gpu


def test_wait_limit_expiry_is_reported_and_the_context_stays_usable(gpu, oracle, monkeypatch):
    monkeypatch.delenv("TCC_PULL_KERNEL", raising=False)  # F = 128: the bulk-copy kernel
    lib = L.lib()
    rp, col, _ = G.rmat_gpu(20, 16 << 20, seed=31, device="cuda")
    g = G.Csr(rp.numel() - 1, rp.numel() - 1, rp.cpu().numpy().astype(np.uint64),
              col.cpu().numpy().view(np.uint32))
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    gen = torch.Generator(device="cuda").manual_seed(32)
    X = torch.randn((g.cols, 128), generator=gen, device="cuda")
    assert lib.tcc_get_wait_limit_ns() == L.DEFAULT_WAIT_LIMIT_NS
    tiles.bcsr_spmm(t, X, tc_threshold=65)  # builds the plan; default limit
    assert tiles.pull_device_error(t) == 0
    try:
        lib.tcc_set_wait_limit_ns(1)
        assert lib.tcc_get_wait_limit_ns() == 1
        Y = tiles.bcsr_spmm(t, X, tc_threshold=65)
        code = tiles.pull_device_error(t)  # synchronises: the kernel returned
    finally:
        lib.tcc_set_wait_limit_ns(0)  # 0 restores the default
    assert lib.tcc_get_wait_limit_ns() == L.DEFAULT_WAIT_LIMIT_NS
    assert code == L.DEVERR_WAIT_TIMEOUT
    assert tiles.pull_device_error(t) == 0  # reading cleared the word
    # same context, default limit: complete and correct
    Y = tiles.bcsr_spmm(t, X, tc_threshold=65)
    assert tiles.pull_device_error(t) == 0
    want = oracle.csr_spmm(g, X.cpu().numpy())
    assert rel_fro(Y.cpu().numpy(), want) <= 1e-5
