"""Bounded waits of the bulk-copy pull kernel run out without faulting the GPU.

The kernel's mbarrier waits give up after the limit of tcc_set_wait_limit_ns,
record TCC_DEVERR_WAIT_TIMEOUT in the pull scratch's error word, wait (with
their own 2 s bound) for the copies they already issued, and return.  A limit
of 1 ns makes the first wait of every warp whose copy has not landed yet run
out; every copy still reads valid memory, so nothing faults.  The next launch
with the default limit must give the right answer on the same context.
"""
import numpy as np
import pytest
import torch

from gpu_util import csr_dev, dense, rel_fro
from tcc_b200 import _lib as L
from tcc_b200 import graphs as G
from tcc_b200 import tiles

pytestmark = pytest.mark.gpu


def test_wait_limit_expiry_is_reported_and_the_context_stays_usable(gpu, oracle, monkeypatch):
    monkeypatch.delenv("TCC_PULL_KERNEL", raising=False)  # F = 128: the bulk-copy kernel
    lib = L.lib()
    g = G.rmat(15, 16 << 15, seed=31)
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    X = dense(G.features(g.cols, 128, seed=32))
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
    want = oracle.csr_spmm(g, G.features(g.cols, 128, seed=32))
    assert rel_fro(Y.cpu().numpy(), want) <= 1e-5
