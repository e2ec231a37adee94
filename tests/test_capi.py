"""The C-ABI library: loads, exports every symbol include/tcc_b200.h declares,
and rejects bad arguments before touching a GPU (CPU only)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "tcc_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tcc_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from tcc_b200 import build, _lib
    build.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    from tcc_b200 import _lib
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.PROTOTYPES, f"{n} has no ctypes prototype"


def test_version_and_scratch_query(lib):
    assert b"sm_100a" in lib.tcc_version()
    assert lib.tcc_pull_scratch_bytes(1000, 5000) > 0
    assert lib.tcc_pull_scratch_bytes(2000, 5000) > lib.tcc_pull_scratch_bytes(1000, 5000)


def test_null_arguments_are_rejected_without_a_gpu(lib):
    from tcc_b200 import _lib
    assert lib.tcc_swtcf_alloc(None, 4, 4, 4, 16) == 1
    assert b"null" in lib.tcc_last_error()
    m = _lib.Swtcf()
    assert lib.tcc_swtcf_alloc(C.byref(m), 4, 0, 4, 16) == 1          # cols == 0
    assert lib.tcc_swtcf_alloc(C.byref(m), 4, 4, 4, 33) == 1          # S > 32
    assert lib.tcc_swtcf_spmm(None, None, None, 12, None) == 1
    assert lib.tcc_swtcf_prepare_pull(None, None) == 1
    assert lib.tcc_swtcf_prepare_pull(C.byref(_lib.Swtcf()), None) == 1  # never allocated
    assert b"unallocated" in lib.tcc_last_error()
    # the ctypes mirror of tcc_swtcf ends with the forward-pull fields
    assert _lib.Swtcf._fields_[-1][0] == "fwd_plan_ready"
    assert lib.tcc_bcsr_spmm(None, None, 0, None, 0, 128, 12, None, None, 0, None, 0, 0, None) == 1
    ws = C.c_void_p()
    assert lib.tcc_swtcf_workspace_create(C.byref(ws), 0, 10, 16) == 1
    assert lib.tcc_tiles_workspace_create(C.byref(ws), 10, 0, 10) == 1
    with pytest.raises(_lib.TccError):
        _lib.call("tcc_swtcf_spmm", None, None, None, 12, None)
    # the partitioned step: no arguments, no operands, a missing tiling
    assert lib.tcc_dist_step(None, None, None) == 1
    a = _lib.DistStepArgs()
    assert lib.tcc_dist_step(C.byref(a), None, None) == 1               # n_ops == 0
    assert b"n_ops" in lib.tcc_last_error()
    a.n_ops = 1
    assert lib.tcc_dist_step(C.byref(a), None, None) == 1               # no local tiles
    # the halo exchange: no arguments, a bad tag, step number 0
    assert lib.tcc_halo_push(None, None) == 1
    h = _lib.HaloPushArgs()
    h.world, h.rank, h.tag, h.seq, h.width = 2, 0, 9, 1, 4
    assert lib.tcc_halo_push(C.byref(h), None) == 1
    h.tag, h.seq = 0, 0
    assert lib.tcc_halo_push(C.byref(h), None) == 1
    assert lib.tcc_halo_wait(None, 0, 1, 1, 1000, None) == 1
    assert lib.tcc_peer_alloc(0, C.byref(C.c_void_p()), C.byref(_lib.IpcHandle())) == 1


def test_reference_build_exports_harness():
    path = os.path.join(ROOT, "oracle", "_ref", "libtcc_ref.so")
    if not os.path.exists(path):
        pytest.skip("reference build absent (built by `make -C oracle ref`)")
    L = C.CDLL(path)
    for n in ("ref_swtcf_convert", "ref_swtcf_spmm", "ref_cnic_spmm"):
        assert hasattr(L, n)


def test_wait_limit_setting_round_trips_without_a_gpu(lib):
    from tcc_b200 import _lib
    assert lib.tcc_get_wait_limit_ns() == _lib.DEFAULT_WAIT_LIMIT_NS
    try:
        lib.tcc_set_wait_limit_ns(12345)
        assert lib.tcc_get_wait_limit_ns() == 12345
    finally:
        lib.tcc_set_wait_limit_ns(0)
    assert lib.tcc_get_wait_limit_ns() == _lib.DEFAULT_WAIT_LIMIT_NS
    assert lib.tcc_noalloc_device_error(None, None) == 1  # NULL code: refused before any CUDA call
