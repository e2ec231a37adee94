"""The peer-memory halo exchange kernels on one GPU (tcc_halo_push / wait /
release).  Two flag blocks and a receive buffer in this GPU's memory stand in
for a sender and a receiver; every launch runs in stream order on one stream,
so each wait is satisfied by an earlier launch -- except the last, which waits
for a release that nothing sends and must give up after its limit, record
TCC_DEVERR_WAIT_TIMEOUT and write no rows."""
import ctypes as C

import pytest
import torch

from tcc_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _alloc(nbytes):
    ptr, h = C.c_void_p(), L.IpcHandle()
    L.call("tcc_peer_alloc", nbytes, C.byref(ptr), C.byref(h))
    assert any(h.bytes)
    return ptr.value


def _error(flags):
    code = C.c_int(-1)
    L.call("tcc_peer_device_error", C.c_void_p(flags), C.byref(code), None)
    return code.value


def _push(X, idx, dst, ld_dst, flags_send, flags_recv, seq, wait_ns, tag=0, buffers=0):
    a = L.HaloPushArgs()
    a.x, a.ldx, a.num_rows = X.data_ptr(), X.stride(0), X.shape[0]
    a.send_idx = idx.data_ptr()
    a.width, a.world, a.rank, a.tag, a.seq = X.shape[1], 2, 0, tag, seq
    a.max_blocks = 0
    a.buffers = buffers
    a.seg[0], a.seg[1], a.seg[2] = 0, 0, idx.numel()  # every row goes to rank 1
    a.dst[1] = dst
    a.ld_dst = ld_dst
    a.peer_flags[1] = flags_recv
    a.flags = flags_send
    a.wait_ns = wait_ns
    L.call("tcc_halo_push", C.byref(a), None)


def _as_tensor(ptr, rows, width):
    class A:
        __cuda_array_interface__ = {"shape": (rows, width), "typestr": "<f4", "data": (ptr, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(A(), device="cuda")


@pytest.mark.parametrize("width", [128, 48, 260])
def test_push_wait_release_and_timeout(gpu, width):
    torch.cuda.synchronize()
    gen = torch.Generator(device="cuda").manual_seed(width)
    n_local, n_send = 5000, 3001
    X = torch.randn((n_local, width), generator=gen, device="cuda")
    idx = torch.randint(0, n_local, (n_send,), generator=gen, device="cuda", dtype=torch.int64)
    flags_s, flags_r = _alloc(L.PEER_FLAGS_BYTES), _alloc(L.PEER_FLAGS_BYTES)
    buf = _alloc(n_send * width * 4)
    recv = _as_tensor(buf, n_send, width)
    release_to = (C.c_void_p * L.PEER_MAX_RANKS)(flags_s)  # the receiver (rank 1) releases rank 0
    try:
        # step 1: push, wait for arrival, check, release
        _push(X, idx, buf, width, flags_s, flags_r, 1, 1_000_000_000)
        L.call("tcc_halo_wait", C.c_void_p(flags_r), 0, 1, 0b01, 1_000_000_000, None)
        torch.cuda.synchronize()
        assert _error(flags_s) == 0 and _error(flags_r) == 0
        assert torch.equal(recv, X[idx])
        L.call("tcc_halo_release", release_to, 2, 1, 0, 1, 0b01, None)
        # step 2 (released): new rows overwrite the buffer
        X2 = X * 2 + 1
        _push(X2, idx, buf, width, flags_s, flags_r, 2, 1_000_000_000)
        L.call("tcc_halo_wait", C.c_void_p(flags_r), 0, 2, 0b01, 1_000_000_000, None)
        torch.cuda.synchronize()
        assert _error(flags_s) == 0 and _error(flags_r) == 0
        assert torch.equal(recv, X2[idx])
        # step 3 without step 2's release: the push waits 2 ms, gives up, writes nothing
        _push(X * 0 - 7, idx, buf, width, flags_s, flags_r, 3, 2_000_000)
        torch.cuda.synchronize()
        assert _error(flags_s) == L.DEVERR_WAIT_TIMEOUT
        assert torch.equal(recv, X2[idx])
        # nor did it mark step 3 arrived: the receiver's wait runs out as well
        L.call("tcc_halo_wait", C.c_void_p(flags_r), 0, 3, 0b01, 2_000_000, None)
        torch.cuda.synchronize()
        assert _error(flags_r) == L.DEVERR_WAIT_TIMEOUT
        # the context is still usable
        assert torch.equal(X2[:4], X[:4] * 2 + 1)
    finally:
        del recv
        for p in (buf, flags_s, flags_r):
            L.call("tcc_peer_free", C.c_void_p(p))


def test_two_receive_buffers(gpu):
    """buffers = 2: step s goes to buffer (s-1) % 2, and a push waits only for
    the release of step s-2, so steps 1 and 2 go out before any release."""
    torch.cuda.synchronize()
    width, n_local, n_send = 128, 2000, 1500
    gen = torch.Generator(device="cuda").manual_seed(5)
    X = torch.randn((n_local, width), generator=gen, device="cuda")
    idx = torch.randint(0, n_local, (n_send,), generator=gen, device="cuda", dtype=torch.int64)
    flags_s, flags_r = _alloc(L.PEER_FLAGS_BYTES), _alloc(L.PEER_FLAGS_BYTES)
    bufs = [_alloc(n_send * width * 4) for _ in range(2)]
    views = [_as_tensor(b, n_send, width) for b in bufs]
    release_to = (C.c_void_p * L.PEER_MAX_RANKS)(flags_s)
    second = 1 << 30
    try:
        for s in (1, 2):  # no release in between
            _push(X * s, idx, bufs[(s - 1) % 2], width, flags_s, flags_r, s, second, buffers=2)
        L.call("tcc_halo_wait", C.c_void_p(flags_r), 0, 2, 0b01, second, None)
        torch.cuda.synchronize()
        assert _error(flags_s) == 0 and _error(flags_r) == 0
        assert torch.equal(views[0], X[idx]) and torch.equal(views[1], 2 * X[idx])
        # step 3 reuses buffer 0: it waits for step 1's release
        _push(X * 3, idx, bufs[0], width, flags_s, flags_r, 3, 2_000_000, buffers=2)
        torch.cuda.synchronize()
        assert _error(flags_s) == L.DEVERR_WAIT_TIMEOUT
        assert torch.equal(views[0], X[idx])
    finally:
        del views
        for p in bufs + [flags_s, flags_r]:
            L.call("tcc_peer_free", C.c_void_p(p))
    # a fresh pair of flag blocks: release step 1, then step 3 goes out
    flags_s, flags_r = _alloc(L.PEER_FLAGS_BYTES), _alloc(L.PEER_FLAGS_BYTES)
    buf = _alloc(n_send * width * 4)
    view = _as_tensor(buf, n_send, width)
    release_to = (C.c_void_p * L.PEER_MAX_RANKS)(flags_s)
    try:
        _push(X, idx, buf, width, flags_s, flags_r, 1, second, buffers=2)
        L.call("tcc_halo_release", release_to, 2, 1, 0, 1, 0b01, None)
        _push(X * 3, idx, buf, width, flags_s, flags_r, 3, second, buffers=2)
        L.call("tcc_halo_wait", C.c_void_p(flags_r), 0, 3, 0b01, second, None)
        torch.cuda.synchronize()
        assert _error(flags_s) == 0 and _error(flags_r) == 0
        assert torch.equal(view, 3 * X[idx])
    finally:
        del view
        for p in (buf, flags_s, flags_r):
            L.call("tcc_peer_free", C.c_void_p(p))


def test_push_rejects_bad_arguments(gpu):
    X = torch.zeros((8, 6), device="cuda")
    idx = torch.zeros(4, dtype=torch.int64, device="cuda")
    flags = _alloc(L.PEER_FLAGS_BYTES)
    try:
        with pytest.raises(L.TccError):  # width not a multiple of 4
            _push(X, idx, flags, 6, flags, flags, 1, 1000)
        a = L.HaloPushArgs()
        a.world, a.rank, a.seq, a.width, a.ldx, a.ld_dst, a.flags = 2, 0, 1, 4, 4, 4, flags
        a.seg[1] = 3  # rows to itself
        a.seg[2] = 3
        with pytest.raises(L.TccError):
            L.call("tcc_halo_push", C.byref(a), None)
        a.seg[1], a.seg[2], a.seq = 0, 3, 0  # step numbers start at 1
        with pytest.raises(L.TccError):
            L.call("tcc_halo_push", C.byref(a), None)
    finally:
        L.call("tcc_peer_free", C.c_void_p(flags))
