"""Halo exchange of the row-partitioned SpMM through NVLink peer memory.

The NCCL transport of ``DistGraph`` packs the rows each peer needs into a send
buffer and hands both buffers to an all-to-all, whose kernels then copy them
across NVLink.  This transport does both in one kernel (``tcc_halo_push``):
each rank gathers its rows and stores them straight into the receivers' halo
buffers, which live in the receivers' HBM and are mapped into every peer with
CUDA IPC.  Completion is signalled through per-rank flag blocks (also mapped):
the sender marks step s of a tag arrived at each receiver, the receiver's
stream waits on those marks (``tcc_halo_wait``) before its halo tiles, and
releases the buffer back to the senders after them (``tcc_halo_release``) so
step s + 1 may overwrite it.  All waits are bounded; an expired wait leaves
TCC_DEVERR_WAIT_TIMEOUT in the rank's flag block (``device_error``).

One process per GPU of one box, every pair of GPUs with peer access.  Every
rank makes the same calls in the same order (the buffers are allocated
collectively on a tag's first use at a given width, and the step numbers are
counted per tag on each rank).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib as L

DEFAULT_WAIT_NS = 10_000_000_000  # a peer that is 10 s late is treated as gone


class _DeviceRows:
    """A raw device allocation seen by torch (CUDA array interface, no copy)."""

    def __init__(self, ptr: int, rows: int, width: int):
        self.__cuda_array_interface__ = {"shape": (rows, width), "typestr": "<f4",
                                         "data": (ptr, False), "version": 3, "strides": None}


def peers_reachable(group=None) -> bool:
    """Whether every rank's GPU can access every other rank's GPU directly."""
    world = dist.get_world_size(group)
    dev = torch.cuda.current_device()
    t = torch.tensor([dev], dtype=torch.int64, device=torch.device("cuda", dev))
    out = torch.empty(world, dtype=torch.int64, device=t.device)
    dist.all_gather_into_tensor(out, t, group=group)
    devs = out.tolist()
    ok = all(d == dev or torch.cuda.can_device_access_peer(dev, d) for d in devs)
    flag = torch.tensor([1 if ok and len(set(devs)) == world else 0], dtype=torch.int32,
                        device=t.device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())


class PeerExchange:
    """The peer-memory halo exchange for one partition.

    send_idx [sum(send_counts)] int64 (device): local rows to send, grouped by
    receiver; send_counts / recv_counts: rows to / from each rank (lists)."""

    def __init__(self, group, send_idx: torch.Tensor, send_counts: list, recv_counts: list,
                 wait_ns: int = DEFAULT_WAIT_NS, buffers: int = 2):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > L.PEER_MAX_RANKS:
            raise ValueError(f"at most {L.PEER_MAX_RANKS} ranks")
        self.device = send_idx.device
        self.send_idx = send_idx
        self.send_counts = list(send_counts)
        self.recv_counts = list(recv_counts)
        self.halo_rows = sum(self.recv_counts)
        self.wait_ns = int(wait_ns)
        # receive buffers per tag, step s in buffer (s - 1) % buffers: with two,
        # a sender may run one step ahead of a receiver that is still reading
        # the previous step's halo
        self.buffers = max(1, int(buffers))
        # push CTAs (512 threads): DistGraph sets this to the SMs its pull
        # kernels leave free, so the push never delays a pull CTA
        self.max_blocks = 32
        self.seg = [0]
        for c in self.send_counts:
            self.seg.append(self.seg[-1] + c)
        # where this rank's rows start in each receiver's halo buffer
        displ = [0]
        for c in self.recv_counts[:-1]:
            displ.append(displ[-1] + c)
        t = torch.tensor(displ, dtype=torch.int64, device=self.device)
        out = torch.empty_like(t)
        dist.all_to_all_single(out, t, group=group)
        self.dst_row = out.tolist()
        self.send_mask = sum(1 << p for p in range(self.world) if self.send_counts[p])
        self.recv_mask = sum(1 << p for p in range(self.world) if self.recv_counts[p])
        self._own = []     # allocations of this rank (freed by close)
        self._mapped = []  # peers' allocations mapped here (closed by close)
        self.flags, self.peer_flags = self._shared(L.PEER_FLAGS_BYTES)
        self._bufs = {}    # (tag, width) -> [(tensor view, [peer buffer base per rank])] per buffer
        self.seq = [0] * L.PEER_MAX_TAGS
        self.closed = False

    def _shared(self, nbytes: int):
        """Collective: allocate nbytes here, map every peer's allocation."""
        ptr = C.c_void_p()
        h = L.IpcHandle()
        L.call("tcc_peer_alloc", nbytes, C.byref(ptr), C.byref(h))
        self._own.append(ptr.value)
        mine = torch.tensor(list(bytes(h.bytes)), dtype=torch.uint8, device=self.device)
        alls = torch.empty(self.world * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(alls, mine, group=self.group)
        alls = alls.cpu().numpy().reshape(self.world, 64)
        peers = [None] * self.world
        for p in range(self.world):
            if p == self.rank:
                continue
            hp = L.IpcHandle()
            C.memmove(hp.bytes, alls[p].tobytes(), 64)
            q = C.c_void_p()
            L.call("tcc_peer_open", C.byref(hp), C.byref(q))
            self._mapped.append(q.value)
            peers[p] = q.value
        return ptr.value, peers

    def _buffers(self, tag: int, width: int):
        key = (tag, width)
        if key not in self._bufs:  # collective on first use
            rows = max(self.halo_rows, 1)
            bufs = []
            for _ in range(self.buffers):
                own, peers = self._shared(rows * width * 4)
                view = torch.as_tensor(_DeviceRows(own, rows, width), device=self.device)
                bufs.append((view[:self.halo_rows], peers))
            self._bufs[key] = bufs
        return self._bufs[key]

    def recv_buffer(self, tag: int, width: int, seq: int) -> torch.Tensor:
        """The halo rows of step ``seq`` of ``tag`` at ``width`` floats per row."""
        return self._buffers(tag, width)[(seq - 1) % self.buffers][0]

    def push(self, X: torch.Tensor, tag: int, stream: torch.cuda.Stream) -> int:
        """Send this rank's rows of X to their receivers (step number returned)."""
        a = self.push_args(X, tag)
        L.call("tcc_halo_push", C.byref(a), C.c_void_p(stream.cuda_stream))
        return a.seq

    def push_args(self, X: torch.Tensor, tag: int) -> "L.HaloPushArgs":
        """tcc_halo_push's arguments for the next step of ``tag`` (the step
        number advances; the caller launches the push, e.g. through
        tcc_dist_step)."""
        width = X.shape[1]
        bufs = self._buffers(tag, width)
        self.seq[tag] += 1
        _, peers = bufs[(self.seq[tag] - 1) % self.buffers]
        a = L.HaloPushArgs()
        a.x = X.data_ptr()
        a.ldx = X.stride(0)
        a.num_rows = X.shape[0]
        a.send_idx = self.send_idx.data_ptr() if self.send_idx.numel() else None
        a.width, a.world, a.rank, a.tag, a.seq = width, self.world, self.rank, tag, self.seq[tag]
        a.max_blocks = self.max_blocks
        a.buffers = self.buffers
        for p in range(self.world + 1):
            a.seg[p] = self.seg[p]
        for p in range(self.world):
            if peers[p] is not None:
                a.dst[p] = peers[p] + self.dst_row[p] * width * 4
                a.peer_flags[p] = self.peer_flags[p]
        a.ld_dst = width
        a.flags = self.flags
        a.wait_ns = self.wait_ns
        return a

    def wait(self, tag: int, seq: int, stream: torch.cuda.Stream):
        """``stream`` continues once every sender's rows of step ``seq`` arrived."""
        L.call("tcc_halo_wait", C.c_void_p(self.flags), tag, seq, self.recv_mask, self.wait_ns,
               C.c_void_p(stream.cuda_stream))

    def release(self, tag: int, seq: int, stream: torch.cuda.Stream):
        """After the kernels that read step ``seq``'s halo: senders may reuse it."""
        arr = (C.c_void_p * L.PEER_MAX_RANKS)(*[p or 0 for p in self.peer_flags] +
                                             [0] * (L.PEER_MAX_RANKS - self.world))
        L.call("tcc_halo_release", arr, self.world, self.rank, tag, seq, self.recv_mask,
               C.c_void_p(stream.cuda_stream))

    def device_error(self) -> int:
        """The flag block's error word (0, or a TCC_DEVERR_* code); synchronises."""
        code = C.c_int(0)
        s = torch.cuda.current_stream(self.device)
        L.call("tcc_peer_device_error", C.c_void_p(self.flags), C.byref(code),
               C.c_void_p(s.cuda_stream))
        return code.value

    def close(self):
        """Collective: unmap the peers' buffers, then free this rank's."""
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group, device_ids=[self.device.index])
        for q in self._mapped:
            L.call("tcc_peer_close", C.c_void_p(q))
        dist.barrier(group=self.group, device_ids=[self.device.index])
        for q in self._own:
            L.call("tcc_peer_free", C.c_void_p(q))
        self._mapped, self._own, self._bufs = [], [], {}
        self.closed = True


class PeerWork:
    """The handle ``DistGraph.exchange`` returns for the peer transport."""

    def __init__(self, ex: PeerExchange, tag: int, seq: int, device):
        self.ex, self.tag, self.seq, self.device = ex, tag, seq, device
        self.waited = False

    def wait(self, stream=None):
        stream = stream or torch.cuda.current_stream(self.device)
        self.ex.wait(self.tag, self.seq, stream)
        self.waited = True

    def release(self, stream=None):
        stream = stream or torch.cuda.current_stream(self.device)
        self.ex.release(self.tag, self.seq, stream)
