"""Row-partitioned SpMM across the GPUs of one box (one process per GPU).

The graph A (N x N) is split into contiguous row blocks P_g = [bounds[g],
bounds[g+1]) with about equal nonzeros.  Rank g holds A's rows P_g and the
feature rows X[P_g].  Its rows reference local columns (inside P_g) and a halo
of remote columns; the halo is compacted to the distinct remote columns, and
each owner learns once, at set-up, which of its rows every peer needs.

One SpMM step on rank g:
  1. on a high-priority side stream, send the rows peers need: with the peer
     transport (the default when every pair of GPUs has peer access), one
     kernel gathers them and stores them straight into the receivers' halo
     buffers over NVLink (tcc_b200.peer); with the NCCL transport, the
     tcc_gather_rows kernel packs them and an NCCL all-to-all (uneven splits)
     moves them;
  2. meanwhile run the local-column tiles on the caller's stream:
     Y = A_loc · X[P_g];
  3. wait for the halo, then Y += A_halo · X_halo (and, with the peer
     transport, hand the halo buffer back to the senders).
A_loc and A_halo are BCSR tilings of the local rows with column ids remapped to
[0, |P_g|) and [0, |halo|).  The process group should give NCCL high-priority
streams (ProcessGroupNCCL.Options.is_high_priority_stream) so the exchange's
kernels are scheduled ahead of the local tiles' queued blocks.  The same class
runs on CPU tensors over gloo without tilings, as the test harness of the
index plumbing (packing with index_select there).

This replaces the reference's multi-GPU feature access -- direct loads from a
peer GPU's feature cache inside the kernel
(TAC_training_backend/spmm_cnic/src/core/spmm_kernel.cu:145-147) -- with an
explicit exchange into local HBM.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def gather_rows(X: torch.Tensor, idx: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
    """out[i] = X[idx[i]] on the GPU (tcc_gather_rows); idx int64."""
    import ctypes as C
    from . import _lib as L
    assert X.is_cuda and X.dtype == torch.float32 and out.dtype == torch.float32
    assert idx.dtype == torch.int64 and out.shape[0] == idx.numel() and out.shape[1] == X.shape[1]
    s = (stream or torch.cuda.current_stream(X.device)).cuda_stream
    L.call("tcc_gather_rows", C.c_void_p(X.data_ptr()), X.stride(0), X.shape[0],
           C.c_void_p(idx.data_ptr()), idx.numel(), C.c_void_p(out.data_ptr()), out.stride(0),
           X.shape[1], None, C.c_void_p(s))
    return out


def _event(stream):
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    return e


def nccl_options():
    """ProcessGroupNCCL options with high-priority NCCL streams (the halo
    exchange then overlaps the local tiles instead of queueing behind them)."""
    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    return opts


def balanced_bounds(degrees: torch.Tensor, parts: int) -> list:
    """Contiguous row bounds with about equal nonzeros per part."""
    cum = torch.cumsum(degrees.to(torch.int64), 0)
    total = int(cum[-1])
    cuts = [int(torch.searchsorted(cum, total * k // parts).item()) for k in range(1, parts)]
    return [0] + cuts + [int(degrees.numel())]


# Rates behind push_sms, measured on B200 at F = 128 (both scale with F, so
# their ratio holds at other widths): one 512-thread push CTA stores ~12 GB/s
# of gathered rows over NVLink (210 MB in 0.47 ms on 32 CTAs), and one SM runs
# ~12.3 K tiles per ms of the pull kernel (3.76 M tiles in 2.06 ms on 148).
PUSH_BYTES_PER_CTA_MS = 12e6
PULL_TILES_PER_SM_MS = 12.3e3
# Past ~64 CTAs a push gets no faster (4 GPUs, config 2: the largest sender's
# push took 0.47 ms per operand on 64 CTAs and on 82), so more SMs would only
# slow the rank's local passes.
PUSH_SMS_CAP = 64


def push_sms(send_rows: int, local_tiles: int, sms: int) -> int:
    """SMs the peer push gets (and the local passes leave free) so that the
    rank's pushes of a pipelined pair end about when its local passes do:
    the push and local work split the SMs in proportion to their SM-time (at
    F = 128; both scale with F).  A rank that sends little beside much local
    work (2 GPUs: ~30 of 148) keeps most SMs for its tiles; one whose local
    work shrank with N but whose halo did not (R-MAT at 4-8 GPUs) hands more
    of them to the push, up to PUSH_SMS_CAP."""
    push = send_rows * 128 * 4 / PUSH_BYTES_PER_CTA_MS
    local = local_tiles / PULL_TILES_PER_SM_MS
    k = round(sms * push / max(push + local, 1e-9))
    return int(max(16, min(sms - 16, PUSH_SMS_CAP, k)))


def _csr_from_pairs(rows: torch.Tensor, cols: torch.Tensor, n_rows: int):
    order = torch.argsort(rows * (1 << 32) + cols)
    rows, cols = rows[order], cols[order]
    counts = torch.bincount(rows, minlength=n_rows)
    rowptr = torch.zeros(n_rows + 1, dtype=torch.int64, device=rows.device)
    rowptr[1:] = torch.cumsum(counts, 0)
    return rowptr, cols.to(torch.int32)


class DistGraph:
    """This rank's row block of a row-partitioned square graph.

    rowptr / col: the CSR of rows [bounds[rank], bounds[rank+1]) with GLOBAL
    column ids.  rs_local: row scale of the local rows; cs_global: column scale
    of every node (replicated, N floats) -- both optional (GCN normalisation).
    """

    def __init__(self, rowptr: torch.Tensor, col: torch.Tensor, bounds: list, group=None,
                 rs_local=None, cs_global=None, tc_threshold: int = 12, build_tiles: bool = True,
                 symmetric: bool = False, transport: str = "auto", peer_buffers: int = 2):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.bounds = list(bounds)
        r0, r1 = self.bounds[self.rank], self.bounds[self.rank + 1]
        self.r0, self.r1 = r0, r1
        self.n_local = r1 - r0
        dev = rowptr.device
        self.device = dev
        self.nnz = col.numel()
        if self.world == 1:
            # every column is local: the CSR is the local-column CSR as is
            self.halo = torch.empty(0, dtype=torch.int64, device=dev)
            self.recv_counts = [0]
            self.send_counts = [0]
            self.send_idx = torch.empty(0, dtype=torch.int64, device=dev)
            self.loc_rowptr, self.loc_col = rowptr, col.to(torch.int32)
            self.halo_rowptr = torch.zeros(self.n_local + 1, dtype=torch.int64, device=dev)
            self.halo_col = torch.empty(0, dtype=torch.int32, device=dev)
        else:
            col64 = col.to(torch.int64)
            rows = torch.repeat_interleave(torch.arange(self.n_local, device=dev),
                                           torch.diff(rowptr))
            is_loc = (col64 >= r0) & (col64 < r1)
            # compacted halo: distinct remote columns, ascending (so grouped by owner)
            self.halo = torch.unique(col64[~is_loc])
            bnd = torch.tensor(self.bounds, dtype=torch.int64, device=dev)
            owner = torch.searchsorted(bnd, self.halo, right=True) - 1
            self.recv_counts = torch.bincount(owner, minlength=self.world).tolist()
            # tell every owner which of its rows we need (local ids at the owner)
            req_local = (self.halo - bnd[owner]).to(torch.int64)
            self.send_counts = self._exchange_counts(self.recv_counts)
            self.send_idx = torch.empty(sum(self.send_counts), dtype=torch.int64, device=dev)
            dist.all_to_all_single(self.send_idx, req_local, self.send_counts, self.recv_counts,
                                   group=group)
            # local-column and halo-column CSRs of the local rows, remapped ids
            self.loc_rowptr, self.loc_col = _csr_from_pairs(rows[is_loc], col64[is_loc] - r0,
                                                            self.n_local)
            hcol = torch.searchsorted(self.halo, col64[~is_loc])
            self.halo_rowptr, self.halo_col = _csr_from_pairs(rows[~is_loc], hcol, self.n_local)
            del rows, col64, is_loc, hcol
        self.rs = rs_local
        self.cs_local = None if cs_global is None else cs_global[r0:r1].contiguous()
        self.cs_halo = None if cs_global is None or not self.halo.numel() else \
            cs_global[self.halo].contiguous()
        self.tc_threshold = tc_threshold
        self._bufs = {}
        self._side = None
        self._tstream = None
        self.comm_sms = 32  # SMs left to the exchange during the local tiles (measured best of 0-32)
        # which passes of spmm_pair (local X, local G, halo X, halo G) leave
        # comm_sms SMs free for the exchange still in flight (set below by
        # transport: the peer pushes end during the local passes, NCCL's
        # all-to-all runs into the first halo pass)
        self.pair_reserve = (True, True, True, False)
        # who sequences a step with the peer transport: "native" -- one call
        # of tcc_dist_step, the library enqueues the pushes, passes, waits and
        # releases; "python" -- the same sequence from here, call by call
        self.host_step = "native"
        self.symmetric = symmetric
        self.tiles_loc = self.tiles_halo = None
        self.tiles_loc_t = self.tiles_halo_t = None  # BCSC tilings, built by the first spmm_t
        # halo transport of the forward exchange: "peer" (rows stored into the
        # receivers' HBM over NVLink by one kernel, tcc_b200.peer) or "nccl"
        # (packed rows, one all-to-all); "auto" takes peer when every pair of
        # the ranks' GPUs has peer access
        self.peer = None
        if transport not in ("auto", "peer", "nccl"):
            raise ValueError("transport must be auto, peer or nccl")
        if self.world > 1 and rowptr.is_cuda and transport != "nccl":
            from .peer import PeerExchange, peers_reachable
            if peers_reachable(group):
                self.peer = PeerExchange(group, self.send_idx, self.send_counts, self.recv_counts,
                                         buffers=peer_buffers)
                self.peer.max_blocks = self.comm_sms
            elif transport == "peer":
                raise RuntimeError("transport='peer' needs peer access between every pair of GPUs")
        self.transport = "peer" if self.peer is not None else ("nccl" if self.world > 1 else "none")
        if self.transport == "peer":
            self.pair_reserve = (True, True, False, False)
        if build_tiles:
            from . import tiles
            self.tiles_loc = tiles.from_csr(self.loc_rowptr, self.loc_col, self.n_local,
                                            self.n_local, kind="bcsr")
            if self.halo.numel():
                self.tiles_halo = tiles.from_csr(self.halo_rowptr, self.halo_col, self.n_local,
                                                 int(self.halo.numel()), kind="bcsr")
            if self.peer is not None:
                sms = torch.cuda.get_device_properties(dev).multi_processor_count
                self.comm_sms = push_sms(int(self.send_idx.numel()), self.tiles_loc.num_TCBlocks, sms)
                self.peer.max_blocks = self.comm_sms

    def _exchange_counts(self, recv_counts):
        if self.world == 1:
            return [0]
        t = torch.tensor(recv_counts, dtype=torch.int64, device=self.device)
        out = torch.empty_like(t)
        dist.all_to_all_single(out, t, group=self.group)
        return out.tolist()

    @property
    def halo_rows(self) -> int:
        return int(self.halo.numel())

    def _buf(self, name, rows, like):
        key = (name, like.shape[1], like.dtype, like.device)
        b = self._bufs.get(key)
        if b is None or b.shape[0] != rows:
            b = torch.empty((rows, like.shape[1]), dtype=like.dtype, device=like.device)
            self._bufs[key] = b
        return b

    def exchange(self, X_local: torch.Tensor, async_op: bool = True, tag: int = 0,
                 timer: dict | None = None):
        """Start the halo exchange; returns (halo buffer, work handle or None).
        The halo buffer (one per ``tag`` and width) is reused by the next
        exchange with the same tag.  ``timer``: a dict that receives CUDA
        events "pack{tag}" (rows packed) and "xchg{tag}" (halo arrived)."""
        if self.peer is not None:
            return self._peer_exchange(X_local, async_op, tag, timer)
        recv = self._buf(f"recv{tag}", self.halo_rows, X_local)
        if self.world == 1:
            return recv, None
        send = self._buf(f"send{tag}", self.send_idx.numel(), X_local)
        if not X_local.is_cuda:
            torch.index_select(X_local, 0, self.send_idx, out=send)
            work = dist.all_to_all_single(recv, send, self.recv_counts, self.send_counts,
                                          group=self.group, async_op=async_op)
            return recv, work
        if self._side is None:
            self._side = torch.cuda.Stream(device=X_local.device, priority=-1)
        side = self._side
        side.wait_stream(torch.cuda.current_stream(X_local.device))
        with torch.cuda.stream(side):
            gather_rows(X_local, self.send_idx, send, stream=side)
            if timer is not None:
                timer[f"pack{tag}"] = _event(side)
            work = dist.all_to_all_single(recv, send, self.recv_counts, self.send_counts,
                                          group=self.group, async_op=True)
        if timer is not None:  # the arrival, seen from a stream nothing else waits on
            if self._tstream is None:
                self._tstream = torch.cuda.Stream(device=X_local.device)
            with torch.cuda.stream(self._tstream):
                work.wait()
                timer[f"xchg{tag}"] = _event(self._tstream)
        if not async_op:
            work.wait()
            work = None
        return recv, work

    def _peer_exchange(self, X_local, async_op, tag, timer):
        from .peer import PeerWork
        main = torch.cuda.current_stream(X_local.device)
        if self._side is None:
            self._side = torch.cuda.Stream(device=X_local.device, priority=-1)
        side = self._side
        side.wait_stream(main)
        seq = self.peer.push(X_local, tag, side)
        recv = self.peer.recv_buffer(tag, X_local.shape[1], seq)
        if timer is not None:
            timer[f"pack{tag}"] = _event(side)  # this rank's rows stored at the receivers
        work = PeerWork(self.peer, tag, seq, X_local.device)
        if timer is not None:  # the arrival, seen from a stream nothing else waits on
            if self._tstream is None:
                self._tstream = torch.cuda.Stream(device=X_local.device)
            # the timing wait is a kernel: start it no earlier than this step,
            # or it would sit on an SM through the previous step's passes (a
            # pull CTA needs a whole SM's registers)
            self._tstream.wait_stream(main)
            self.peer.wait(tag, seq, self._tstream)
            timer[f"xchg{tag}"] = _event(self._tstream)
        if not async_op:
            work.wait(main)
        return recv, work

    def device_error(self) -> int:
        """The peer transport's device error word (0 when none, or with NCCL)."""
        return self.peer.device_error() if self.peer is not None else 0

    def close(self):
        """Collective: release the peer transport's mapped buffers."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _local(self, X_local, out, reserve):
        from . import tiles
        from . import _lib as L
        # leave SMs for the exchange's NCCL kernels while these tiles run
        prev = L.lib().tcc_get_grid_reserve()
        L.lib().tcc_set_grid_reserve(self.comm_sms if reserve else 0)
        try:
            with torch.cuda.nvtx.range("tcc.local_tiles"):
                return tiles.bcsr_spmm(self.tiles_loc, X_local, out, tc_threshold=self.tc_threshold,
                                       rs=self.rs, cs=self.cs_local)
        finally:
            L.lib().tcc_set_grid_reserve(prev)

    def _halo(self, halo, work, Y, reserve=False):
        from . import tiles
        from . import _lib as L
        if work is not None and not getattr(work, "waited", False):
            work.wait()
        if self.tiles_halo is not None:
            prev = L.lib().tcc_get_grid_reserve()
            L.lib().tcc_set_grid_reserve(self.comm_sms if reserve else 0)
            try:
                with torch.cuda.nvtx.range("tcc.halo_tiles"):
                    tiles.bcsr_spmm(self.tiles_halo, halo, Y, tc_threshold=self.tc_threshold,
                                    rs=self.rs, cs=self.cs_halo, accumulate=True)
            finally:
                L.lib().tcc_set_grid_reserve(prev)
        if hasattr(work, "release"):  # peer transport: the senders may reuse the buffer
            work.release()

    def spmm(self, X_local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Y[P_g] = (diag(rs) A diag(cs) X)[P_g], exchange overlapped with the
        local-column tiles."""
        X_local = X_local.contiguous()
        if self._native():
            if out is None:
                out = torch.empty((self.n_local, X_local.shape[1]), dtype=X_local.dtype,
                                  device=X_local.device)
            self._native_step([(X_local, out, 0)], (True, False, False, False))
            return out
        with torch.cuda.nvtx.range("tcc.halo_exchange_start"):
            halo, work = self.exchange(X_local)
        Y = self._local(X_local, out, reserve=work is not None)
        self._halo(halo, work, Y)
        self._join_side(X_local.device)
        return Y

    def _native(self) -> bool:
        return self.host_step == "native" and self.peer is not None and self.tiles_loc is not None

    def _native_step(self, ops, reserve, timer=None):
        """One step enqueued by the library (tcc_dist_step): ops = [(X_local,
        Y, tag)] for one or two operands; reserve = which of the passes (local
        0, local 1, halo 0, halo 1) leave comm_sms SMs to the pushes."""
        import ctypes as C
        from . import _lib as L
        dev = ops[0][0].device
        main = torch.cuda.current_stream(dev)
        if self._side is None:
            self._side = torch.cuda.Stream(device=dev, priority=-1)
        a = L.DistStepArgs()
        keep = []  # ctypes structs the call reads
        sl = self.tiles_loc.struct()
        keep.append(sl)
        a.local = C.addressof(sl)
        sc = self.tiles_loc.scratch()
        a.local_scratch, a.local_scratch_bytes = sc.data_ptr(), sc.numel()
        a.local_plan_ready = int(self.tiles_loc._plan_ready)
        if self.tiles_halo is not None:
            sh = self.tiles_halo.struct()
            keep.append(sh)
            a.halo = C.addressof(sh)
            hc = self.tiles_halo.scratch()
            a.halo_scratch, a.halo_scratch_bytes = hc.data_ptr(), hc.numel()
            a.halo_plan_ready = int(self.tiles_halo._plan_ready)
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        a.rs, a.cs_local, a.cs_halo = ptr(self.rs), ptr(self.cs_local), ptr(self.cs_halo)
        a.tc_threshold = self.tc_threshold
        a.recv_mask = self.peer.recv_mask
        a.reserve_sms = self.comm_sms
        a.reserve_passes = sum(1 << i for i, x in enumerate(reserve) if x)
        for p in range(self.world):
            a.peer_flags[p] = self.peer.peer_flags[p] or 0
        a.n_ops = len(ops)
        if timer is not None:
            timer["start"] = _event(main)
        seqs = []
        for i, (X, Y, tag) in enumerate(ops):
            pa = self.peer.push_args(X, tag)
            seqs.append((tag, pa.seq))
            op = a.ops[i]
            op.push = pa
            halo = self.peer.recv_buffer(tag, X.shape[1], pa.seq)
            op.halo, op.ld_halo = (halo.data_ptr() if halo.numel() else None), X.shape[1]
            op.y, op.ldy = Y.data_ptr(), Y.stride(0)
        if timer is not None:
            names = [f"pack{i}" for i in range(len(ops))] + [f"local{i}" for i in range(len(ops))] + \
                    [f"done{i}" for i in range(len(ops))]
            slots = list(range(len(ops))) + [2 + i for i in range(len(ops))] + \
                [4 + i for i in range(len(ops))]
            for name, k in zip(names, slots):
                e = torch.cuda.Event(enable_timing=True)
                e.record(main)  # creates the event; the library records it again in place
                timer[name] = e
                a.events[k] = e.cuda_event
            if self._tstream is None:
                self._tstream = torch.cuda.Stream(device=dev)
            self._tstream.wait_stream(main)
            for i, (tag, seq) in enumerate(seqs):  # arrival, seen from a stream nothing waits on
                self.peer.wait(tag, seq, self._tstream)
                timer[f"xchg{i}"] = _event(self._tstream)
        with torch.cuda.nvtx.range("tcc.dist_step"):
            L.call("tcc_dist_step", C.byref(a), C.c_void_p(main.cuda_stream),
                   C.c_void_p(self._side.cuda_stream))
        self.tiles_loc._plan_ready = True
        if self.tiles_halo is not None:
            self.tiles_halo._plan_ready = True
        del keep

    def _join_side(self, device):
        """The caller's stream waits for the side stream's push (which reads
        the caller's rows), so the caller may overwrite or free them after
        the call; the push has long finished by then, so this costs nothing."""
        if self._side is not None:
            torch.cuda.current_stream(device).wait_stream(self._side)

    def spmm_pair(self, X_local: torch.Tensor, Y: torch.Tensor, G_local: torch.Tensor,
                  Z: torch.Tensor, timer: dict | None = None):
        """Two SpMMs over the partition, Y = Â[P_g, :]·X and Z = Â[P_g, :]·G,
        with both halo exchanges queued back to back at the start and both
        local passes run before either halo pass, so the halos travel while
        the local tiles (which need nothing remote) run.  ``timer``: a dict
        that receives CUDA events -- "start", "pack0/1", "xchg0/1" (halos
        arrived), "local0/1" (local tiles of Y / Z done) and "done0/1" (Y, Z
        complete)."""
        if self._native():
            self._native_step([(X_local, Y, 0), (G_local, Z, 1)], self.pair_reserve, timer)
            return Y, Z
        main = torch.cuda.current_stream(X_local.device)
        if timer is not None:
            timer["start"] = _event(main)
        with torch.cuda.nvtx.range("tcc.halo_exchange_start"):
            hx, wx = self.exchange(X_local, tag=0, timer=timer)
            hg, wg = self.exchange(G_local, tag=1, timer=timer)
        comm = wx is not None
        r = [comm and x for x in self.pair_reserve]
        self._local(X_local, Y, reserve=r[0])
        if timer is not None:
            timer["local0"] = _event(main)
        self._local(G_local, Z, reserve=r[1])  # the halos are still on the wire
        if timer is not None:
            timer["local1"] = _event(main)
        self._halo(hx, wx, Y, reserve=r[2])
        if timer is not None:
            timer["done0"] = _event(main)
        self._halo(hg, wg, Z, reserve=r[3])
        if timer is not None:
            timer["done1"] = _event(main)
        self._join_side(X_local.device)
        return Y, Z

    def spmm_t(self, G_local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Z[P_g] = (diag(cs) Aᵀ diag(rs) G)[P_g] with G and Z split like the rows.

        symmetric=True: Aᵀ = A, so this is the forward pass on the same
        partition.  Otherwise the exchange runs backwards: the rank's rows give
        partial sums for the local columns (kept) and for its halo columns,
        whose rows go back to their owners -- the all-to-all of the forward
        pass with the send and receive counts swapped -- and each owner adds
        the rows it receives into its own (tcc_scatter_add_rows; the rows it
        receives are the ones it sent in the forward exchange).  The local
        columns' pull overlaps the returning exchange."""
        if self.symmetric:
            return self.spmm(G_local, out)
        import ctypes as C
        from . import tiles
        from . import _lib as L
        G_local = G_local.contiguous()
        if self.tiles_loc_t is None:
            self.tiles_loc_t = tiles.from_csr(self.loc_rowptr, self.loc_col, self.n_local,
                                              self.n_local, kind="bcsc")
            if self.halo.numel():
                self.tiles_halo_t = tiles.from_csr(self.halo_rowptr, self.halo_col, self.n_local,
                                                   int(self.halo.numel()), kind="bcsc")
        main = torch.cuda.current_stream(G_local.device)
        work = None
        if self.tiles_halo_t is not None:
            # partial rows for the halo columns, scaled by their column scale
            Zh = self._buf("halo_part", self.halo_rows, G_local)
            tiles.bcsc_spmm_t(self.tiles_halo_t, G_local, Zh, tc_threshold=self.tc_threshold,
                              rs=self.rs, cs=self.cs_halo)
            back = self._buf("returned", int(self.send_idx.numel()), G_local)
            if self._side is None:
                self._side = torch.cuda.Stream(device=G_local.device, priority=-1)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                work = dist.all_to_all_single(back, Zh, self.send_counts, self.recv_counts,
                                              group=self.group, async_op=True)
        Z = tiles.bcsc_spmm_t(self.tiles_loc_t, G_local, out, tc_threshold=self.tc_threshold,
                              rs=self.rs, cs=self.cs_local)
        if work is not None:
            work.wait()
            if self.send_idx.numel():
                L.call("tcc_scatter_add_rows", C.c_void_p(back.data_ptr()), back.stride(0),
                       C.c_void_p(self.send_idx.data_ptr()), self.send_idx.numel(),
                       C.c_void_p(Z.data_ptr()), Z.stride(0), Z.shape[0], Z.shape[1], None,
                       C.c_void_p(main.cuda_stream))
        return Z


def exchange_window_cost(parts: int) -> float:
    """Per-window cost for tile_balanced_bounds when the halo is exchanged
    every pass.  On 2 GPUs a rank's local tiles outweigh the rows it sends,
    and balancing tiles is best (config 2: 2.90 ms per step at 2 against 3.00
    at 6).  From 4 GPUs on, the rank that sends the most rows (the power-law
    tail, whose rows many windows reference) paces every rank's halo passes,
    so each window also carries its rows' share of the sending (config 2 at
    4 GPUs: 2.05 / 1.98 / 1.90 ms per step at 2 / 6 / 10)."""
    return 2.0 if parts <= 2 else 10.0


def tile_balanced_bounds(window_offset: torch.Tensor, num_rows: int, parts: int,
                         window_cost: float = 2.0) -> list:
    """Contiguous row bounds, on window boundaries (multiples of 8), with about
    equal pull-kernel work per part: an 8-row window costs its tile count
    (``window_offset``, the BCSR rowWindowOffset of the whole graph) plus
    ``window_cost`` tiles' worth of per-window work.  Power-law graphs put
    their hub rows, whose windows hold many tiles per nonzero less than the
    tail's, at one end, so balancing nonzeros leaves the tail ranks slower."""
    off = window_offset.to(torch.int64)
    cost = torch.diff(off).to(torch.float64) + window_cost
    cum = torch.cumsum(cost, 0)
    total = float(cum[-1])
    W = cost.numel()
    cuts = []
    for k in range(1, parts):
        w = int(torch.searchsorted(cum, torch.tensor(total * k / parts, dtype=torch.float64,
                                                     device=cum.device)).item())
        cuts.append(min(num_rows, 8 * min(w + 1, W)))
    b = [0] + cuts + [num_rows]
    for k in range(1, len(b)):  # keep every part non-empty where rows allow
        b[k] = max(b[k], min(num_rows, b[k - 1] + 8))
    return b
