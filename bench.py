"""Benchmark of the tcc graph-aggregation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload spmm|gcn4|config5] [--dist-mode exchange|replicated]
                    [--no-extras]

Workload (config 2 of the benchmark set): seeded R-MAT graph, 2^20 nodes, 16M
directed edges (a,b,c,d = 0.57,0.19,0.19,0.05) symmetrised, deduplicated,
self-loops added; GCN normalisation D^-1/2 (A+I) D^-1/2 fused as diagonal
scales; X, G fp32 [N x 128] ~ N(0,1).  One step = the forward SpMM Y = A.X
(pull over BCSR row windows) plus the transposed SpMM Z = A^T.G (pull over BCSC
column windows: the backward pass).  Metric: SpMM GFLOP/s = 2 nnz F per SpMM,
whole job.  Before timing, sampled output rows of both passes are checked
against an fp64 recomputation (torch, on the device; no code of this library)
and the errors go into the line's "parity" field.

Multi-GPU (torchrun, one process per GPU; rank 0 prints the line with the max
time over ranks), strong scaling -- every N runs the same config-2 graph, split
into contiguous row blocks balanced by tiles:
  --dist-mode exchange (default): rank g holds only its rows of A, X and G; each
      SpMM exchanges the compacted feature halo (the distinct remote rows its
      rows reference) with an NCCL all-to-all, overlapped with the local tiles,
      the two SpMMs' exchanges queued back to back (tcc_b200.partition);
      Z = A[P_g, :].G on the same partition (A is symmetric);
  --dist-mode replicated: X and G resident on every GPU, no communication in
      the step (the transposed pass over a BCSC tiling of the rank's columns).
The e2e leg runs the same step through tcc_b200.hostio.HostPipeline: the
rank's rows of X and G from pinned host memory in, Y and Z out, every step.
--workload gcn4 reports config 4's GCN epoch time (tcc_b200.train_gcn);
--workload config5 the scale-26 forward SpMM (strong scaling).  At N = 1 the
line also carries config 3 (SBM, 602 -> 256 projection then the F = 256 SpMM),
config 4's 10-epoch GCN training, converter throughput and a torch.sparse CPU
baseline as extra fields (--no-extras leaves them out).

--impl reference: the reference's SpMMs are CUDA kernels with no CPU
implementation of their own; this arm times the CPU restatement of the path
(oracle/, fp32 CSR SpMM over all host threads) and torch.sparse.mm (the CPU
sparse product the reference's training script calls) on a bounded row sample
of the same workload, reports the faster as its value, and reports the
reference's own CUDA kernels (built from source for sm_100a into oracle/_ref)
on the same graph alongside: launchSWTCFSpMM, the spmm_cnic BCSR and BCSC
kernels, and the converter's GEdges/s.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

F = 128


def workload_name(world: int, mode: str) -> str:
    base = ("config2: R-MAT 2^20 nodes, 16 directed edges per node symmetrised+dedup+self-loops, "
            "GCN-normalised, F=128, forward A.X (BCSR pull) + transposed A^T.G")
    if world == 1:
        return base + " (BCSC pull)"
    if mode == "exchange":
        return base + (f"; {world} GPUs, rows split by tiles, feature halo exchanged over NCCL "
                       "every SpMM")
    return base + f"; {world} GPUs, rows split by tiles, X and G resident on every GPU"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--tc-threshold", type=int, default=12)
    p.add_argument("--scale", type=int, default=20, help="R-MAT scale (20 = config 2)")
    p.add_argument("--dist-mode", choices=["exchange", "replicated"], default="exchange",
                   help="N > 1: 'exchange' = rows, X and G split across GPUs, the feature "
                        "halo exchanged every SpMM; 'replicated' = X and G resident on every GPU")
    p.add_argument("--transport", choices=["auto", "peer", "nccl"], default="auto",
                   help="exchange mode's halo transport: 'peer' = one kernel stores the rows "
                        "into the receivers' HBM over NVLink (CUDA IPC); 'nccl' = packed rows, "
                        "one NCCL all-to-all; 'auto' = peer when every GPU pair has peer access")
    p.add_argument("--peer-buffers", type=int, default=2,
                   help="peer transport: receive buffers per tag a receiver rotates through "
                        "(2: a sender may run a step ahead)")
    p.add_argument("--window-cost", type=float, default=None,
                   help="N > 1: per-window cost (in tiles) added to each 8-row window's tile "
                        "count when the rows are cut into equal-work parts (default: 2 in "
                        "replicated mode; partition.exchange_window_cost(N) in exchange mode)")
    p.add_argument("--host-step", choices=["native", "python"], default="native",
                   help="peer transport: a step sequenced by one tcc_dist_step call (native) "
                        "or call by call from Python")
    p.add_argument("--push-sms", type=int, default=0,
                   help="peer transport: SMs for the halo push and held back from the local "
                        "passes (0: sized per rank from its send rows and local tiles)")
    p.add_argument("--pair-reserve", default=None,
                   help="exchange mode: four 0/1 digits, whether the local X, local G, halo X "
                        "and halo G passes leave SMs free for the exchange (default: 1100 with "
                        "the peer transport, 1110 with NCCL)")
    p.add_argument("--workload", choices=["spmm", "gcn4", "config5"], default="spmm",
                   help="spmm: the config-2 SpMM step (headline); gcn4: config-4 GCN epoch time "
                        "(tcc_b200.train_gcn, epochs = --steps); config5: the scale-26 forward "
                        "SpMM, strong scaling")
    p.add_argument("--no-extras", action="store_true",
                   help="N = 1: leave out the config-3, config-4, converter and torch.sparse fields")
    p.add_argument("--aggregate-first", action="store_true",
                   help="gcn4: compute layer 2 as (A.H).W, the reference's order, instead of "
                        "choosing by width (A.(H.W) for 256 -> 47)")
    p.add_argument("--scale5", type=int, default=26, help="config5: R-MAT scale (26 = config 5)")
    p.add_argument("--c5-mode", choices=["exchange", "replicated"], default="exchange",
                   help="config5 on N > 1 GPUs: exchange the X halo every step, or all-gather X "
                        "once at set-up (static input features) and run without communication")
    p.add_argument("--profile", choices=["fwd", "bwd", "swtcf"], default=None,
                   help="build the workload, run only the forward (or transposed) pull, or the "
                        "reference-named SWTCF forward (push), --steps times and exit: the "
                        "command ncu captures")
    return p.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            j = json.load(f)
        return j.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def pull_kernel_name(F):
    """The BCSR pull kernel the library dispatches for width F (the bulk-copy
    kernel for F a multiple of 128 unless TCC_PULL_KERNEL picks another)."""
    choice = os.environ.get("TCC_PULL_KERNEL", "")
    if choice == "tma" or (choice == "" and F % 128 == 0):
        return "pull_tma_kernel"
    if choice == "umma":
        return "pull_umma_kernel"
    return "pull_kernel"


def profiled_traffic(kernel_tag):
    """dram bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for name in sorted(os.listdir(d)):
        if not name.endswith((".md", ".txt")):
            continue
        with open(os.path.join(d, name)) as f:
            for line in f:
                m = re.match(rf"\s*traffic_bytes_per_launch\[{re.escape(kernel_tag)}\]\s*[:=]\s*([0-9.eE+]+)", line)
                if m:
                    return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, device_index):
        self.proc = None
        self.dir = tempfile.mkdtemp(prefix="tcc_clocks_")
        self.path = os.path.join(self.dir, f"clocks_rank{device_index}.csv")
        self.idx = device_index

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}",
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        shutil.rmtree(self.dir, ignore_errors=True)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def host_csr(rowptr, col, cols):
    """The device CSR as the oracle's host Csr (uint64 rowptr, uint32 col)."""
    from tcc_b200 import graphs as G
    return G.Csr(rowptr.numel() - 1, cols, rowptr.cpu().numpy().astype(np.uint64),
                 col.cpu().numpy().view(np.uint32))


def cpu_baseline(g, X, rs, cs, budget_s=12.0):
    """Oracle fp32 CSR SpMM (OpenMP, all host threads) on a contiguous row sample."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    # calibrate on a small prefix, then size the sample to ~budget_s
    rows = min(g.rows, 4096)
    t0 = time.time()
    O.csr_spmm_f32_omp(g, X, rs, cs, threads=threads, rows=rows)
    dt = max(time.time() - t0, 1e-4)
    nnz_small = int(g.rowptr[rows])
    rate = nnz_small / dt
    target = int(rate * budget_s / 3)
    rows = int(np.searchsorted(g.rowptr, min(target, g.nnz))) if target < g.nnz else g.rows
    rows = max(1, min(rows, g.rows))
    nnz = int(g.rowptr[rows])
    times = []
    for _ in range(3):
        t0 = time.time()
        O.csr_spmm_f32_omp(g, X, rs, cs, threads=threads, rows=rows)
        times.append(time.time() - t0)
    t = statistics.median(times)
    gflops = 2.0 * nnz * X.shape[1] / t / 1e9
    return {"value": round(gflops, 3), "unit": "GFLOP/s", "cores": threads, "kind": "port",
            "sample": f"first {rows} of {g.rows} rows ({nnz} of {g.nnz} nnz, F={X.shape[1]}), "
                      f"median of 3, fp32 OpenMP CSR SpMM"}


# ------------------------------------------------------------------ inputs --

def gen_config2(scale, device):
    """Config 2's graph on the device (the same graph on every rank and every
    N): CSR rowptr int64 [n+1], col int32 [nnz], GCN scale s = deg^-1/2."""
    import torch
    from tcc_b200 import graphs as G
    rowptr, col, _ = G.rmat_gpu(scale, 16 << scale, seed=1, device=device)
    deg = torch.diff(rowptr)
    s = torch.where(deg > 0, deg.to(torch.float64).clamp(min=1).rsqrt(),
                    torch.zeros_like(deg, dtype=torch.float64)).to(torch.float32)
    return rowptr, col, s


def features(n, seed, device):
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return torch.randn((n, F), generator=gen, device=device)


def row_block(rowptr, col, r0, r1):
    lrp = (rowptr[r0:r1 + 1] - rowptr[r0]).contiguous()
    return lrp, col[rowptr[r0]:rowptr[r1]].contiguous()


def column_block(rowptr, col, c0, c1):
    """CSR of A[:, c0:c1] (every row; columns shifted to [0, c1 - c0))."""
    import torch
    n = rowptr.numel() - 1
    keep = (col >= c0) & (col < c1)
    rows = torch.repeat_interleave(torch.arange(n, device=col.device), torch.diff(rowptr))
    counts = torch.bincount(rows[keep], minlength=n)
    rp = torch.zeros(n + 1, dtype=torch.int64, device=col.device)
    rp[1:] = torch.cumsum(counts, 0)
    return rp, (col[keep] - c0).to(torch.int32).contiguous()


# ------------------------------------------------------------------ parity --

def check_rows(rowptr, col, rows, rs, cs, Xin, Yout, chunk=1 << 21):
    """fp64 recomputation of sampled output rows of Y = diag(rs) A diag(cs) X
    (torch gathers and index_add on the device, none of this library's code):
    returns (relative Frobenius, relative inf-norm) over the sample.
    rowptr/col: CSR whose rows index Y's rows and whose columns index X's rows;
    rs: scale per Y row (indexed like rows), cs: scale per X row."""
    import torch
    rows = rows.to(torch.int64)
    starts, ends = rowptr[rows], rowptr[rows + 1]
    counts = ends - starts
    out = torch.repeat_interleave(torch.arange(rows.numel(), device=rows.device), counts)
    base = torch.repeat_interleave(starts - torch.cumsum(counts, 0) + counts, counts)
    pos = base + torch.arange(out.numel(), device=rows.device)
    inn = col[pos].to(torch.int64)
    ref = torch.zeros((rows.numel(), Xin.shape[1]), dtype=torch.float64, device=Xin.device)
    for a in range(0, inn.numel(), chunk):
        i = inn[a:a + chunk]
        v = Xin[i].to(torch.float64)
        if cs is not None:
            v *= cs[i].to(torch.float64)[:, None]
        ref.index_add_(0, out[a:a + chunk], v)
    if rs is not None:
        ref *= rs[rows].to(torch.float64)[:, None]
    got = Yout[rows].to(torch.float64)
    fro = (torch.linalg.norm(got - ref) / torch.linalg.norm(ref).clamp(min=1e-300)).item()
    inf = ((got - ref).abs().max() / ref.abs().max().clamp(min=1e-300)).item()
    return fro, inf


def sample_rows(n, seed, device, head=256, total=4096):
    """The first `head` rows (the hub rows of an R-MAT block) plus random others."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    rnd = torch.randint(0, max(n, 1), (max(total - head, 0),), generator=gen, device=device)
    return torch.unique(torch.cat([torch.arange(min(head, n), device=device), rnd]))


# ------------------------------------------------------------------ timing --

def time_steps(step, steps, warmup, world, local_rank, per_step_events=False):
    """W warm-up steps, then K steps between a barrier + synchronize on both
    sides, timed with CUDA events on the current stream; clocks sampled during
    the timed region.  step(i, ev) gets a dict to fill with per-step events."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        step(None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = [dict() for _ in range(steps)]
    stream = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h0 = time.perf_counter()
    for i in range(steps):
        step(evs[i])
    host_ms = (time.perf_counter() - h0) * 1e3
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    clocks["host_enqueue_ms"] = round(host_ms, 3)  # host time to enqueue the K steps
    return e0.elapsed_time(e1), evs, clocks


def ev_ms(evs, a, b):
    import statistics as st
    return st.mean(e[a].elapsed_time(e[b]) for e in evs)


def allreduce(vals, op, device, dtype=None):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=dtype or torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=op)
    return t.tolist()


# ------------------------------------------------------------- our arm ----

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from tcc_b200 import tiles as T
    from tcc_b200.hostio import HostPipeline
    from tcc_b200.partition import DistGraph, exchange_window_cost, tile_balanced_bounds
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    mode = "single" if world == 1 else args.dist_mode
    thr = args.tc_threshold
    t0 = time.time()
    rowptr, col, s = gen_config2(args.scale, device)
    n = rowptr.numel() - 1
    X = features(n, 1000, device)
    Gm = features(n, 1001, device)
    torch.cuda.synchronize()
    gen_s = time.time() - t0
    t0 = time.time()
    full_bcsr = T.from_csr(rowptr, col, n, n, kind="bcsr")
    if args.window_cost is None:
        args.window_cost = exchange_window_cost(world) if mode == "exchange" else 2.0
    bounds = [0, n] if world == 1 else tile_balanced_bounds(full_bcsr.windowOffset, n, world,
                                                            window_cost=args.window_cost)
    r0, r1 = bounds[rank], bounds[rank + 1]
    n_loc = r1 - r0
    lrp, lcol = row_block(rowptr, col, r0, r1)
    stream = torch.cuda.current_stream()
    Y = torch.empty((n_loc, F), device=device)
    Z = torch.empty((n_loc, F), device=device)
    X_loc, G_loc = X[r0:r1], Gm[r0:r1]
    halo_rows = 0
    push_sms_all = None
    if mode == "exchange":
        dg = DistGraph(lrp, lcol, bounds, rs_local=s[r0:r1].contiguous(), cs_global=s,
                       tc_threshold=thr, transport=args.transport, peer_buffers=args.peer_buffers)
        halo_rows = dg.halo_rows
        if args.pair_reserve:
            dg.pair_reserve = tuple(c == "1" for c in args.pair_reserve[:4])
        dg.host_step = args.host_step
        if args.push_sms and dg.peer is not None:
            dg.comm_sms = dg.peer.max_blocks = args.push_sms
        push_sms_all = [int(dg.comm_sms)]
        if world > 1:  # every rank's exchange SMs (sized from its own rows and tiles)
            t = torch.tensor([float(dg.comm_sms)], dtype=torch.float64, device=device)
            g = torch.empty(world, dtype=torch.float64, device=device)
            dist.all_gather_into_tensor(g, t)
            push_sms_all = [int(v) for v in g.tolist()]
        X_loc, G_loc = X_loc.contiguous(), G_loc.contiguous()

        def step(ev):
            dg.spmm_pair(X_loc, Y, G_loc, Z, timer=ev)

        fwd_pass = lambda Xd, Yd: dg.spmm(Xd, Yd)  # noqa: E731
        bwd_pass = fwd_pass  # A symmetric: the rank's rows of A^T are its rows of A
        # per SpMM -- peer: push, zero + pull (local), wait, pull (halo), release,
        # and the timer's arrival wait; nccl: pack, zero + pull (local), pull (halo)
        launches_per_step = 2 * (7 if dg.transport == "peer" else 4)
    else:
        tl = full_bcsr if world == 1 else T.from_csr(lrp, lcol, n_loc, n, kind="bcsr")
        crp, ccol = (rowptr, col) if world == 1 else column_block(rowptr, col, r0, r1)
        tl_t = T.from_csr(crp, ccol, n, n_loc, kind="bcsc")
        rs_loc = s[r0:r1].contiguous()

        def fwd_pass(Xd, Yd):
            T.bcsr_spmm(tl, Xd, Yd, tc_threshold=thr, rs=rs_loc, cs=s)

        def bwd_pass(Gd, Zd):  # Z[P_g] = diag(s) A[:, P_g]^T diag(s) G
            T.bcsc_spmm_t(tl_t, Gd, Zd, tc_threshold=thr, rs=s, cs=rs_loc)

        def step(ev):
            if ev is not None:
                ev["start"] = _event(stream)
            fwd_pass(X, Y)
            if ev is not None:
                ev["done0"] = _event(stream)
            bwd_pass(Gm, Z)
            if ev is not None:
                ev["done1"] = _event(stream)

        launches_per_step = 2 * 2  # per SpMM: zero + pull
    torch.cuda.synchronize()
    conv_s = time.time() - t0
    nnz_loc = int(lcol.numel())

    # correctness before timing: sampled rows of Y and Z against fp64 torch
    step(None)
    torch.cuda.synchronize()
    rows = sample_rows(n_loc, 77 + rank, device)
    e_fwd = check_rows(lrp, lcol, rows, s[r0:r1], s, X, Y)
    if mode == "exchange":  # Z = A[P_g, :] G
        e_bwd = check_rows(lrp, lcol, rows, s[r0:r1], s, Gm, Z)
    else:  # Z = (A^T)[P_g, :] G: rows of the transposed column block
        trp, tcol = csr_transpose(crp, ccol, n_loc)
        e_bwd = check_rows(trp, tcol, rows, s[r0:r1], s, Gm, Z)
        del trp, tcol
    errs = allreduce([e_fwd[0], e_fwd[1], e_bwd[0], e_bwd[1], float(rows.numel())],
                     dist.ReduceOp.MAX if world > 1 else None, device)

    ms, evs, clocks = time_steps(step, args.steps, args.warmup, world, local_rank)
    host_ms = allreduce([clocks.pop("host_enqueue_ms") / args.steps],
                        dist.ReduceOp.MAX if world > 1 else None, device)[0]
    fwd_ms = ev_ms(evs, "start", "done0")
    bwd_ms = ev_ms(evs, "done0", "done1")
    phases = None
    if mode == "exchange":
        phases = {k: ev_ms(evs, "start", k) for k in
                  ("pack0", "pack1", "xchg0", "xchg1", "local0", "done0", "local1", "done1")}
    mx = allreduce([ms, fwd_ms, bwd_ms] + ([phases[k] for k in sorted(phases)] if phases else []),
                   dist.ReduceOp.MAX if world > 1 else None, device)
    by_rank = None
    if phases and world > 1:  # every rank's phases (rows of an all-gather)
        keys = sorted(phases)
        mine = torch.tensor([phases[k] for k in keys], dtype=torch.float64, device=device)
        allp = torch.empty((world, len(keys)), dtype=torch.float64, device=device)
        dist.all_gather_into_tensor(allp, mine)
        by_rank = [{k: round(v, 4) for k, v in zip(keys, row)} for row in allp.tolist()]
    ms, fwd_ms_max, bwd_ms_max = mx[:3]
    if mode == "exchange":  # the two passes interleave (local, local, halo, halo): half a step each
        fwd_ms = bwd_ms = ms / args.steps / 2
        fwd_ms_max = bwd_ms_max = ms / args.steps / 2
    if phases:
        phases = {k: round(v, 4) for k, v in zip(sorted(phases), mx[3:])}
    tot = allreduce([float(nnz_loc), float(halo_rows)], dist.ReduceOp.SUM if world > 1 else None,
                    device)
    nnz_total, halo_total = tot

    # end to end through the public API: HostPipeline, the rank's rows of X and
    # G from pinned host memory and its rows of Y and Z back, every step
    hX = X[r0:r1].cpu().pin_memory()
    hG = Gm[r0:r1].cpu().pin_memory()
    hY = torch.empty((n_loc, F)).pin_memory()
    hZ = torch.empty((n_loc, F)).pin_memory()
    if mode == "replicated":  # each pass all-gathers the full X (G) from the rows
        parts_x = [X[bounds[g]:bounds[g + 1]] for g in range(world)]
        parts_g = [Gm[bounds[g]:bounds[g + 1]] for g in range(world)]

        def e2e_fwd(Xd, Yd):
            dist.all_gather(parts_x, Xd)
            fwd_pass(X, Yd)

        def e2e_bwd(Gd, Zd):
            dist.all_gather(parts_g, Gd)
            bwd_pass(Gm, Zd)
    else:
        e2e_fwd, e2e_bwd = fwd_pass, bwd_pass
    pipe = HostPipeline(e2e_fwd, e2e_bwd, (n_loc, F), (n_loc, F), (n_loc, F), (n_loc, F), device)
    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        pipe.submit(hX, hG, hY, hZ)
    pipe.synchronize()
    if world > 1:
        dist.barrier()
    h2d0, d2h0 = pipe.h2d_bytes, pipe.d2h_bytes
    a0 = pipe.start_event()
    for _ in range(e2e_steps):
        pipe.submit(hX, hG, hY, hZ)
    a1 = pipe.end_event()
    pipe.synchronize()
    e2e = allreduce([a0.elapsed_time(a1) / e2e_steps, (pipe.h2d_bytes - h2d0) / e2e_steps,
                     (pipe.d2h_bytes - d2h0) / e2e_steps],
                    dist.ReduceOp.MAX if world > 1 else None, device)
    e2e_ms, h2d_step, d2h_step = e2e
    # the same outputs as the device-resident run (split windows reduce in any order)
    e2e_ok = all(((a - b).abs().max() / b.abs().max().clamp(min=1e-30)).item() <= 1e-5
                 for a, b in ((hY, Y.cpu()), (hZ, Z.cpu())))
    transport = "none"
    if mode == "exchange":
        transport = dg.transport
        dev_err = dg.device_error()
        dg.close()  # collective: every rank, before rank 0 reports
        if dev_err:
            raise RuntimeError(f"halo exchange device error {dev_err}")

    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    ms_per_step = ms / args.steps
    flops_step = 2 * (2.0 * nnz_total * F)
    n_in = n if mode != "exchange" else n_loc + halo_rows  # X rows rank 0's forward reads
    b_alg = 4 * F * (n_in + n_loc) + 8 * nnz_loc + 4 * (n_loc + 1)
    achieved = b_alg / (fwd_ms * 1e-3) / 1e9
    kern = pull_kernel_name(F)
    line = {
        "metric": "SpMM GFLOP/s (2*nnz*F)",
        "value": round(flops_step / (ms_per_step * 1e-3) / 1e9, 2),
        "unit": "GFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded R-MAT, torch GPU generator seed 1)",
        "config": {"workload": workload_name(world, mode), "rmat_scale": args.scale, "nodes": n,
                   "nnz_total": int(nnz_total), "nnz_rank0": nnz_loc, "F": F,
                   "halo_rows_total": int(halo_total), "halo_rows_rank0": int(halo_rows),
                   "tc_threshold": thr, "l2": "inputs larger than L2 (X, G 512 MiB)",
                   "parallelism": ("1 GPU" if world == 1 else
                                   f"{world}-way 1D row partition balanced by tiles; " +
                                   (("compacted feature halo stored into the receivers' HBM "
                                     "over NVLink by one gather kernel (CUDA IPC peer memory)"
                                     if transport == "peer" else
                                     "compacted feature halo all-to-all over NCCL") +
                                    " each SpMM, overlapped with the local tiles"
                                    if mode == "exchange" else "X, G resident on every GPU")),
                   "transport": transport,
                   "pair_reserve": ("".join("1" if x else "0" for x in dg.pair_reserve)
                                    if mode == "exchange" else None),
                   "peer_buffers": args.peer_buffers if transport == "peer" else None,
                   "exchange_sms_by_rank": push_sms_all if mode == "exchange" else None,
                   "host_step": (args.host_step if mode == "exchange" and transport == "peer"
                                 else None),
                   "row_bounds": bounds if world > 1 else None,
                   "window_cost": args.window_cost if world > 1 else None,
                   "gen_s": round(gen_s, 3), "convert_s": round(conv_s, 3)},
        "parity": {"checker": "fp64 torch recomputation of sampled output rows (device gathers "
                              "+ index_add), before timing",
                   "rows_sampled_per_rank": int(errs[4]),
                   "forward": {"rel_fro": errs[0], "rel_inf": errs[1]},
                   "transposed": {"rel_fro": errs[2], "rel_inf": errs[3]},
                   "tolerance": {"rel_fro": 5e-3, "rel_inf": 1e-3},
                   "ok": bool(max(errs[0], errs[2]) <= 5e-3 and max(errs[1], errs[3]) <= 1e-3)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profiled_traffic(f"{kern}_config2") if world == 1 else None,
                     "kernel": f"{kern}, forward SpMM" + (
                         "" if world == 1 else " (rank 0: local + halo tiles, exchange overlapped)"
                         if mode == "exchange" else " (rank 0's rows)"),
                     "fwd_ms": round(fwd_ms, 4), "alg_bytes_per_launch": b_alg,
                     "x_rows_read": int(n_in), "peak_kind": peak_kind},
        "transposed": {"kernel": (f"{kern} over BCSC column windows" if mode != "exchange" else
                                  "forward kernels over the partition (A symmetric)"),
                       "ms": round(bwd_ms, 4), "ms_max_over_ranks": round(bwd_ms_max, 4),
                       "frac": round(b_alg / (bwd_ms * 1e-3) / 1e9 / peak, 4)},
        "e2e": {"value": round(flops_step / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s",
                "h2d_bytes_per_step": int(h2d_step), "d2h_bytes_per_step": int(d2h_step),
                "bytes_per_step_are": "max over ranks",
                "ms_per_step": round(e2e_ms, 3), "outputs_match_device_run": bool(e2e_ok),
                "api": "tcc_b200.hostio.HostPipeline (uploads, passes and downloads on three "
                       "streams; two device buffer sets alternate across steps)"},
        "gpu_launches": launches_per_step * args.steps,
        "host_enqueue_ms_per_step": round(host_ms, 4),  # max over ranks; below ms_per_step: GPU-bound
        "clocks": clocks,
    }
    if phases:
        line["phases_ms_from_step_start"] = phases
        if by_rank:
            line["phases_ms_by_rank"] = by_rank
        line["phases_note"] = ("max over ranks of the mean over steps; pack/xchg: rows packed / "
                               "halo arrived (0 = X, 1 = G), local/done: local tiles / all tiles "
                               "of that SpMM finished")
    if world == 1:
        line["swtcf_forward"] = swtcf_forward(rowptr, col, n, X, device)
        if not args.no_extras:
            line.update(extras(args, device, rowptr, col, s, X))
        g = host_csr(rowptr, col, n)
        sh = s.cpu().numpy()
        line["cpu_baseline"] = cpu_baseline(g, X.cpu().numpy(), sh, sh)
    print(json.dumps(line), flush=True)


def _event(stream):
    import torch
    e = torch.cuda.Event(enable_timing=True)
    e.record(stream)
    return e


def csr_transpose(rowptr, col, ncols):
    """CSR of A^T from the CSR of A (rows of A^T = columns of A)."""
    import torch
    n = rowptr.numel() - 1
    r = torch.repeat_interleave(torch.arange(n, device=col.device), torch.diff(rowptr))
    c = col.to(torch.int64)
    order = torch.argsort(c * n + r)
    counts = torch.bincount(c, minlength=ncols)
    rp = torch.zeros(ncols + 1, dtype=torch.int64, device=col.device)
    rp[1:] = torch.cumsum(counts, 0)
    return rp, r[order].to(torch.int32)


def swtcf_forward(rowptr, col, n, X, device, reps=5):
    """Informative: the reference-named SWTCF forward (tcc_swtcf_spmm;
    pattern-only, F = 128, tc_threshold 12, Y accumulates) on the same graph,
    the call the reference arm times for the reference kernel
    (reference_gpu_kernel): as converted (push over column windows), and after
    tcc_swtcf_prepare_pull (pull over row windows).  Conversion and preparation
    outside the timing; median of reps."""
    import torch
    from tcc_b200 import swtcf
    E = col.numel()
    m = swtcf.SWTCFMatrix(n, n, E, 16)
    ws = swtcf.SWTCFConvertWorkspace(E, n, 16)
    swtcf.convert_csr(rowptr, col, m, ws)
    ws.free()
    Y = torch.zeros((n, 128), device=device)
    swtcf.spmm(m, X, Y, tc_threshold=12)
    def timed():
        ts = []
        for _ in range(reps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            swtcf.spmm(m, X, Y, tc_threshold=12)
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)
    ms = timed()  # push over column windows (no preparation, allocates nothing)
    swtcf.prepare_pull(m)
    swtcf.spmm(m, X, Y, tc_threshold=12)
    ms_pull = timed()  # pull over the prepared row-window tiling
    m.free()
    return {"what": "tcc_swtcf_spmm (launchSWTCFSpMM's entry point), pattern-only, forward only",
            "ms": round(ms, 3), "value": round(2.0 * E * 128 / (ms * 1e-3) / 1e9, 2),
            "unit": "GFLOP/s", "after_prepare_pull_ms": round(ms_pull, 3),
            "after_prepare_pull_value": round(2.0 * E * 128 / (ms_pull * 1e-3) / 1e9, 2)}


# ----------------------------------------------------- N = 1 extra fields --

def extras(args, device, rowptr, col, s, X):
    import torch
    out = {}
    for name, fn in (("convert", lambda: convert_rates(rowptr, col, device)),
                     ("config3", lambda: config3(device)),
                     ("gcn4", lambda: gcn4(device)),
                     ("cpu_baseline_torch_sparse", lambda: torch_sparse_baseline(rowptr, col, s, X))):
        try:
            out[name] = fn()
        except Exception as e:  # an extra field never sinks the headline line
            out[name] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
        torch.cuda.empty_cache()
    return out


def convert_rates(rowptr, col, device, reps=5):
    """Converter throughput on config 2 (the reference's instrument: edges per
    second over repeated conversions, src/swtcf_convert_main.cu:376-417):
    tcc_swtcf_convert_csr into a preallocated matrix and workspace, and the
    CSR -> BCSR tiling."""
    import torch
    from tcc_b200 import swtcf
    from tcc_b200 import tiles as T
    n = rowptr.numel() - 1
    E = col.numel()
    m = swtcf.SWTCFMatrix(n, n, E, 16)
    ws = swtcf.SWTCFConvertWorkspace(E, n, 16)
    # the reference's input form: COO (dst = row, src = column), dst ascending
    dst = torch.repeat_interleave(torch.arange(n, device=device, dtype=torch.int32),
                                  torch.diff(rowptr))
    src = col

    def timed(fn):
        ts = []
        for i in range(reps + 1):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i:
                ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    ms_coo = timed(lambda: swtcf.convert_coo(dst, src, m, ws))
    ms = timed(lambda: swtcf.convert_csr(rowptr, col, m, ws))
    assert ws.device_error() == 0
    ws.free()
    m.free()
    del dst
    tw = T.TilesWorkspace(E, n, n)
    tt = []
    for i in range(reps + 1):
        t0 = time.perf_counter()
        T.from_csr(rowptr, col, n, n, kind="bcsr", ws=tw)
        torch.cuda.synchronize()
        if i:
            tt.append((time.perf_counter() - t0) * 1e3)
    tw.free()
    mt = statistics.median(tt)
    return {"edges": E, "swtcf_convert_coo_ms": round(ms_coo, 3),
            "swtcf_coo_gedges_per_s": round(E / (ms_coo * 1e-3) / 1e9, 3),
            "swtcf_convert_csr_ms": round(ms, 3),
            "swtcf_gedges_per_s": round(E / (ms * 1e-3) / 1e9, 3),
            "bcsr_tiles_ms": round(mt, 3), "bcsr_gedges_per_s": round(E / (mt * 1e-3) / 1e9, 3),
            "timing": "SWTCF: CUDA events around the call (COO: the reference's input form, "
                      "dst-ascending; CSR: rows in order, so only the window digits are sorted), "
                      "median of %d; BCSR: host wall clock of prepare (synchronises for the tile "
                      "count) + fill, median of %d" % (reps, reps)}


def config3(device, reps=10, warmup=3):
    """Config 3: SBM, 232,965 nodes in 50 communities, ~114.6 M edges, GCN
    scales; H = X W (602 -> 256, fp32 GEMM, timed on its own), then
    Y = D^-1/2 (A+I) D^-1/2 H at F = 256 (the default pull kernel)."""
    import torch
    from tcc_b200 import graphs as G
    from tcc_b200 import tiles as T
    n = 232_965
    t0 = time.time()
    rp, col = G.sbm_gpu(n, 50, 114_600_000, 40.0, 1.2, seed=2, device=device)
    deg = torch.diff(rp)
    s = deg.to(torch.float64).clamp(min=1).rsqrt().to(torch.float32)
    gen = torch.Generator(device=device)
    gen.manual_seed(2)
    X = torch.rand((n, 602), generator=gen, device=device) * 2 - 1
    W = torch.randn((602, 256), generator=gen, device=device) / 602 ** 0.5
    tl = T.from_csr(rp, col, n, n, kind="bcsr")
    torch.cuda.synchronize()
    build_s = time.time() - t0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        H = X @ W
        gemm = []
        for i in range(warmup + reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(X, W, out=H)
            e1.record()
            torch.cuda.synchronize()
            if i >= warmup:
                gemm.append(e0.elapsed_time(e1))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    Y = torch.empty((n, 256), device=device)
    spmm = []
    for i in range(warmup + reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        T.bcsr_spmm(tl, H, Y, tc_threshold=12, rs=s, cs=s)
        e1.record()
        torch.cuda.synchronize()
        if i >= warmup:
            spmm.append(e0.elapsed_time(e1))
    rows = sample_rows(n, 3, device)
    fro, inf = check_rows(rp, col, rows, s, s, H, Y)
    E = col.numel()
    ms = statistics.mean(spmm)
    peak, kind = measured_peaks()
    b_alg = 4 * 256 * (2 * n) + 8 * E + 4 * (n + 1)
    gms = statistics.mean(gemm)
    return {"workload": "config3: SBM 232,965 nodes, 50 blocks, intra/inter 40, log-normal(1.2) "
                        "propensities, ~114.6 M edges symmetrised+dedup+self-loops, GCN scales; "
                        "X U[-1,1] [N x 602] -> H = X W [N x 256] -> Y = A H",
            "nnz": E, "spmm_ms": round(ms, 4), "spmm_gflops": round(2.0 * E * 256 / (ms * 1e-3) / 1e9, 2),
            "roofline": {"bound": "hbm", "alg_bytes": b_alg,
                         "achieved": round(b_alg / (ms * 1e-3) / 1e9, 1), "peak": peak,
                         "frac": round(b_alg / (ms * 1e-3) / 1e9 / peak, 4), "peak_kind": kind,
                         "kernel": pull_kernel_name(256)},
            "projection_gemm_ms": round(gms, 4),
            "projection_gemm_tflops": round(2.0 * n * 602 * 256 / (gms * 1e-3) / 1e12, 2),
            "projection_gemm": "torch.matmul fp32 (TF32 off; cuBLAS), timed separately",
            "parity": {"rows_sampled": int(rows.numel()), "rel_fro": fro, "rel_inf": inf},
            "build_s": round(build_s, 2), "tiles": tl.num_TCBlocks}


def gcn4(device):
    """Config 4: 2-layer GCN on 2,449,029 nodes (R-MAT, ~123.8 M nonzeros with
    self-loops), 10 epochs, Adam 1e-2, hot/cold feature store (tcc_b200.train_gcn)."""
    from tcc_b200 import train_gcn
    cfg = train_gcn.config()
    cfg["epochs"] = 10
    r = train_gcn.train(cfg, device, 1, 0)
    steady = r["epoch_s"][1:] or r["epoch_s"]
    return {"epoch_s_mean_after_first": round(sum(steady) / len(steady), 5),
            "epoch_s": [round(x, 5) for x in r["epoch_s"]],
            "loss_first": round(r["losses"][0], 5), "loss_last": round(r["losses"][-1], 5),
            "nnz": int(r["nnz"]), "hot_rows": r["store_hot"], "cold_rows": r["store_cold"],
            "cold_staging": r["cold_staging"], "transform_first": r["transform_first"],
            "build_s": round(r["gen_s"] + r["conv_s"], 2)}


def torch_sparse_baseline(rowptr, col, s, X, budget_s=6.0):
    """torch.sparse.mm on the CPU (the sparse product of the reference's
    training script, train/tcgnn_conv_release.py:152), CSR fp32 with the GCN
    values, all host threads, on a contiguous row sample."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rp = rowptr.cpu()
    c = col.cpu().to(torch.int64)
    sh = s.cpu()
    Xh = X.cpu()
    n = rp.numel() - 1

    def run(rows):
        nz = int(rp[rows])
        vals = sh[torch.repeat_interleave(torch.arange(rows), torch.diff(rp[:rows + 1]))] * sh[c[:nz]]
        A = torch.sparse_csr_tensor(rp[:rows + 1], c[:nz], vals, size=(rows, n))
        t0 = time.perf_counter()
        torch.sparse.mm(A, Xh)
        return time.perf_counter() - t0, nz

    dt, nz = run(min(n, 8192))
    rate = nz / max(dt, 1e-6)
    target = min(int(rate * budget_s / 2), int(rp[-1]))
    rows = max(1, min(n, int(torch.searchsorted(rp, torch.tensor(target)).item())))
    times = []
    for _ in range(2):
        dt, nz = run(rows)
        times.append(dt)
    t = min(times)
    return {"value": round(2.0 * nz * F / t / 1e9, 3), "unit": "GFLOP/s", "cores": threads,
            "kind": "torch.sparse.mm", "sample": f"first {rows} of {n} rows ({nz} nnz, F={F}), "
                                                 "best of 2, fp32 CSR"}


def run_config5(args, rank, world, local_rank):
    """Config 5: one directed R-MAT graph (scale --scale5, 16 edges per node,
    seed 4, deduplicated, row-normalised), forward Y = A.X with F = 128 on 1..N
    GPUs -- strong scaling: every N partitions the same graph by rows."""
    import torch
    import torch.distributed as dist
    from tcc_b200 import graphs as G
    from tcc_b200.partition import DistGraph, balanced_bounds
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    scale = args.scale5
    edges = 16 << scale
    t0 = time.time()
    deg = G.rmat_gpu_degrees(scale, edges, seed=4, device=device, symmetric=False, loops=False)
    bounds = balanced_bounds(deg, world)
    del deg
    r0, r1 = bounds[rank], bounds[rank + 1]
    lrp, lcol, _ = G.rmat_gpu(scale, edges, seed=4, device=device, row_range=(r0, r1),
                              symmetric=False, loops=False)
    d = torch.diff(lrp)
    rs = torch.where(d > 0, 1.0 / d.clamp(min=1).to(torch.float64),
                     torch.zeros_like(d, dtype=torch.float64)).to(torch.float32)
    torch.cuda.synchronize()
    gen_s = time.time() - t0
    t0 = time.time()
    F = 128
    n = 1 << scale
    replicated = args.c5_mode == "replicated" and world > 1
    allgather_s = None
    gen = torch.Generator(device=device)
    gen.manual_seed(4000 + rank)
    X = torch.randn((r1 - r0, F), generator=gen, device=device)
    Y = torch.empty_like(X)
    if replicated:
        # X is static input: all-gather the row blocks once, then every step
        # runs the rank's rows against the full local copy (no exchange)
        from tcc_b200 import tiles as T
        tl = T.from_csr(lrp, lcol, r1 - r0, n, kind="bcsr")
        del lcol
        torch.cuda.empty_cache()
        torch.cuda.synchronize()
        conv_s = time.time() - t0
        Xfull = torch.empty((n, F), device=device)
        parts = [Xfull[bounds[g]:bounds[g + 1]] for g in range(world)]
        dist.barrier()
        t1 = time.time()
        dist.all_gather(parts, X)
        torch.cuda.synchronize()
        allgather_s = time.time() - t1

        import types
        dg = types.SimpleNamespace(nnz=tl.nnz, halo_rows=0)

        def spmm():
            T.bcsr_spmm(tl, Xfull, Y, tc_threshold=args.tc_threshold, rs=rs)
    else:
        dg = DistGraph(lrp, lcol, bounds, rs_local=rs, cs_global=None, tc_threshold=args.tc_threshold,
                       transport=args.transport)
        del lcol
        torch.cuda.empty_cache()
        torch.cuda.synchronize()
        conv_s = time.time() - t0

        def spmm():
            dg.spmm(X, Y)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        spmm()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        spmm()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=device)
    tot = torch.tensor([float(dg.nnz), float(dg.halo_rows)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    ms = t.item()
    nnz_total, halo_total = tot.tolist()
    transport = getattr(dg, "transport", "none")
    if hasattr(dg, "close"):
        dev_err = dg.device_error()
        dg.close()  # collective: every rank
        if dev_err:
            raise RuntimeError(f"halo exchange device error {dev_err}")
    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    b_alg = 4 * F * (n + n) + 8 * nnz_total + 4 * (n + 1)  # the whole job's SpMM
    achieved = b_alg / (ms * 1e-3) / 1e9
    line = {
        "metric": "SpMM GFLOP/s (2*nnz*F)",
        "value": round(2.0 * nnz_total * F / (ms * 1e-3) / 1e9, 2),
        "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded directed R-MAT, torch GPU generator seed 4)",
        "config": {"workload": "config5: R-MAT 2^%d nodes, %d directed edges (16 per node), "
                               "deduplicated, row-normalised, F=128, forward A.X" % (scale, edges),
                   "rmat_scale": scale, "nnz_total": int(nnz_total), "nnz_rank0": dg.nnz,
                   "halo_rows_total": int(halo_total), "tc_threshold": args.tc_threshold,
                   "parallelism": (f"{world}-way 1D row partition, " +
                                   ("X all-gathered once at set-up (static input features)"
                                    if replicated else f"halo exchanged every step ({transport})"))
                   if world > 1 else "1 GPU",
                   "transport": transport,
                   "allgather_s": None if allgather_s is None else round(allgather_s, 3),
                   "gen_s": round(gen_s, 2), "convert_s": round(conv_s, 2)},
        "roofline": {"bound": "hbm", "achieved": round(achieved / world, 1), "peak": peak,
                     "unit": "GB/s per GPU", "frac": round(achieved / world / peak, 4),
                     "traffic": None, "kernel": "forward SpMM (exchange + local + halo tiles)",
                     "peak_kind": peak_kind},
        "e2e": None,
        "gpu_launches": args.steps * (2 if world == 1 or replicated else
                                      6 if transport == "peer" else 5),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_profile(args):
    """The command ncu captures: build config 2, then only the named kernel."""
    import torch
    from tcc_b200 import tiles as T
    device = torch.device("cuda", 0)
    rowptr, col, s = gen_config2(args.scale, device)
    n = rowptr.numel() - 1
    X = features(n, 1000, device)
    if args.profile == "swtcf":
        from tcc_b200 import swtcf
        m = swtcf.SWTCFMatrix(n, n, col.numel(), 16)
        ws = swtcf.SWTCFConvertWorkspace(col.numel(), n, 16)
        swtcf.convert_csr(rowptr, col, m, ws)
        ws.free()
        Y = torch.zeros((n, F), device=device)
        for _ in range(args.steps):
            swtcf.spmm(m, X, Y, tc_threshold=12)
    elif args.profile == "fwd":
        tl = T.from_csr(rowptr, col, n, n, kind="bcsr")
        Y = torch.empty((n, F), device=device)
        for _ in range(args.steps):
            T.bcsr_spmm(tl, X, Y, tc_threshold=args.tc_threshold, rs=s, cs=s)
    else:
        tl = T.from_csr(rowptr, col, n, n, kind="bcsc")
        Gm = features(n, 1001, device)
        Z = torch.empty((n, F), device=device)
        for _ in range(args.steps):
            T.bcsc_spmm_t(tl, Gm, Z, tc_threshold=args.tc_threshold, rs=s, cs=s)
    torch.cuda.synchronize()
    print(f"profile {args.profile}: {args.steps} launches done", flush=True)


# -------------------------------------------------------- reference arm ----

def run_reference(args, rank, world, local_rank):
    """The reference's CPU path on our arm's workload (rank 0 only): the CPU
    restatement (oracle/, OpenMP fp32 CSR SpMM) and torch.sparse.mm, each on a
    bounded row sample of config 2, the faster reported as the value; the
    reference's own CUDA kernels on the same graph alongside (informative)."""
    if rank != 0:
        return
    import torch
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    rowptr, col, s = gen_config2(args.scale, dev)
    n = rowptr.numel() - 1
    g = host_csr(rowptr, col, n)
    sh = s.cpu().numpy()
    X = features(n, 1000, dev)
    Xh = X.cpu().numpy()
    # each step a bounded sample (~2 s of CPU work), so the whole run stays
    # within a few minutes at the driver's --steps / --warmup
    for _ in range(args.warmup):
        cpu_baseline(g, Xh, sh, sh, budget_s=1.0)
    vals = []
    for _ in range(args.steps):
        cb = cpu_baseline(g, Xh, sh, sh, budget_s=2.0)
        vals.append(cb["value"])
    cb["value"] = statistics.median(vals)
    ts = torch_sparse_baseline(rowptr, col, s, X, budget_s=4.0)
    best = cb if cb["value"] >= ts["value"] else ts
    value = best["value"]
    line = {"impl": "reference", "metric": "SpMM GFLOP/s (2*nnz*F)", "value": value,
            "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded R-MAT, torch GPU generator seed 1)",
            "config": {"workload": workload_name(world, args.dist_mode), "rmat_scale": args.scale,
                       "nodes": n, "nnz_total": g.nnz, "F": F},
            "cpu_baseline": dict(best, kind="port" if best is cb else "reference",
                                 note="faster of the OpenMP port (median of --steps samples) "
                                      "and torch.sparse.mm"),
            "cpu_port": cb, "cpu_torch_sparse": ts,
            "e2e": {"value": value, "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    line["reference_gpu"] = reference_gpu_kernels(g, Xh, sh)
    print(json.dumps(line), flush=True)


def reference_gpu_kernels(g, Xh, sh):
    """The reference's own CUDA kernels built from source for sm_100a
    (oracle/_ref) on config 2, informative: launchSWTCFSpMM (pattern-only,
    forward), the spmm_cnic BCSR kernel (tf32_spmm_bcsr, the counterpart of our
    forward pull) and BCSC kernel (tf32_spmm_bcsc) on the canonical tiles of the
    same graph, and convertCOOToSWTCF's GEdges/s."""
    import torch
    out = {}
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if O.ref_lib() is None or not torch.cuda.is_available():
            return {"error": "reference build absent"}
        dst, src = g.coo()
        _, ms = O.ref_swtcf_spmm(g.rows, g.cols, dst, src, Xh, tc_threshold=12, warmup=2, reps=5)
        out["launchSWTCFSpMM"] = {"ms": round(ms, 3),
                                  "gflops": round(2.0 * g.nnz * F / (ms * 1e-3) / 1e9, 2)}
        cms = O.ref_swtcf_convert_ms(g.rows, g.cols, dst, src, warmup=1, reps=5)
        out["convertCOOToSWTCF"] = {"ms": round(cms, 3),
                                    "gedges_per_s": round(g.nnz / (cms * 1e-3) / 1e9, 3)}
        bcsr = O.bcsr_from_csr(g)
        _, ms_r = O.ref_cnic_spmm(g.rows, g.cols, Xh, bcsr=bcsr, warmup=2, reps=5)
        out["tf32_spmm_bcsr"] = {"ms": round(ms_r, 3),
                                 "gflops": round(2.0 * g.nnz * F / (ms_r * 1e-3) / 1e9, 2),
                                 "note": "pattern-only, TF32 on every tile, memset of C included"}
        del bcsr
        bcsc = O.bcsc_from_csr(g)
        _, ms_c = O.ref_cnic_spmm(g.rows, g.cols, Xh, bcsc=bcsc, warmup=2, reps=5)
        out["tf32_spmm_bcsc"] = {"ms": round(ms_c, 3),
                                 "gflops": round(2.0 * g.nnz * F / (ms_c * 1e-3) / 1e9, 2),
                                 "note": "pattern-only push over column windows, fp32 atomics"}
    except Exception as e:  # informative only
        out["error"] = f"{type(e).__name__}: {str(e)[:200]}"
    return out


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and rank == 0:
        print(f"note: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.workload == "gcn4":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference GCN trainer needs DGL "
                                  "and its absent ipc_service sampler"}), flush=True)
            return
        from tcc_b200 import train_gcn
        train_gcn.main(["--epochs", str(max(args.steps, 2))] +
                       (["--aggregate-first"] if args.aggregate_first else []))
        return
    pg = False
    if world > 1 and args.impl == "ours":
        import datetime
        import torch
        import torch.distributed as dist
        from tcc_b200.partition import nccl_options
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                pg_options=nccl_options(),
                                device_id=torch.device("cuda", local_rank))
        pg = True
    if args.profile:
        run_profile(args)
        return
    try:
        if args.impl == "ours" and args.workload == "config5":
            run_config5(args, rank, world, local_rank)
        elif args.impl == "reference" and args.workload == "config5":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no "
                                  "row-partitioned multi-GPU SpMM"}), flush=True)
        elif args.impl == "ours":
            run_ours(args, rank, world, local_rank)
        else:
            run_reference(args, rank, world, local_rank)
    finally:
        if pg:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
