"""Benchmark of the tcc graph-aggregation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload spmm|gcn4|config5] [--dist-mode replicated|exchange]

Workload (config 2 of the benchmark set): seeded R-MAT graph, 2^20 nodes, 16M directed
edges (a,b,c,d = 0.57,0.19,0.19,0.05) symmetrised, deduplicated, self-loops
added; GCN normalisation D^-1/2 (A+I) D^-1/2 fused as diagonal scales; X, G
fp32 [N x 128] ~ N(0,1).  One step = forward SpMM A.X plus the transposed SpMM
A^T.G (the backward pass; A is symmetric, so both run over the BCSR tiles).
Metric: SpMM GFLOP/s = 2 nnz F per SpMM, whole job.

Multi-GPU (torchrun, one process per GPU; rank 0 prints the line with the max
time over ranks):
  --dist-mode replicated (default): strong scaling -- the same config-2 job is
      split into nnz-balanced row blocks; X and G are resident on every GPU
      (the e2e leg copies each rank's row blocks from the host and all-gathers
      them over NCCL every step);
  --dist-mode exchange: weak scaling -- the R-MAT scale grows with log2(N)
      (about 32 M nonzeros per GPU) and every SpMM exchanges the compacted
      feature halo with an NCCL all-to-all overlapped with the local tiles.
--workload gcn4 reports config 4's GCN epoch time (tcc_b200.train_gcn);
--workload config5 the scale-26 forward SpMM (strong scaling).

--impl reference: the reference path has no CPU implementation of its own (its
SpMMs are CUDA kernels); this arm times the CPU restatement of the path
(oracle/, fp32 CSR SpMM over all host threads) on a bounded row sample of the
same workload, and reports the reference's own CUDA kernel (built from source
for sm_100a into oracle/_ref) on the same graph alongside.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import shutil
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

def workload_name(weak: bool) -> str:
    if weak:
        return ("config2 per GPU: R-MAT 2^(20+log2 N) nodes, 16 directed edges per node "
                "symmetrised+dedup+self-loops, GCN-normalised, F=128, forward A.X + transposed "
                "A^T.G over BCSR tiles, halo exchanged every step")
    return ("config2: R-MAT 2^20 nodes, 16 directed edges per node symmetrised+dedup+self-loops, "
            "GCN-normalised, F=128, forward A.X + transposed A^T.G over BCSR tiles; on N GPUs "
            "split by rows with X and G resident on every GPU")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--tc-threshold", type=int, default=12)
    p.add_argument("--scale", type=int, default=20, help="R-MAT scale (20 = config 2)")
    p.add_argument("--dist-mode", choices=["replicated", "exchange"], default="replicated",
                   help="spmm on N > 1 GPUs: 'replicated' = the config-2 job split by rows "
                        "(strong scaling; X and G resident on every GPU, all-gathered from the "
                        "ranks' row blocks in the e2e leg); 'exchange' = config 2 per GPU "
                        "(weak scaling, scale 20 + log2 N) with the X halo exchanged every step")
    p.add_argument("--workload", choices=["spmm", "gcn4", "config5"], default="spmm",
                   help="spmm: the config-2 SpMM step (headline, weak scaling); gcn4: config-4 GCN "
                        "epoch time (tcc_b200.train_gcn, epochs = --steps); config5: the scale-26 "
                        "forward SpMM, strong scaling")
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


def build_workload(scale, device, world=1, rank=0, tc_threshold=12):
    """The rank's share of the R-MAT graph (scale `scale`, 16 * 2^scale directed
    edges, seed 1, symmetrised + dedup + self-loops; GPU generator), partitioned
    by nonzeros across `world` ranks, with GCN scales and seeded features."""
    import torch
    from tcc_b200 import graphs as G
    from tcc_b200.partition import DistGraph, balanced_bounds
    t0 = time.time()
    rowptr, col, _ = G.rmat_gpu(scale, 16 << scale, seed=1, device=device)
    deg = torch.diff(rowptr)
    n = deg.numel()
    s = torch.where(deg > 0, deg.to(torch.float64).clamp(min=1).rsqrt(),
                    torch.zeros_like(deg, dtype=torch.float64)).to(torch.float32)
    bounds = balanced_bounds(deg, world)
    r0, r1 = bounds[rank], bounds[rank + 1]
    lrp = (rowptr[r0:r1 + 1] - rowptr[r0]).contiguous()
    lcol = col[rowptr[r0]:rowptr[r1]].contiguous()
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    X = torch.randn((r1 - r0, 128), generator=gen, device=device)
    Gm = torch.randn((r1 - r0, 128), generator=gen, device=device)
    torch.cuda.synchronize()
    gen_s = time.time() - t0
    t0 = time.time()
    dg = DistGraph(lrp, lcol, bounds, rs_local=s[r0:r1].contiguous(), cs_global=s,
                   tc_threshold=tc_threshold)
    torch.cuda.synchronize()
    conv_s = time.time() - t0
    return dict(dg=dg, n=n, bounds=bounds, rowptr=lrp, col=lcol, s=s, X=X, G=Gm,
                gen_s=gen_s, conv_s=conv_s, full_rowptr=rowptr, full_col=col)


def build_replicated(scale, device, world=1, rank=0, tc_threshold=12):
    """Config 2 split by rows for strong scaling: every rank generates the whole
    graph (same seeds), keeps its nnz-balanced row block tiled against the
    global columns, and holds full copies of X and G (the same seeded draws on
    every rank, i.e. what an all-gather of the row blocks produces)."""
    import torch
    from tcc_b200 import graphs as G
    from tcc_b200 import tiles as T
    from tcc_b200.partition import balanced_bounds
    t0 = time.time()
    rowptr, col, _ = G.rmat_gpu(scale, 16 << scale, seed=1, device=device)
    deg = torch.diff(rowptr)
    n = deg.numel()
    s = torch.where(deg > 0, deg.to(torch.float64).clamp(min=1).rsqrt(),
                    torch.zeros_like(deg, dtype=torch.float64)).to(torch.float32)
    bounds = balanced_bounds(deg, world)
    r0, r1 = bounds[rank], bounds[rank + 1]
    lrp = (rowptr[r0:r1 + 1] - rowptr[r0]).contiguous()
    lcol = col[rowptr[r0]:rowptr[r1]].contiguous()
    gen = torch.Generator(device=device)
    gen.manual_seed(1000)
    X = torch.randn((n, 128), generator=gen, device=device)
    Gm = torch.randn((n, 128), generator=gen, device=device)
    torch.cuda.synchronize()
    gen_s = time.time() - t0
    t0 = time.time()
    tl = T.from_csr(lrp, lcol, r1 - r0, n, kind="bcsr")
    torch.cuda.synchronize()
    conv_s = time.time() - t0
    return dict(tiles=tl, n=n, bounds=bounds, r0=r0, r1=r1, rowptr=lrp, col=lcol, s=s,
                rs=s[r0:r1].contiguous(), X=X, G=Gm, gen_s=gen_s, conv_s=conv_s)


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


def run_ours(args, rank, world, local_rank):
    import math
    import torch
    import torch.distributed as dist
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    replicated = args.dist_mode == "replicated" or world == 1
    scale = args.scale if replicated else args.scale + int(round(math.log2(world)))
    F = 128
    stream = torch.cuda.current_stream()
    if replicated:
        W = build_replicated(scale, device, world, rank, args.tc_threshold)
        tl, rs_loc, s_all = W["tiles"], W["rs"], W["s"]
        X, Gm = W["X"], W["G"]  # full copies on every GPU
        r0, r1 = W["r0"], W["r1"]
        Y = torch.empty((r1 - r0, F), device=device)
        Z = torch.empty_like(Y)
        from tcc_b200 import tiles as T

        def step(fwd_events=None):
            if fwd_events:
                fwd_events[0].record(stream)
            T.bcsr_spmm(tl, X, Y, tc_threshold=args.tc_threshold, rs=rs_loc, cs=s_all)
            if fwd_events:
                fwd_events[1].record(stream)
            # A^T G: A is symmetric, so the rank's rows of A^T are its rows of A
            T.bcsr_spmm(tl, Gm, Z, tc_threshold=args.tc_threshold, rs=rs_loc, cs=s_all)

        import types
        dg = types.SimpleNamespace(nnz=tl.nnz, halo_rows=0, n_local=r1 - r0, tiles_halo=None)
    else:
        W = build_workload(scale, device, world, rank, args.tc_threshold)
        dg = W["dg"]
        X, Gm = W["X"], W["G"]
        Y = torch.empty_like(X)
        Z = torch.empty_like(Gm)

        def step(fwd_events=None):
            if fwd_events:
                fwd_events[0].record(stream)
            dg.spmm(X, Y)
            if fwd_events:
                fwd_events[1].record(stream)
            dg.spmm_t(Gm, Z)  # A^T G: A is symmetric, same partition and tiles

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    fwd = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(fwd[i])
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in fwd)
    t = torch.tensor([ms, fwd_ms], device=device)
    tot = torch.tensor([float(dg.nnz), float(dg.halo_rows)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    ms, fwd_ms = t.tolist()
    nnz_total, halo_total = tot.tolist()
    ms_per_step = ms / args.steps
    flops_step = 2 * (2.0 * nnz_total * F)

    # end to end through the public API, every step: the rank's inputs from
    # pinned host memory to the device (replicated mode: its row blocks of X and
    # G, then an NCCL all-gather builds the full copies; exchange mode: its
    # rows, the halo moving inside the passes), both passes, and its rows of
    # Y, Z back to pinned host memory
    if replicated:
        hX = X[r0:r1].cpu().pin_memory()
        hG = Gm[r0:r1].cpu().pin_memory()
        bounds = W["bounds"]
        xparts = [X[bounds[g]:bounds[g + 1]] for g in range(world)]
        gparts = [Gm[bounds[g]:bounds[g + 1]] for g in range(world)]
    else:
        hX = X.cpu().pin_memory()
        hG = Gm.cpu().pin_memory()
    hY = torch.empty(tuple(Y.shape)).pin_memory()
    hZ = torch.empty(tuple(Z.shape)).pin_memory()

    def e2e_step():
        if replicated:
            X[r0:r1].copy_(hX, non_blocking=True)
            Gm[r0:r1].copy_(hG, non_blocking=True)
            if world > 1:
                dist.all_gather(xparts, X[r0:r1])
                dist.all_gather(gparts, Gm[r0:r1])
        else:
            X.copy_(hX, non_blocking=True)
            Gm.copy_(hG, non_blocking=True)
        step()
        hY.copy_(Y, non_blocking=True)
        hZ.copy_(Z, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([a0.elapsed_time(a1) / e2e_steps], device=device)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = e2e_ms.item()

    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    n_loc = dg.n_local
    n_in = W["n"] if replicated else n_loc  # rows of X a rank's forward pass reads
    b_alg = 4 * F * (n_in + n_loc) + 8 * dg.nnz + 4 * (n_loc + 1)
    achieved = b_alg / (fwd_ms * 1e-3) / 1e9
    # per SpMM: pull + zero pass on the local tiles; with a halo also the pack
    # kernel and pull + zero pass on the halo tiles
    per_step_launches = 2 * (2 if dg.tiles_halo is None else 5)
    line = {
        "metric": "SpMM GFLOP/s (2*nnz*F)",
        "value": round(flops_step / (ms_per_step * 1e-3) / 1e9, 2),
        "unit": "GFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if replicated else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded R-MAT, torch GPU generator seed 1)",
        "config": {"workload": workload_name(not replicated), "rmat_scale": scale, "nodes": W["n"],
                   "nnz_total": int(nnz_total), "nnz_rank0": dg.nnz, "F": F,
                   "halo_rows_total": int(halo_total), "tc_threshold": args.tc_threshold,
                   "l2": "inputs larger than L2 (X, G 512 MiB per GPU)",
                   "parallelism": ("1 GPU" if world == 1 else
                                   f"{world}-way 1D row partition (nnz-balanced); X, G resident "
                                   "on every GPU (all-gathered from the row blocks in the e2e leg)"
                                   if replicated else
                                   f"{world}-way 1D row partition (nnz-balanced), compacted "
                                   "halo all-to-all over NCCL overlapped with local tiles"),
                   "convert_s": round(W["conv_s"], 3)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profiled_traffic(f"{pull_kernel_name(F)}_config2") if world == 1 else None,
                     "kernel": f"{pull_kernel_name(F)}, forward SpMM" + (" (local + halo tiles and the "
                                                              "exchange)" if not replicated else
                                                              " (rank 0's rows)" if world > 1 else ""),
                     "fwd_ms": round(fwd_ms, 4), "alg_bytes_per_launch": b_alg,
                     "peak_kind": peak_kind},
        "e2e": {"value": round(flops_step / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s",
                "h2d_bytes_per_step": int(hX.numel() * 4 + hG.numel() * 4),
                "d2h_bytes_per_step": int(hY.numel() * 4 + hZ.numel() * 4),
                "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": per_step_launches * args.steps,
        "clocks": clocks,
    }
    if world == 1:
        line["swtcf_forward"] = swtcf_forward(W["rowptr"], W["col"], W["n"], X, device)
        g = host_csr(W["rowptr"], W["col"], W["n"])
        s = W["s"].cpu().numpy()
        line["cpu_baseline"] = cpu_baseline(g, X.cpu().numpy(), s, s)
    print(json.dumps(line), flush=True)


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
        dg = DistGraph(lrp, lcol, bounds, rs_local=rs, cs_global=None, tc_threshold=args.tc_threshold)
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
                                    if replicated else "halo exchanged every step"))
                   if world > 1 else "1 GPU",
                   "allgather_s": None if allgather_s is None else round(allgather_s, 3),
                   "gen_s": round(gen_s, 2), "convert_s": round(conv_s, 2)},
        "roofline": {"bound": "hbm", "achieved": round(achieved / world, 1), "peak": peak,
                     "unit": "GB/s per GPU", "frac": round(achieved / world / peak, 4),
                     "traffic": None, "kernel": "forward SpMM (exchange + local + halo tiles)",
                     "peak_kind": peak_kind},
        "e2e": None,
        "gpu_launches": args.steps * (2 if world == 1 or replicated else 5),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_profile(args):
    import torch
    device = torch.device("cuda", 0)
    W = build_workload(args.scale, device, tc_threshold=args.tc_threshold)
    if args.profile == "swtcf":
        from tcc_b200 import swtcf
        rowptr, col, n = W["full_rowptr"], W["full_col"], W["n"]
        m = swtcf.SWTCFMatrix(n, n, col.numel(), 16)
        ws = swtcf.SWTCFConvertWorkspace(col.numel(), n, 16)
        swtcf.convert_csr(rowptr, col, m, ws)
        ws.free()
        Y = torch.zeros((n, 128), device=device)
        for _ in range(args.steps):
            swtcf.spmm(m, W["X"], Y, tc_threshold=12)
        torch.cuda.synchronize()
        print(f"profile swtcf: {args.steps} launches done", flush=True)
        return
    dg = W["dg"]
    src = W["X"] if args.profile == "fwd" else W["G"]
    out = torch.empty_like(src)
    for _ in range(args.steps):
        dg.spmm(src, out)
    torch.cuda.synchronize()
    print(f"profile {args.profile}: {args.steps} launches done", flush=True)


def run_reference(args, rank, world, local_rank):
    if rank != 0:
        return
    import math
    import torch
    from tcc_b200 import graphs as G
    # our arm's workload: the config-2 graph at every N (strong scaling) by
    # default, scale 20 + log2 N with --dist-mode exchange (weak scaling)
    weak = args.dist_mode == "exchange" and world > 1
    scale = args.scale + (int(round(math.log2(world))) if weak else 0)
    # the same graph as our arm (torch's CUDA and CPU generators draw different streams)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    rowptr, col, _ = G.rmat_gpu(scale, 16 << scale, seed=1, device=dev)
    g = host_csr(rowptr, col, rowptr.numel() - 1)
    del rowptr, col
    deg = g.degrees().astype(np.float64)
    s = np.where(deg > 0, 1.0 / np.sqrt(np.maximum(deg, 1)), 0).astype(np.float32)
    gen = torch.Generator().manual_seed(1000)
    X = torch.randn((g.rows, 128), generator=gen).numpy()
    for _ in range(args.warmup):
        cb = cpu_baseline(g, X, s, s, budget_s=3.0)
    vals = []
    for _ in range(args.steps):
        cb = cpu_baseline(g, X, s, s, budget_s=6.0)
        vals.append(cb["value"])
    value = statistics.median(vals)
    cb["value"] = value
    line = {"impl": "reference", "metric": "SpMM GFLOP/s (2*nnz*F)", "value": value,
            "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak" if weak else "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded R-MAT, torch generator seed 1)",
            "config": {"workload": workload_name(weak), "rmat_scale": scale, "nodes": g.rows,
                       "nnz": g.nnz, "F": 128},
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    try:  # the reference's own CUDA SpMM, built from source for sm_100a (informative)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if O.ref_lib() is not None and torch.cuda.is_available():
            dst, src = g.coo()
            _, ms = O.ref_swtcf_spmm(g.rows, g.cols, dst, src, X, tc_threshold=12, warmup=2,
                                     reps=5)
            line["reference_gpu_kernel"] = {
                "what": "launchSWTCFSpMM (src/swtcf_spmm.cu) built for sm_100a, pattern-only, "
                        "forward only", "ms": round(ms, 3),
                "value": round(2.0 * g.nnz * 128 / (ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s"}
    except Exception as e:  # informative only
        line["reference_gpu_kernel"] = {"error": str(e)[:200]}
    print(json.dumps(line), flush=True)


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
