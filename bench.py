"""Benchmark of the tcc graph-aggregation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: seeded R-MAT graph, 2^20 nodes, 16M directed
edges (a,b,c,d = 0.57,0.19,0.19,0.05) symmetrised, deduplicated, self-loops
added; GCN normalisation D^-1/2 (A+I) D^-1/2 fused as diagonal scales; X, G
fp32 [N x 128] ~ N(0,1).  One step = forward SpMM A.X over BCSR tiles plus the
transposed SpMM A^T.G over BCSC tiles (the backward pass).  Metric: SpMM
GFLOP/s = 2 nnz F per SpMM, whole job.

Multi-GPU (torchrun, one process per GPU): every rank runs the same per-GPU
workload (weak scaling, no data-path collective); rank 0 prints the line with
the max time over ranks.

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
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = ("config2: R-MAT 2^20 nodes, 16M directed edges symmetrised+dedup+self-loops, "
            "GCN-normalised, F=128, forward A.X (BCSR) + transposed A^T.G (BCSC)")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--tc-threshold", type=int, default=12)
    p.add_argument("--scale", type=int, default=20, help="R-MAT scale (20 = config 2)")
    p.add_argument("--profile", choices=["fwd", "bwd"], default=None,
                   help="build the workload, run only the forward (or transposed) pull "
                        "--steps times and exit: the command ncu captures")
    return p.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            j = json.load(f)
        return j.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


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
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_rank{device_index}.csv")
        self.idx = device_index

    def start(self):
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
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
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_workload(scale, device):
    import torch
    from tcc_b200 import graphs as G
    from tcc_b200 import tiles
    t0 = time.time()
    g = G.rmat(scale, 16 << scale, seed=1)
    rs, cs = G.gcn_scales(g)
    X = G.features(g.cols, 128, seed=1)
    Gm = G.features(g.rows, 128, seed=11)
    gen_s = time.time() - t0
    rp = torch.from_numpy(g.rowptr.view(np.int64)).to(device)
    col = torch.from_numpy(g.col.view(np.int32)).to(device)
    torch.cuda.synchronize()
    t0 = time.time()
    bcsr = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    bcsc = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    torch.cuda.synchronize()
    conv_s = time.time() - t0
    return dict(g=g, rs=rs, cs=cs, X=X, G=Gm, rp=rp, col=col, bcsr=bcsr, bcsc=bcsc,
                gen_s=gen_s, conv_s=conv_s)


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
    import torch
    import torch.distributed as dist
    from tcc_b200 import tiles
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    W = build_workload(args.scale, device)
    g, bcsr, bcsc = W["g"], W["bcsr"], W["bcsc"]
    E, F = g.nnz, 128
    rs = torch.from_numpy(W["rs"]).to(device)
    cs = torch.from_numpy(W["cs"]).to(device)
    X = torch.from_numpy(W["X"]).to(device)
    Gm = torch.from_numpy(W["G"]).to(device)
    Y = torch.empty((g.rows, F), device=device)
    Z = torch.empty((g.cols, F), device=device)
    thr = args.tc_threshold
    stream = torch.cuda.current_stream()

    def step(fwd_events=None):
        if fwd_events:
            fwd_events[0].record(stream)
        tiles.bcsr_spmm(bcsr, X, Y, tc_threshold=thr, rs=rs, cs=cs)
        if fwd_events:
            fwd_events[1].record(stream)
        # transposed pass: Z = diag(cs) A^T diag(rs) G
        tiles.bcsc_spmm_t(bcsc, Gm, Z, tc_threshold=thr, rs=rs, cs=cs)

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
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_ms = t.tolist()
    ms_per_step = ms / args.steps
    flops_step = 2 * (2.0 * E * F)

    # end to end through the public API: pinned host X, G -> device, both passes,
    # Y, Z -> pinned host, every step
    hX = torch.from_numpy(W["X"]).pin_memory()
    hG = torch.from_numpy(W["G"]).pin_memory()
    hY = torch.empty((g.rows, F), dtype=torch.float32).pin_memory()
    hZ = torch.empty((g.cols, F), dtype=torch.float32).pin_memory()

    def e2e_step():
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
    b_alg = 4 * F * (g.rows + g.cols) + 8 * E + 4 * (g.rows + 1)
    achieved = b_alg / (fwd_ms * 1e-3) / 1e9
    line = {
        "metric": "SpMM GFLOP/s (2*nnz*F)",
        "value": round(world * flops_step / (ms_per_step * 1e-3) / 1e9, 2),
        "unit": "GFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded R-MAT, numpy PCG64 seed 1)",
        "config": {"workload": WORKLOAD, "nodes": g.rows, "nnz": E, "F": F,
                   "tiles_bcsr": bcsr.num_TCBlocks, "tc_threshold": thr,
                   "l2": "inputs larger than L2 (X, G 512 MiB each)",
                   "parallelism": f"{world} independent per-GPU replicas" if world > 1 else "1 GPU",
                   "convert_s": round(W["conv_s"], 3)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profiled_traffic("pull_kernel_config2"),
                     "kernel": "pull_kernel (BCSR forward)", "fwd_ms": round(fwd_ms, 4),
                     "alg_bytes_per_launch": b_alg, "peak_kind": peak_kind},
        "e2e": {"value": round(world * flops_step / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GFLOP/s",
                "h2d_bytes_per_step": int(hX.numel() * 4 + hG.numel() * 4),
                "d2h_bytes_per_step": int(hY.numel() * 4 + hZ.numel() * 4),
                "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": 4 * args.steps,
        "clocks": clocks,
    }
    line["cpu_baseline"] = cpu_baseline(g, W["X"], W["rs"], W["cs"])
    print(json.dumps(line), flush=True)


def run_profile(args):
    import torch
    from tcc_b200 import tiles
    device = torch.device("cuda", 0)
    W = build_workload(args.scale, device)
    g = W["g"]
    rs = torch.from_numpy(W["rs"]).to(device)
    cs = torch.from_numpy(W["cs"]).to(device)
    if args.profile == "fwd":
        X = torch.from_numpy(W["X"]).to(device)
        Y = torch.empty((g.rows, 128), device=device)
        for _ in range(args.steps):
            tiles.bcsr_spmm(W["bcsr"], X, Y, tc_threshold=args.tc_threshold, rs=rs, cs=cs)
    else:
        Gm = torch.from_numpy(W["G"]).to(device)
        Z = torch.empty((g.cols, 128), device=device)
        for _ in range(args.steps):
            tiles.bcsc_spmm_t(W["bcsc"], Gm, Z, tc_threshold=args.tc_threshold, rs=rs, cs=cs)
    torch.cuda.synchronize()
    print(f"profile {args.profile}: {args.steps} launches done", flush=True)


def run_reference(args, rank, world, local_rank):
    if rank != 0:
        return
    from tcc_b200 import graphs as G
    g = G.rmat(args.scale, 16 << args.scale, seed=1)
    rs, cs = G.gcn_scales(g)
    X = G.features(g.cols, 128, seed=1)
    for _ in range(args.warmup):
        cb = cpu_baseline(g, X, rs, cs, budget_s=3.0)
    vals = []
    for _ in range(args.steps):
        cb = cpu_baseline(g, X, rs, cs, budget_s=6.0)
        vals.append(cb["value"])
    value = statistics.median(vals)
    cb["value"] = value
    line = {"impl": "reference", "metric": "SpMM GFLOP/s (2*nnz*F)", "value": value,
            "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded R-MAT, numpy PCG64 seed 1)",
            "config": {"workload": WORKLOAD, "nodes": g.rows, "nnz": g.nnz, "F": 128},
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    try:  # the reference's own CUDA SpMM, built from source for sm_100a (informative)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if O.ref_lib() is not None:
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
    pg = False
    if world > 1 and args.impl == "ours":
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        pg = True
    if args.profile:
        run_profile(args)
        return
    try:
        if args.impl == "ours":
            run_ours(args, rank, world, local_rank)
        else:
            run_reference(args, rank, world, local_rank)
    finally:
        if pg:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
