"""Full-graph 2-layer GCN training on tcc_b200's SpMM, one process per GPU.

The reference trains the GCN of train/tcgnn_conv_release.py:196-268 (GCNConv =
aggregate, then transform, :169-194) with DDP across GPUs (:434-435).  Here the
graph is 1D row-partitioned (tcc_b200.partition) and every rank trains on its
own rows:

* layer 1 (F_in -> hidden): Z1 = Â[P_g, :] · X gathered straight from the rank's
  hot/cold feature store (hot rows in HBM, cold rows in pinned host memory read
  zero-copy, the reference's mixed gather) -- no exchange, since every rank's
  store holds all features; H1 = dropout(relu(Z1 · W1));
* layer 2 (hidden -> classes): Z2 = Â · H1 over the partition (halo exchange of
  H1 rows), logits = Z2 · W2;
* backward: Âᵀ = Â (the graphs are symmetric and Â = D^-½(A+I)D^-½), so the
  layer-2 input gradient is the same distributed SpMM on dZ2; layer 1 needs no
  input gradient;
* the weight gradients are summed across ranks with one all-reduce of a flat
  buffer (DDP's gradient all-reduce, issued explicitly so every rank's
  collectives run in the same order as its halo exchanges), then Adam.

Cold feature rows stay in pinned host memory; each epoch the ones this rank's
tiles read are brought into an HBM staging buffer on a side stream, overlapped
with the previous epoch: one bulk copy when the rank reads every cold row, the
row-gather kernel otherwise (``--cold-zero-copy`` reads them zero-copy in every
gather instead, one PCIe read per gather; staging is only used when the staged
rows fit a quarter of free HBM).

Layer order by width: a layer aggregates at the narrower of its input and
output widths.  Layer 1 (100 -> 256) aggregates first; layer 2 (256 -> 47)
transforms first, Â·(H1·W2), so both of its SpMMs run 48 wide instead of 256
(``transform_first``; None picks by width, ``--aggregate-first`` keeps the
reference's order for every layer).  ``--save`` / ``--resume`` write and read a
checkpoint of the weights, the Adam state and the epoch count (the reference
saves none).

Run: ``python -m tcc_b200.train_gcn`` (1 GPU) or under torch.distributed.run.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import time

import numpy as np
import torch
import torch.distributed as dist

from . import graphs as G
from . import tiles as T
from .feature_store import FeatureStore
from .gcn import relu_dropout
from .partition import DistGraph, balanced_bounds, nccl_options, tile_balanced_bounds


def _store_aggregate(tiles_g: T.Tiles, store: FeatureStore, rs: torch.Tensor,
                     staged: bool = False) -> torch.Tensor:
    """Â[P_g, :] · X with X read from the store (whose rows carry the column
    scale); the row scale is applied here.  ``staged``: read the cold rows from
    the store's HBM staging buffer (this epoch's copy), else from pinned host
    memory, zero-copy."""
    import ctypes as C
    from . import _lib as L
    F = store.F
    W = tiles_g.num_windows
    full = torch.empty(((W + 1) * 8, F), dtype=torch.float32, device=rs.device)
    sc = tiles_g.scratch()
    s = tiles_g.struct()
    cold_ptr = store.cold_stage.data_ptr() if staged else store.cpu_ptr
    id_map = store.stage_id_map if staged else store.id_map
    L.call("tcc_cnic_forward_mixed", C.byref(s), None, C.c_void_p(id_map.data_ptr()),
           C.c_void_p(cold_ptr), C.c_void_p(store.cache_search_map.data_ptr()),
           C.c_void_p(store.gpu_ptrs.data_ptr()), store.capacity, C.c_void_p(full.data_ptr()), F, 0,
           C.c_void_p(sc.data_ptr()), sc.numel(), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    tiles_g._plan_ready = True
    n = tiles_g.num_rows
    return full[:n].mul_(rs[:, None])


class _DistAggregate(torch.autograd.Function):
    """Y = Â[P_g, :] · H over the partition; backward Âᵀ = Â (symmetric)."""

    @staticmethod
    def forward(ctx, dg: DistGraph, H: torch.Tensor):
        ctx.dg = dg
        return dg.spmm(H.contiguous())

    @staticmethod
    def backward(ctx, dY):
        return None, ctx.dg.spmm(dY.contiguous())


def build(cfg: dict, device, world: int, rank: int):
    """The rank's graph, tilings, feature store and labels."""
    n, edges, seed = cfg["nodes"], cfg["edges"], cfg["seed"]
    scale = max(1, math.ceil(math.log2(n)))
    t0 = time.time()
    rowptr, col, _ = G.rmat_gpu(scale, edges, seed=seed, device=device, n=n)
    deg = torch.diff(rowptr)
    if world > 1 and cfg.get("partition", "tiles") == "tiles":
        # equal pull work per rank: R-MAT's hub rows pack many nonzeros into
        # few tiles, so equal nonzeros leave the tail ranks slower
        full = T.from_csr(rowptr, col, n, n, kind="bcsr")
        bounds = tile_balanced_bounds(full.windowOffset, n, world)
        del full
    else:
        bounds = balanced_bounds(deg, world)
    r0, r1 = bounds[rank], bounds[rank + 1]
    s = deg.to(torch.float64).clamp(min=1).rsqrt().to(torch.float32)  # D^-1/2 of A + I
    lrp = (rowptr[r0:r1 + 1] - rowptr[r0]).contiguous()
    lcol = col[rowptr[r0]:rowptr[r1]].contiguous()
    del rowptr, col
    gen_s = time.time() - t0
    t0 = time.time()
    tiles_g = T.from_csr(lrp, lcol, r1 - r0, n, kind="bcsr")  # layer 1: global columns
    dg = DistGraph(lrp, lcol, bounds, rs_local=s[r0:r1].contiguous(), cs_global=s, tc_threshold=0)
    conv_s = time.time() - t0
    # features (same on every rank) and the hot/cold store, column scale folded in
    rng = np.random.Generator(np.random.PCG64(seed))
    X = rng.standard_normal((n, cfg["F_in"]), dtype=np.float32)
    store = FeatureStore(X, deg.cpu().numpy(), hot_fraction=cfg["hot_fraction"], device=device,
                         col_scale=s.cpu().numpy())
    del X
    lab_rng = np.random.Generator(np.random.PCG64(seed + 1))
    labeled = lab_rng.random(n) < cfg["label_fraction"]
    labels = lab_rng.integers(0, cfg["classes"], size=n)
    mine = np.nonzero(labeled[r0:r1])[0]
    lab_idx = torch.from_numpy(mine).to(device)
    lab_y = torch.from_numpy(labels[r0:r1][mine]).to(device)
    return dict(tiles_g=tiles_g, dg=dg, store=store, rs=s[r0:r1].contiguous(), lab_idx=lab_idx,
                lab_y=lab_y, n_lab=int(labeled.sum()), bounds=bounds, r0=r0, r1=r1,
                nnz=int(lcol.numel()), gen_s=gen_s, conv_s=conv_s)


def train(cfg: dict, device, world: int, rank: int, transform_first: bool | None = None):
    if transform_first is None:  # aggregate at the narrower width of layer 2
        transform_first = cfg["classes"] < cfg["hidden"]
    R = build(cfg, device, world, rank)
    torch.manual_seed(cfg["seed"])
    W1 = torch.empty(cfg["F_in"], cfg["hidden"], device=device)
    W2 = torch.empty(cfg["hidden"], cfg["classes"], device=device)
    torch.nn.init.xavier_uniform_(W1)
    torch.nn.init.xavier_uniform_(W2)
    W1.requires_grad_(True)
    W2.requires_grad_(True)
    params = [W1, W2]
    opt = torch.optim.Adam(params, lr=cfg["lr"])
    start_epoch = 0
    if cfg.get("resume"):
        ck = torch.load(cfg["resume"], map_location=device)
        with torch.no_grad():
            W1.copy_(ck["W1"])
            W2.copy_(ck["W2"])
        opt.load_state_dict(ck["opt"])
        start_epoch = int(ck["epoch"])
    # cold rows: streamed into an HBM staging buffer once per epoch on a side
    # stream (the copy for epoch e + 1 overlaps the rest of epoch e), or read
    # zero-copy from pinned host memory by every gather that touches them
    store = R["store"]
    # more than one GPU: the ranks stage the cold block cooperatively (each
    # copies a chunk over PCIe, an all-gather on its own communicator, so it
    # does not queue behind the halo exchanges, assembles the rest)
    stage_group = None
    if world > 1 and bool(cfg.get("cold_stage_coop", True)):
        stage_group = dist.new_group(backend="nccl", pg_options=nccl_options())
    staged = bool(cfg.get("cold_staging", True)) and store.enable_cold_staging(
        columns=R["tiles_g"].sparseIdx, force_gather=bool(cfg.get("cold_stage_gather", False)),
        group=stage_group)
    if stage_group is not None:
        # cooperative staging runs collectives: every rank stages, or none does
        agree = torch.tensor([1 if staged else 0], device=device)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN)
        staged = bool(agree.item())
        if not staged:
            store.stage_group = None
    if staged:
        side = torch.cuda.Stream(device=device)
        # the staging buffer and its row ids were made on the current stream
        # (the ids by an asynchronous gather): the side stream starts after them
        side.wait_stream(torch.cuda.current_stream())
        store.cold_stage.record_stream(side)  # written on the side stream
        if store.stage_ids is not None:
            store.stage_ids.record_stream(side)  # read on the side stream
        if getattr(store, "stage_chunk", None) is not None:
            store.stage_chunk.record_stream(side)  # the rank's chunk, written on the side stream
        ready = torch.cuda.Event()
        used = torch.cuda.Event()
        store.stage_cold(side)
        ready.record(side)
    drop_seed = (cfg["seed"] * 1000 + rank) << 20  # dropout draw of epoch e: drop_seed + e
    epoch_no = [start_epoch]
    cls_pad = (cfg["classes"] + 3) // 4 * 4  # transform-first SpMM width, multiple of 4

    def epoch(stage_next: bool):
        opt.zero_grad(set_to_none=True)
        if staged:
            # an unfinished copy shows up here, in this epoch's time
            torch.cuda.current_stream().wait_event(ready)
            Z1 = _store_aggregate(R["tiles_g"], store, R["rs"], staged=True)
            if stage_next:  # next epoch's copy, overlapping the rest of this one
                used.record()
                side.wait_event(used)
                store.stage_cold(side)
                ready.record(side)
        else:
            Z1 = _store_aggregate(R["tiles_g"], store, R["rs"])
        # relu + dropout fused (one pass; the backward reads only H1)
        H1 = relu_dropout(Z1 @ W1, cfg["dropout"], drop_seed + epoch_no[0])
        epoch_no[0] += 1
        if transform_first:
            P = torch.nn.functional.pad(H1 @ W2, (0, cls_pad - cfg["classes"]))
            logits = _DistAggregate.apply(R["dg"], P)[:, :cfg["classes"]]
        else:
            logits = _DistAggregate.apply(R["dg"], H1) @ W2
        loss = torch.nn.functional.cross_entropy(logits[R["lab_idx"]], R["lab_y"],
                                                 reduction="sum") / R["n_lab"]
        loss.backward()
        flat = torch.cat([p.grad.reshape(-1) for p in params])
        if world > 1:
            dist.all_reduce(flat)
        off = 0
        for p in params:
            p.grad.copy_(flat[off:off + p.numel()].view_as(p))
            off += p.numel()
        opt.step()
        lt = loss.detach().clone()
        if world > 1:
            dist.all_reduce(lt)
        return lt

    times, losses = [], []
    for e in range(start_epoch, cfg["epochs"]):
        # only this stream: a side-stream copy still running is waited for
        # inside the next epoch (and timed there), not between epochs
        torch.cuda.current_stream().synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        lt = epoch(stage_next=e + 1 < cfg["epochs"])
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
        losses.append(float(lt))
    if staged:
        side.synchronize()
    if cfg.get("save") and rank == 0:  # weights are identical on every rank
        torch.save({"W1": W1.detach(), "W2": W2.detach(), "opt": opt.state_dict(),
                    "epoch": cfg["epochs"], "config": {k: v for k, v in cfg.items()
                                                       if k not in ("save", "resume")}},
                   cfg["save"])
    t = torch.tensor(times or [0.0], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    nnz = torch.tensor([float(R["nnz"])], device=device, dtype=torch.float64)
    halo = torch.tensor([float(R["dg"].halo_rows)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(nnz)
        dist.all_reduce(halo)
    transport = R["dg"].transport
    dev_err = R["dg"].device_error()
    R["dg"].close()  # collective: every rank
    if dev_err:
        raise RuntimeError(f"halo exchange device error {dev_err}")
    return dict(transport=transport, cold_coop=getattr(R["store"], "stage_group", None) is not None,
                epoch_s=t.tolist(), losses=losses, nnz=float(nnz), halo_rows=float(halo),
                gen_s=R["gen_s"], conv_s=R["conv_s"], store_hot=R["store"].n_hot,
                store_cold=R["store"].n_cold, cold_staging=staged, transform_first=transform_first)


CONFIG4 = dict(nodes=2_449_029, edges=61_900_000, seed=3, F_in=100, hidden=256, classes=47,
               label_fraction=0.08, hot_fraction=0.2, dropout=0.5, lr=1e-2, epochs=10)


def config(shrink: int = 0) -> dict:
    c = dict(CONFIG4)
    c["nodes"] >>= shrink
    c["edges"] >>= shrink
    return c


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--shrink", type=int, default=0, help="divide nodes and edges by 2**shrink")
    p.add_argument("--epochs", type=int, default=10)
    order = p.add_mutually_exclusive_group()
    order.add_argument("--transform-first", dest="order", action="store_const", const="transform",
                       help="layer 2 as A.(H.W) (the default for these widths)")
    order.add_argument("--aggregate-first", dest="order", action="store_const", const="aggregate",
                       help="layer 2 as (A.H).W, the reference's order")
    p.add_argument("--cold-zero-copy", action="store_true",
                   help="read cold rows from pinned host memory in every gather (no HBM staging)")
    p.add_argument("--partition", choices=["tiles", "nnz"], default="tiles",
                   help="N > 1: cut the rows into parts of equal pull work (tiles) or equal "
                        "nonzeros")
    p.add_argument("--save", default=None, help="checkpoint path written at the end (rank 0)")
    p.add_argument("--resume", default=None, help="checkpoint to continue from")
    a = p.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                pg_options=nccl_options(), device_id=device)
    try:
        cfg = config(a.shrink)
        cfg["epochs"] = a.epochs
        cfg["save"], cfg["resume"] = a.save, a.resume
        cfg["cold_staging"] = not a.cold_zero_copy
        cfg["partition"] = a.partition
        tf = {"transform": True, "aggregate": False}.get(a.order)
        r = train(cfg, device, world, rank, tf)
        if rank == 0:
            steady = r["epoch_s"][1:] or r["epoch_s"]
            print(json.dumps({
                "metric": "GCN epoch time (2-layer, full graph)", "value": round(sum(steady) / len(steady), 5),
                "unit": "s/epoch", "n_gpus": world, "epochs": cfg["epochs"], "higher_is_better": False,
                "scaling": "strong", "loss_first": round(r["losses"][0], 5), "loss_last": round(r["losses"][-1], 5),
                "epoch_s": [round(x, 5) for x in r["epoch_s"]], "data": "synthetic (seeded R-MAT, GPU generator)",
                "config": {"workload": "config4", "nodes": cfg["nodes"], "nnz": int(r["nnz"]),
                           "F_in": cfg["F_in"], "hidden": cfg["hidden"], "classes": cfg["classes"],
                           "hot_rows": r["store_hot"], "cold_rows": r["store_cold"],
                           "cold_rows_path": (("pinned host -> HBM staging buffer once per epoch on "
                                               "a side stream (overlapped)" +
                                               ("; a chunk per rank over PCIe, then an NCCL "
                                                "all-gather" if r.get("cold_coop") else ""))
                                              if r["cold_staging"]
                                              else "zero-copy reads of pinned host memory"),
                           "halo_transport": r["transport"],
                           "partition": cfg["partition"] if world > 1 else None,
                           "halo_rows_total": int(r["halo_rows"]), "transform_first": r["transform_first"],
                           "order": "layer 1 from the hot/cold store, layer 2 over the row partition"}}),
                  flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
