"""Row-partitioned SpMM across GPUs: every rank's rows equal the single-GPU
result -- the forward pass, the pipelined pair the bench times (several steps,
new operands each, so a halo buffer is reused only after its readers released
it), and the transposed pass of a directed graph (partial rows returned to
their owners) -- with the halo moved by the peer-memory transport (steps
sequenced by the library's tcc_dist_step, and call by call from Python) and
by NCCL.
Spawns one process per visible GPU (2 or more); skipped otherwise."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, transport, q):
    transport, _, host_step = transport.partition("-")
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    from tcc_b200.partition import nccl_options
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), pg_options=nccl_options(),
                            device_id=torch.device("cuda", rank))
    try:
        from tcc_b200 import graphs as G
        from tcc_b200 import tiles
        from tcc_b200.partition import DistGraph, balanced_bounds
        dev = torch.device("cuda", rank)
        rowptr, col, _ = G.rmat_gpu(15, 16 << 15, seed=9, device=dev)
        deg = torch.diff(rowptr)
        s = deg.to(torch.float32).clamp(min=1).rsqrt()
        bounds = balanced_bounds(deg, world)
        r0, r1 = bounds[rank], bounds[rank + 1]
        dg = DistGraph((rowptr[r0:r1 + 1] - rowptr[r0]).contiguous(),
                       col[rowptr[r0]:rowptr[r1]].contiguous(), bounds,
                       rs_local=s[r0:r1].contiguous(), cs_global=s, tc_threshold=65,
                       transport=transport)
        assert dg.transport == transport
        if host_step:
            dg.host_step = host_step
        gen = torch.Generator(device=dev)
        gen.manual_seed(3)
        X = torch.randn((deg.numel(), 64), generator=gen, device=dev)  # same X on every rank
        Y = dg.spmm(X[r0:r1].contiguous())
        full = tiles.from_csr(rowptr, col, deg.numel(), deg.numel(), kind="bcsr")
        Yref = tiles.bcsr_spmm(full, X, tc_threshold=65, rs=s, cs=s)[r0:r1]
        err = (torch.linalg.norm(Y - Yref) / torch.linalg.norm(Yref)).item()
        # the pipelined pair of the bench's step (A symmetric: Z = A[P_g, :] G),
        # four steps back to back with new operands, checked after each
        Gm = torch.randn((deg.numel(), 64), generator=gen, device=dev)
        Zref = tiles.bcsr_spmm(full, Gm, tc_threshold=65, rs=s, cs=s)[r0:r1]
        Y2, Z2 = torch.empty_like(Y), torch.empty_like(Y)
        for step in range(4):
            a, b = float(step + 1), float(1 - 2 * (step & 1))
            dg.spmm_pair((a * X[r0:r1]).contiguous(), Y2, (b * Gm[r0:r1]).contiguous(), Z2)
            err = max(err, (torch.linalg.norm(Y2 - a * Yref) / torch.linalg.norm(a * Yref)).item(),
                      (torch.linalg.norm(Z2 - b * Zref) / torch.linalg.norm(Zref)).item())
        assert dg.device_error() == 0
        # a directed graph: the transposed pass returns partial rows to owners
        drp, dcol, _ = G.rmat_gpu(15, 16 << 15, seed=10, device=dev, symmetric=False,
                                  loops=False)
        ddeg = torch.diff(drp)
        rsd = torch.where(ddeg > 0, 1.0 / ddeg.clamp(min=1).to(torch.float32),
                          torch.zeros_like(ddeg, dtype=torch.float32))
        db = balanced_bounds(ddeg, world)
        a0, a1 = db[rank], db[rank + 1]
        ddg = DistGraph((drp[a0:a1 + 1] - drp[a0]).contiguous(),
                        dcol[drp[a0]:drp[a1]].contiguous(), db, rs_local=rsd[a0:a1].contiguous(),
                        cs_global=None, tc_threshold=65, transport=transport)
        if host_step:
            ddg.host_step = host_step
        Zd = ddg.spmm_t(Gm[a0:a1].contiguous())
        dfull = tiles.from_csr(drp, dcol, ddeg.numel(), ddeg.numel(), kind="bcsc")
        Zdref = tiles.bcsc_spmm_t(dfull, Gm, tc_threshold=65, rs=rsd)[a0:a1]
        err = max(err, (torch.linalg.norm(Zd - Zdref) / torch.linalg.norm(Zdref)).item())
        Yd = ddg.spmm(X[a0:a1].contiguous())
        dfull_r = tiles.from_csr(drp, dcol, ddeg.numel(), ddeg.numel(), kind="bcsr")
        Ydref = tiles.bcsr_spmm(dfull_r, X, tc_threshold=65, rs=rsd)[a0:a1]
        err = max(err, (torch.linalg.norm(Yd - Ydref) / torch.linalg.norm(Ydref)).item())
        torch.cuda.synchronize()
        assert ddg.device_error() == 0
        dg.close()
        ddg.close()
        q.put((rank, err, dg.halo_rows))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
@pytest.mark.parametrize("transport", ["peer-native", "peer-python", "nccl"])
def test_row_partitioned_spmm_matches_single_gpu(gpu, transport):
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, transport, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err, halo in res:
        assert err <= FP32_TOL, (rank, err)
        assert halo > 0


def _gcn_worker(rank, world, port, cfg, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    from tcc_b200.partition import nccl_options
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), pg_options=nccl_options(),
                            device_id=torch.device("cuda", rank))
    try:
        from tcc_b200 import train_gcn
        r = train_gcn.train(cfg, torch.device("cuda", rank), world, rank)
        torch.cuda.synchronize()
        if rank == 0:
            q.put((r["losses"], r["cold_staging"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_gcn_training_across_gpus_matches_one_gpu(gpu):
    """The row-partitioned GCN trainer (layer-2 halo exchange, gradient
    all-reduce, cold rows staged cooperatively: each rank copies a chunk of the
    cold block over PCIe and an all-gather assembles the rest) follows the
    one-GPU loss trajectory (dropout off, so only summation order differs)."""
    from tcc_b200 import train_gcn
    cfg = train_gcn.config(shrink=5)
    cfg["dropout"] = 0.0
    cfg["epochs"] = 4
    one = train_gcn.train(dict(cfg), torch.device("cuda", 0), 1, 0)["losses"]
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gcn_worker, args=(r, world, port, dict(cfg), q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    losses, staged = q.get(timeout=10)
    assert staged
    assert max(abs(a - b) / b for a, b in zip(losses, one)) < 1e-3, (losses, one)
