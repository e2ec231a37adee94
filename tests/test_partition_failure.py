"""Failure detection of the row-partitioned set-up on CPU ranks (gloo): a rank
that dies before the request-list exchange makes its peer's collective fail
with an error within the process-group timeout instead of hanging; the
failure is injected on the host (the rank exits), no GPU is involved."""
import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    from tcc_b200 import graphs as G
    from tcc_b200.partition import DistGraph, balanced_bounds
    rowptr, col, _ = G.rmat_gpu(10, 8 << 10, seed=3, device="cpu")
    bounds = balanced_bounds(torch.diff(rowptr), world)
    r0, r1 = bounds[rank], bounds[rank + 1]
    if rank == world - 1:
        q.put((rank, "died", 0.0))
        q.close()
        q.join_thread()  # flush before the hard exit
        os._exit(0)  # the injected failure: this rank never reaches the exchange
    t0 = time.time()
    try:
        DistGraph((rowptr[r0:r1 + 1] - rowptr[r0]).contiguous(), col[rowptr[r0]:rowptr[r1]],
                  bounds, build_tiles=False)
        q.put((rank, "no error", time.time() - t0))
    except Exception as e:  # the collective reports the dead peer
        q.put((rank, type(e).__name__, time.time() - t0))


def test_dead_rank_fails_peer_collective_with_error():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert res[1][1] == "died"
    rank0 = res[0]
    assert rank0[1] != "no error", rank0
    assert rank0[2] < 60, rank0
