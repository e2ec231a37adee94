"""Row partition + halo exchange on CPU ranks (gloo, world size 2 and 3).

The distributed SpMM's index plumbing -- nnz-balanced bounds, compacted halo,
per-peer request lists, remapped local / halo CSRs, the all-to-all exchange --
is checked by emulating the tile SpMM with a CSR SpMM on each rank and
comparing every rank's rows with the single-process result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _csr_mm(rowptr, col, X, n_rows):
    Y = np.zeros((n_rows, X.shape[1]), np.float64)
    rp = rowptr.numpy()
    c = col.numpy().astype(np.int64)
    for r in range(n_rows):
        if rp[r + 1] > rp[r]:
            Y[r] = X[c[rp[r]:rp[r + 1]]].sum(0)
    return Y


def _worker(rank, world, port, scale, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tcc_b200 import graphs as G
        from tcc_b200.partition import DistGraph, balanced_bounds
        rowptr, col, _ = G.rmat_gpu(scale, 8 << scale, seed=5, device="cpu")
        deg = torch.diff(rowptr)
        bounds = balanced_bounds(deg, world)
        r0, r1 = bounds[rank], bounds[rank + 1]
        lrp = rowptr[r0:r1 + 1] - rowptr[r0]
        lcol = col[rowptr[r0]:rowptr[r1]]
        dg = DistGraph(lrp, lcol, bounds, build_tiles=False)
        rng = np.random.default_rng(1)
        X = rng.standard_normal((deg.numel(), 8)).astype(np.float32)
        Xl = torch.from_numpy(X[r0:r1].copy())
        halo, work = dg.exchange(Xl, async_op=True)
        if work is not None:
            work.wait()
        # the halo holds exactly X[halo ids]
        assert np.array_equal(halo.numpy(), X[dg.halo.numpy()])
        Y = _csr_mm(dg.loc_rowptr, dg.loc_col, Xl.numpy(), dg.n_local) + \
            _csr_mm(dg.halo_rowptr, dg.halo_col, halo.numpy(), dg.n_local)
        Yg = _csr_mm(rowptr[r0:r1 + 1] - rowptr[r0], col[rowptr[r0]:rowptr[r1]], X, r1 - r0)
        err = float(np.abs(Y - Yg).max())
        out_q.put((rank, err, dg.halo_rows, dg.nnz, sum(dg.send_counts)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_partition_halo_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 11, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err, halo, nnz, sent in res:
        assert err < 1e-4, (rank, err)
        assert halo > 0 and nnz > 0
    # every halo row received was sent by some peer
    assert sum(r[2] for r in res) == sum(r[4] for r in res)
    # nnz balance within 10 %
    nnzs = [r[3] for r in res]
    assert max(nnzs) <= 1.1 * min(nnzs) + 64


def test_balanced_bounds():
    from tcc_b200.partition import balanced_bounds
    deg = torch.tensor([100, 1, 1, 1, 1, 50, 50, 1, 1, 1])
    b = balanced_bounds(deg, 2)
    assert b[0] == 0 and b[-1] == 10 and 0 < b[1] < 10
    assert balanced_bounds(deg, 1) == [0, 10]


def test_tile_balanced_bounds():
    """Row bounds on window boundaries with about equal tiles + per-window work."""
    import torch
    from tcc_b200.partition import tile_balanced_bounds
    gen = torch.Generator().manual_seed(0)
    n = 8 * 1000 + 5
    W = (n + 7) // 8
    per = torch.randint(0, 40, (W,), generator=gen)
    per[:10] = 5000  # hub windows at the front
    off = torch.zeros(W + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(per, 0)
    for parts in (2, 3, 8):
        b = tile_balanced_bounds(off, n, parts)
        assert b[0] == 0 and b[-1] == n and len(b) == parts + 1
        assert all(x < y for x, y in zip(b, b[1:]))
        assert all(x % 8 == 0 for x in b[1:-1])
        cost = [float(per[b[k] // 8:(b[k + 1] + 7) // 8].sum()) + 2.0 * ((b[k + 1] - b[k] + 7) // 8)
                for k in range(parts)]
        # every part within one heavy window of the ideal share
        assert max(cost) <= sum(cost) / parts + 5000 + 50


def test_push_sms_splits_the_sms_by_work():
    """The peer push's SM share follows the ratio of its SM-time to the local
    tiles' SM-time, within [16, sms - 16]."""
    from tcc_b200.partition import push_sms
    # 2 GPUs, config 2: heavy local work beside a modest send (~30 of 148)
    assert 20 <= push_sms(410_000, 870_000, 148) <= 40
    # little to send: the floor of 16
    assert push_sms(1000, 1_000_000, 148) == 16
    # a rank whose local work is small beside its send gets more SMs, up to the cap
    assert 40 <= push_sms(300_000, 400_000, 148) < 64
    assert push_sms(500_000, 230_000, 148) == 64
    assert push_sms(10_000_000, 1, 148) == 64
    assert push_sms(10_000_000, 1, 60) == 44  # and leaves 16 SMs to the tiles


def test_exchange_window_cost_by_rank_count():
    """Tiles alone on 2 ranks, tiles plus the rows' sending from 4 on; a larger
    per-window cost moves rows off the tail part."""
    import torch
    from tcc_b200.partition import exchange_window_cost, tile_balanced_bounds
    assert exchange_window_cost(2) == 2.0 and exchange_window_cost(4) == 10.0
    assert exchange_window_cost(8) == 10.0
    # hub windows hold many tiles, tail windows one: the tail part shrinks as
    # the per-window cost grows
    tiles = torch.tensor([40] * 100 + [1] * 3900, dtype=torch.int64)
    off = torch.zeros(tiles.numel() + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(tiles, 0)
    n = 8 * tiles.numel()
    b2 = tile_balanced_bounds(off, n, 4, window_cost=2.0)
    b10 = tile_balanced_bounds(off, n, 4, window_cost=10.0)
    assert b2[0] == 0 and b2[-1] == n and b10[-1] == n
    assert n - b10[3] < n - b2[3]
