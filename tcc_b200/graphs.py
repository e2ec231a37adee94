"""Seeded synthetic graphs and features with the shapes of the benchmark configs.

The reference ships no datasets (its drivers read user-supplied raw uint32
``dst_local.bin`` / ``src_local.bin`` files, src/swtcf_spmm_main.cu:17-31); these
generators stand in for the graphs the benchmark configurations describe:

* ``uniform``  -- undirected uniform random graph + self-loops (config 1)
* ``rmat``     -- R-MAT (a,b,c,d) edges, symmetrised, deduplicated, self-loops
                  (configs 2, 4, 5)
* ``sbm``      -- degree-corrected stochastic block model with log-normal
                  propensities (config 3)

Every graph is returned as a CSR over uint32 node ids with uint64 row pointers
and ascending, duplicate-free columns.  Generation is numpy (PCG64) and fully
determined by the seed.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np


@dataclasses.dataclass
class Csr:
    rows: int
    cols: int
    rowptr: np.ndarray  # uint64 [rows+1]
    col: np.ndarray     # uint32 [nnz], ascending within each row

    @property
    def nnz(self) -> int:
        return int(self.rowptr[-1])

    def degrees(self) -> np.ndarray:
        return np.diff(self.rowptr).astype(np.int64)

    def coo(self):
        """(dst, src) uint32 arrays: dst = row, src = column."""
        dst = np.repeat(np.arange(self.rows, dtype=np.uint32), self.degrees())
        return dst, self.col

    def transpose(self) -> "Csr":
        dst, src = self.coo()
        return csr_from_pairs(src, dst, self.cols, self.rows)


def csr_from_pairs(rows_idx: np.ndarray, cols_idx: np.ndarray, n_rows: int, n_cols: int,
                   dedup: bool = True) -> Csr:
    """CSR with ascending columns from (row, col) pairs; duplicates removed."""
    keys = (rows_idx.astype(np.uint64) << np.uint64(32)) | cols_idx.astype(np.uint64)
    keys.sort()  # np.unique is far slower than sort + mask on this numpy
    if dedup and keys.size:
        first = np.empty(keys.size, dtype=bool)
        first[0] = True
        np.not_equal(keys[1:], keys[:-1], out=first[1:])
        keys = keys[first]
    r = (keys >> np.uint64(32)).astype(np.int64)
    c = (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    counts = np.bincount(r, minlength=n_rows)
    rowptr = np.zeros(n_rows + 1, dtype=np.uint64)
    np.cumsum(counts, out=rowptr[1:])
    return Csr(n_rows, n_cols, rowptr, c)


def _symmetrise_with_loops(u: np.ndarray, v: np.ndarray, n: int) -> Csr:
    loops = np.arange(n, dtype=np.uint32)
    rows = np.concatenate([u, v, loops])
    cols = np.concatenate([v, u, loops])
    return csr_from_pairs(rows, cols, n, n)


def uniform(n: int, avg_degree: float, seed: int) -> Csr:
    """Undirected uniform random graph with ~avg_degree neighbours + self-loops."""
    rng = np.random.Generator(np.random.PCG64(seed))
    m = int(round(n * avg_degree / 2))
    u = rng.integers(0, n, size=m, dtype=np.uint32)
    v = rng.integers(0, n, size=m, dtype=np.uint32)
    keep = u != v
    return _symmetrise_with_loops(u[keep], v[keep], n)


def rmat_edges(scale: int, m: int, abcd=(0.57, 0.19, 0.19, 0.05), seed: int = 0,
               chunk: int = 1 << 22):
    """m directed R-MAT edges on 2**scale nodes (no noise, no relabelling)."""
    a, b, c, _ = abcd
    rng = np.random.Generator(np.random.PCG64(seed))
    us, vs = [], []
    t1, t2, t3 = np.float32(a), np.float32(a + b), np.float32(a + b + c)
    for start in range(0, m, chunk):
        k = min(chunk, m - start)
        u = np.zeros(k, dtype=np.uint32)
        v = np.zeros(k, dtype=np.uint32)
        for level in range(scale):
            r = rng.random(k, dtype=np.float32)
            rb = r >= t2
            cb = ((r >= t1) & (r < t2)) | (r >= t3)
            bit = np.uint32(1 << (scale - 1 - level))
            u |= rb.astype(np.uint32) * bit
            v |= cb.astype(np.uint32) * bit
        us.append(u)
        vs.append(v)
    return np.concatenate(us), np.concatenate(vs)


def rmat(scale: int, edges: int, seed: int, abcd=(0.57, 0.19, 0.19, 0.05),
         n: int | None = None) -> Csr:
    """R-MAT graph: `edges` directed edges, symmetrised, deduplicated, self-loops.

    With ``n`` smaller than 2**scale, edges touching a node >= n are dropped and
    regenerated until `edges` directed edges remain (config 4's 2,449,029 nodes).
    """
    nodes = (1 << scale) if n is None else n
    if n is None:
        u, v = rmat_edges(scale, edges, abcd, seed)
    else:
        us, vs, have, round_ = [], [], 0, 0
        while have < edges:
            need = int((edges - have) * 1.25) + 1024
            u, v = rmat_edges(scale, need, abcd, seed * 1009 + round_)
            keep = (u < n) & (v < n)
            us.append(u[keep])
            vs.append(v[keep])
            have += int(keep.sum())
            round_ += 1
        u = np.concatenate(us)[:edges]
        v = np.concatenate(vs)[:edges]
    keep = u != v
    return _symmetrise_with_loops(u[keep], v[keep], nodes)


def sbm(n: int, blocks: int, total_edges: int, ratio: float, sigma: float, seed: int) -> Csr:
    """Degree-corrected SBM: contiguous equal blocks, per-pair intra/inter edge
    probability ratio `ratio`, log-normal(sigma) propensities; ~total_edges
    edges after symmetrisation (self-loops added on top)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    block = (np.arange(n, dtype=np.int64) * blocks) // n
    sizes = np.bincount(block, minlength=blocks).astype(np.float64)
    starts = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    prop = rng.lognormal(0.0, sigma, size=n)
    share = float(np.sum((sizes / n) ** 2))
    p_intra = ratio * share / (ratio * share + (1.0 - share))
    m = total_edges // 2
    cdf = np.cumsum(prop)
    cdf /= cdf[-1]
    u = np.searchsorted(cdf, rng.random(m)).astype(np.int64)
    u = np.minimum(u, n - 1)
    intra = rng.random(m) < p_intra
    v = np.searchsorted(cdf, rng.random(m)).astype(np.int64)
    # intra edges: redraw v from u's block by propensity
    bu = block[u[intra]]
    lo, hi = starts[bu], starts[bu + 1]
    clo = np.where(lo > 0, cdf[np.maximum(lo - 1, 0)], 0.0)
    chi = cdf[hi - 1]
    r = clo + rng.random(bu.size) * (chi - clo)
    vi = np.searchsorted(cdf, r).astype(np.int64)
    v[intra] = np.clip(vi, lo, hi - 1)
    v = np.minimum(v, n - 1)
    keep = u != v
    return _symmetrise_with_loops(u[keep].astype(np.uint32), v[keep].astype(np.uint32), n)


# ------------------------------------------------------------ value scales --

def gcn_scales(g: Csr):
    """D^-1/2 (A+I) D^-1/2 as (row_scale, col_scale); self-loops are in g."""
    d = g.degrees().astype(np.float64)
    s = np.where(d > 0, 1.0 / np.sqrt(np.maximum(d, 1.0)), 0.0).astype(np.float32)
    return s, s.copy()


def row_scales(g: Csr):
    """1/deg(row) (row-normalised, D^-1 A) as (row_scale, None)."""
    d = g.degrees().astype(np.float64)
    return np.where(d > 0, 1.0 / np.maximum(d, 1.0), 0.0).astype(np.float32), None


def features(n: int, f: int, seed: int, dist: str = "normal") -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed + 7919))
    if dist == "normal":
        return rng.standard_normal((n, f), dtype=np.float32)
    if dist == "uniform":
        return rng.uniform(-1.0, 1.0, size=(n, f)).astype(np.float32)
    raise ValueError(dist)


# ----------------------------------------------------------------- configs --

def config(idx: int, shrink: int = 0):
    """The five benchmark workloads as dicts (graph, scales, F, feature dist).

    ``shrink`` divides node and edge counts by 2**shrink for test-sized runs.
    """
    if idx == 1:
        g = uniform(4096 >> shrink, 16, seed=0)
        rs, cs = row_scales(g)
        return dict(name="uniform-4096", graph=g, rs=rs, cs=cs, F=64, dist="uniform", seed=0)
    if idx == 2:
        sc = 20 - shrink
        g = rmat(sc, 16 << sc, seed=1)
        rs, cs = gcn_scales(g)
        return dict(name=f"rmat-2^{sc}", graph=g, rs=rs, cs=cs, F=128, dist="normal", seed=1)
    if idx == 3:
        n = 232965 >> shrink
        g = sbm(n, 50, 114_600_000 >> shrink, 40.0, 1.2, seed=2)
        rs, cs = gcn_scales(g)
        return dict(name=f"sbm-{n}", graph=g, rs=rs, cs=cs, F=256, dist="uniform", seed=2)
    if idx == 4:
        n = 2_449_029 >> shrink
        sc = max(1, math.ceil(math.log2(n)))
        g = rmat(sc, 61_900_000 >> shrink, seed=3, n=n)
        rs, cs = gcn_scales(g)
        return dict(name=f"rmat-{n}", graph=g, rs=rs, cs=cs, F=100, dist="normal", seed=3)
    if idx == 5:
        sc = 26 - shrink
        g = rmat(sc, 16 << sc, seed=4)
        rs, cs = row_scales(g)
        return dict(name=f"rmat-2^{sc}", graph=g, rs=rs, cs=cs, F=128, dist="normal", seed=4)
    raise ValueError(idx)


# --------------------------------------------------- GPU (torch) generator --

def _rmat_gpu_edges(scale, edges, seed, device, abcd, chunk, n):
    """Yields the (u, v) int64 edge chunks of rmat_gpu (self-edges removed)."""
    import torch
    a, b, c, _ = abcd
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    have = 0
    while have < edges:
        k = min(chunk, edges - have) if n == 1 << scale else chunk
        u = torch.zeros(k, dtype=torch.int64, device=device)
        v = torch.zeros(k, dtype=torch.int64, device=device)
        for level in range(scale):
            r = torch.rand(k, generator=gen, device=device)
            bit = 1 << (scale - 1 - level)
            u += (r >= a + b).to(torch.int64) * bit
            v += (((r >= a) & (r < a + b)) | (r >= a + b + c)).to(torch.int64) * bit
        if n != 1 << scale:
            inside = (u < n) & (v < n)
            u, v = u[inside], v[inside]
            take = min(u.numel(), edges - have)
            u, v = u[:take], v[:take]
        have += u.numel()
        keep = u != v
        yield u[keep], v[keep]


def rmat_gpu_degrees(scale: int, edges: int, seed: int, device, abcd=(0.57, 0.19, 0.19, 0.05),
                     chunk: int = 1 << 26, n: int | None = None, symmetric: bool = True,
                     loops: bool = True):
    """Row nonzero counts of rmat_gpu's matrix before deduplication, without
    materialising it (partition bounds for a job whose ranks build only their
    rows)."""
    import torch
    n = (1 << scale) if n is None else n
    deg = torch.full((n,), 1 if loops else 0, dtype=torch.int64, device=device)
    for u, v in _rmat_gpu_edges(scale, edges, seed, device, abcd, chunk, n):
        deg += torch.bincount(u, minlength=n)
        if symmetric:
            deg += torch.bincount(v, minlength=n)
    return deg


def rmat_gpu(scale: int, edges: int, seed: int, device, row_range=None,
             abcd=(0.57, 0.19, 0.19, 0.05), chunk: int = 1 << 26, n: int | None = None,
             symmetric: bool = True, loops: bool = True):
    """R-MAT on the GPU with torch's seeded generator: ``edges`` directed edges on
    2**scale nodes, symmetrised (unless ``symmetric`` is False), deduplicated,
    self-loops added (unless ``loops`` is False).

    With ``n`` < 2**scale nodes, edges touching a node >= n are dropped and more
    are drawn until ``edges`` directed edges (before removing self-edges) remain
    (config 4's 2,449,029 nodes).  Every caller with the same arguments draws
    the same edges, so each rank of a multi-GPU job can build just its rows:
    ``row_range = (r0, r1)`` keeps rows r0 <= r < r1.  Returns (rowptr int64
    [r1-r0+1], col int32 [nnz] global column ids, degrees int64 [n]: row
    nonzero counts before deduplication, used for balancing partitions).
    """
    import torch
    n = (1 << scale) if n is None else n
    r0, r1 = (0, n) if row_range is None else row_range
    keys = []
    deg = torch.full((n,), 1 if loops else 0, dtype=torch.int64, device=device)
    for u, v in _rmat_gpu_edges(scale, edges, seed, device, abcd, chunk, n):
        deg += torch.bincount(u, minlength=n)
        if symmetric:
            deg += torch.bincount(v, minlength=n)
        for x, y in (((u, v), (v, u)) if symmetric else ((u, v),)):
            m = (x >= r0) & (x < r1)
            keys.append(((x[m] - r0) << 32) | y[m])
    if loops:
        diag = torch.arange(r0, r1, dtype=torch.int64, device=device)
        keys.append(((diag - r0) << 32) | diag)
    keys = torch.unique(torch.cat(keys))  # sorted, deduplicated
    rows = (keys >> 32)
    col = (keys & 0xFFFFFFFF).to(torch.int32)
    counts = torch.bincount(rows, minlength=r1 - r0)
    rowptr = torch.zeros(r1 - r0 + 1, dtype=torch.int64, device=device)
    rowptr[1:] = torch.cumsum(counts, 0)
    return rowptr, col, deg


def sbm_gpu(n: int, blocks: int, total_edges: int, ratio: float, sigma: float, seed: int,
            device, chunk: int = 1 << 25):
    """``sbm`` on the GPU with torch's seeded generator (config 3 at full size in
    seconds): degree-corrected SBM over contiguous equal blocks, intra/inter
    pair-probability ratio ``ratio``, log-normal(sigma) propensities,
    ~total_edges edges after symmetrisation, deduplicated, self-loops added.
    Returns (rowptr int64 [n+1], col int32 [nnz])."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    block = (torch.arange(n, dtype=torch.int64, device=device) * blocks) // n
    sizes = torch.bincount(block, minlength=blocks).to(torch.float64)
    starts = torch.zeros(blocks + 1, dtype=torch.int64, device=device)
    starts[1:] = torch.cumsum(sizes, 0).to(torch.int64)
    prop = torch.exp(sigma * torch.randn(n, generator=gen, device=device, dtype=torch.float64))
    share = float(torch.sum((sizes / n) ** 2))
    p_intra = ratio * share / (ratio * share + (1.0 - share))
    cdf = torch.cumsum(prop, 0)
    cdf /= cdf[-1].clone()
    m = total_edges // 2
    keys = []
    for s0 in range(0, m, chunk):
        k = min(chunk, m - s0)
        u = torch.searchsorted(cdf, torch.rand(k, generator=gen, device=device, dtype=torch.float64))
        u = u.clamp_(max=n - 1)
        intra = torch.rand(k, generator=gen, device=device) < p_intra
        v = torch.searchsorted(cdf, torch.rand(k, generator=gen, device=device, dtype=torch.float64))
        bu = block[u[intra]]
        lo, hi = starts[bu], starts[bu + 1]
        clo = torch.where(lo > 0, cdf[(lo - 1).clamp(min=0)], torch.zeros_like(lo, dtype=torch.float64))
        chi = cdf[hi - 1]
        r = clo + torch.rand(bu.numel(), generator=gen, device=device, dtype=torch.float64) * (chi - clo)
        vi = torch.searchsorted(cdf, r)
        v[intra] = torch.minimum(torch.maximum(vi, lo), hi - 1)
        v = v.clamp_(max=n - 1)
        keep = u != v
        u, v = u[keep], v[keep]
        keys.append((u << 32) | v)
        keys.append((v << 32) | u)
    diag = torch.arange(n, dtype=torch.int64, device=device)
    keys.append((diag << 32) | diag)
    keys = torch.unique(torch.cat(keys))
    rows = keys >> 32
    col = (keys & 0xFFFFFFFF).to(torch.int32)
    counts = torch.bincount(rows, minlength=n)
    rowptr = torch.zeros(n + 1, dtype=torch.int64, device=device)
    rowptr[1:] = torch.cumsum(counts, 0)
    return rowptr, col
