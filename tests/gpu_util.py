"""Helpers shared by the GPU test modules."""
import numpy as np
import torch

from tcc_b200 import graphs as G

SWTCF_KEYS = ("colWindowOffset", "tileLocalBit", "tileRowSlot", "superWindowRowOffset",
              "superWindowRows", "superWindowRowCacheSlot", "superWindowCachedRowSlot",
              "superWindowCachedCount")


def u32(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).cuda()


def csr_dev(g):
    return (torch.from_numpy(g.rowptr.view(np.int64)).cuda(), u32(g.col))


def dense(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def rel_fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (nb if nb > 0 else 1.0)


def rel_inf(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.abs(b).max() if b.size else 0.0
    return (np.abs(a - b).max() if a.size else 0.0) / (nb if nb > 0 else 1.0)


def edge_case_graphs():
    """Small graphs covering the layout edge cases the reference validators test."""
    rng = np.random.default_rng(42)
    out = []
    out.append(("uniform-4096", G.config(1)["graph"]))
    out.append(("rmat-2^12", G.rmat(12, 16 << 12, seed=1)))
    out.append(("sbm-1456", G.sbm(1456, 50, 60000, 40.0, 1.2, seed=2)))
    out.append(("odd-1003", G.rmat(10, 4000, seed=5, n=1003)))
    # rectangular, rows < cols and rows > cols, ragged last window
    r = rng.integers(0, 301, 3000).astype(np.uint32)
    c = rng.integers(0, 703, 3000).astype(np.uint32)
    out.append(("rect-301x703", G.csr_from_pairs(r, c, 301, 703)))
    out.append(("rect-703x301", G.csr_from_pairs(c, r, 703, 301)))
    # one edge
    out.append(("single-edge", G.csr_from_pairs(np.array([5], np.uint32), np.array([9], np.uint32), 13, 17)))
    # fully dense 8x8 blocks (popcount 64 tiles) and a window with exactly 9 rows
    rows, cols = [], []
    for i in range(16):
        for j in range(16):
            rows.append(i)
            cols.append(j)
    for i in range(9):
        rows.append(40 + i)
        cols.append(3)
    out.append(("dense-blocks", G.csr_from_pairs(np.array(rows, np.uint32), np.array(cols, np.uint32), 64, 64)))
    # a star: node 0 adjacent to everyone (one very heavy row and column window)
    n = 5000
    u = np.zeros(n - 1, np.uint32)
    v = np.arange(1, n, dtype=np.uint32)
    star = G._symmetrise_with_loops(u, v, n)
    out.append(("star-5000", star))
    # isolated nodes: only a few edges in a big id space
    r = rng.integers(0, 20000, 300).astype(np.uint32)
    c = rng.integers(0, 20000, 300).astype(np.uint32)
    out.append(("sparse-20000", G.csr_from_pairs(r, c, 20000, 20000)))
    return out
