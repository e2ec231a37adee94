"""Mini-batch inputs of the reference's training step: raw-binary COO files,
sampled blocks, and the BCSR/BCSC tile sets CNICSPMMFunction consumes.

The reference reads a graph as two raw uint32 files, dst_local.bin and
src_local.bin (src/swtcf_spmm_main.cu:17-31, 128-142; rows = max(dst) + 1,
cols = max(src) + 1), and trains on mini-batches whose sampled blocks, BCSR /
BCSC tilings and feature maps come from its Legion sampler (``ipc_service``,
train/tcgnn_conv_release.py:282-301, absent from the reference tree).  This
module provides those inputs from a CSR on the GPU:

* ``read_coo_bin`` / ``write_coo_bin`` -- the file format, same checks;
* ``sample_blocks`` -- uniform neighbour sampling without replacement
  (per-layer fanouts), blocks ordered input layer first, each block's source
  nodes starting with its destination nodes (the DGL/Legion block convention);
* ``block_tiles`` -- one block as a BCSR part, a BCSC part, or both: the
  "degree" split sends edges whose source has at least ``hub_degree`` edges
  in the block through the BCSC push pass and the rest through the BCSR pull
  pass (the two parts the reference's mixed op adds into one output);
* ``sparse_inputs`` -- SparseMatrixSize / SparseMatrixData / CooData for a
  two-layer model (``s_*`` = first block, ``f_*`` = last block), plus the
  batch's hot/cold feature maps (``batch_feature_maps``).
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np
import torch

from . import gcn
from . import tiles as T


# ------------------------------------------------------------- files --

def read_coo_bin(dst_path: str, src_path: str):
    """(dst, src, rows, cols) from two raw uint32 files (native byte order)."""
    arrays = []
    for p in (dst_path, src_path):
        size = os.path.getsize(p)
        if size % 4:
            raise ValueError(f"invalid file size: {p}")
        arrays.append(np.fromfile(p, dtype=np.uint32))
    dst, src = arrays
    if dst.size == 0 or dst.size != src.size:
        raise ValueError("invalid COO")
    return dst, src, int(dst.max()) + 1, int(src.max()) + 1


def write_coo_bin(dst_path: str, src_path: str, dst, src) -> None:
    np.ascontiguousarray(dst, dtype=np.uint32).tofile(dst_path)
    np.ascontiguousarray(src, dtype=np.uint32).tofile(src_path)


def swtcf_from_coo_bin(dst_path: str, src_path: str, S: int = 16):
    """Read the files and convert on the GPU (convertCOOToSWTCF); returns the
    SWTCFMatrix and the workspace (its device error word holds codes 1/4/5)."""
    from . import swtcf
    dst, src, rows, cols = read_coo_bin(dst_path, src_path)
    m = swtcf.SWTCFMatrix(rows, cols, dst.size, S)
    ws = swtcf.SWTCFConvertWorkspace(dst.size, cols, S)
    d = torch.from_numpy(dst.view(np.int32)).cuda()
    s = torch.from_numpy(src.view(np.int32)).cuda()
    swtcf.convert_coo(d, s, m, ws)
    return m, ws


# ------------------------------------------------------------ blocks --

@dataclasses.dataclass
class Block:
    """Edges dst_local <- src_local of one layer; src_ids[:num_dst] == dst_ids."""
    dst_ids: torch.Tensor   # int64 [num_dst] global ids
    src_ids: torch.Tensor   # int64 [num_src] global ids
    edge_dst: torch.Tensor  # int64 [E] local destination index
    edge_src: torch.Tensor  # int64 [E] local source index

    @property
    def num_dst(self) -> int:
        return int(self.dst_ids.numel())

    @property
    def num_src(self) -> int:
        return int(self.src_ids.numel())


def _sample_layer(rowptr, col, dst_ids, fanout, gen):
    dev = dst_ids.device
    starts = rowptr[dst_ids]
    deg = rowptr[dst_ids + 1] - starts
    owner = torch.repeat_interleave(torch.arange(dst_ids.numel(), device=dev), deg)
    pos = torch.arange(owner.numel(), device=dev) - torch.repeat_interleave(
        torch.cumsum(deg, 0) - deg, deg)
    nbr = col[(starts[owner] + pos)].to(torch.int64)
    if fanout >= 0:
        # random rank inside each destination's neighbour list; keep the first fanout
        key = torch.rand(owner.numel(), generator=gen, device=dev)
        order = torch.argsort(owner.to(torch.float64) * 2.0 + key.to(torch.float64))
        owner, nbr = owner[order], nbr[order]
        first = torch.cumsum(deg, 0) - deg
        rank = torch.arange(owner.numel(), device=dev) - torch.repeat_interleave(first, deg)
        keep = rank < fanout
        owner, nbr = owner[keep], nbr[keep]
    # sources: the destinations first, then the other sampled nodes ascending
    extra = torch.unique(nbr)
    extra = extra[~torch.isin(extra, dst_ids)]
    src_ids = torch.cat([dst_ids, extra])
    lookup_keys, lookup_pos = torch.sort(src_ids)
    src_local = lookup_pos[torch.searchsorted(lookup_keys, nbr)]
    return Block(dst_ids, src_ids, owner, src_local)


def sample_blocks(rowptr: torch.Tensor, col: torch.Tensor, seeds: torch.Tensor, fanouts,
                  generator: torch.Generator | None = None) -> list:
    """Blocks of a len(fanouts)-layer model for the seed nodes, input layer
    first.  fanouts[-1] is sampled around the seeds; -1 takes every neighbour."""
    seeds = seeds.to(torch.int64)
    blocks = []
    dst = seeds
    for f in reversed(list(fanouts)):
        b = _sample_layer(rowptr, col, dst, int(f), generator)
        blocks.append(b)
        dst = b.src_ids
    return blocks[::-1]


def _csr(rows: torch.Tensor, cols: torch.Tensor, n_rows: int):
    order = torch.argsort(rows * (1 << 32) + cols)
    rows, cols = rows[order], cols[order]
    rowptr = torch.zeros(n_rows + 1, dtype=torch.int64, device=rows.device)
    rowptr[1:] = torch.cumsum(torch.bincount(rows, minlength=n_rows), 0)
    return rowptr, cols.to(torch.int32)


def block_tiles(block: Block, split: str = "bcsr", hub_degree: int = 32):
    """(bcsr Tiles or None, bcsc Tiles or None) of the block's num_dst x num_src
    matrix; split = "bcsr" | "bcsc" | "degree"."""
    nd, ns = block.num_dst, block.num_src
    if split == "bcsr":
        push = torch.zeros(block.edge_src.numel(), dtype=torch.bool, device=block.edge_src.device)
    elif split == "bcsc":
        push = torch.ones(block.edge_src.numel(), dtype=torch.bool, device=block.edge_src.device)
    elif split == "degree":
        out_deg = torch.bincount(block.edge_src, minlength=ns)
        push = out_deg[block.edge_src] >= hub_degree
    else:
        raise ValueError(split)
    parts = []
    for kind, mask in (("bcsr", ~push), ("bcsc", push)):
        if not bool(mask.any()):
            parts.append(None)
            continue
        rp, c = _csr(block.edge_dst[mask], block.edge_src[mask], nd)
        parts.append(T.from_csr(rp, c, nd, ns, kind=kind))
    return tuple(parts)


def _empty_part(kind: str, nd: int, ns: int, device):
    W = (nd + 7) // 8 if kind == "bcsr" else (ns + 7) // 8
    z = torch.zeros(W + 1, dtype=torch.int32, device=device)
    return T.Tiles(kind, nd, ns, 0, 0, W, z, torch.zeros(1, dtype=torch.int32, device=device),
                   torch.full((1,), -1, dtype=torch.int32, device=device),
                   torch.zeros(1, dtype=torch.int64, device=device))


def _fields(t: T.Tiles):
    return (t.num_rows, t.num_cols, t.nnz, t.num_TCBlocks, t.num_windows), \
        (t.windowOffset, t.tcOffset, t.sparseIdx, t.tcLocalBit,
         torch.ones(max(t.nnz, 1), dtype=torch.float32, device=t.windowOffset.device))


def sparse_inputs(blocks: list, split: str = "bcsr", hub_degree: int = 32):
    """SparseMatrixSize, SparseMatrixData, CooData of a two-layer model (the
    namedtuples of train/tcgnn_conv_release.py:282-297); s_* describe the first
    (input) block, f_* the last one."""
    if len(blocks) != 2:
        raise ValueError("the reference model has two layers")
    sizes, datas = {}, {}
    for prefix, b in (("s", blocks[0]), ("f", blocks[1])):
        bcsr, bcsc = block_tiles(b, split, hub_degree)
        dev = b.edge_src.device
        bcsr = bcsr or _empty_part("bcsr", b.num_dst, b.num_src, dev)
        bcsc = bcsc or _empty_part("bcsc", b.num_dst, b.num_src, dev)
        for kind, t in (("bcsr", bcsr), ("bcsc", bcsc)):
            (nr, nc, nnz, nt, nw), (wo, tco, idx, bits, vals) = _fields(t)
            win = "rowWindows" if kind == "bcsr" else "colWindows"
            sizes.update({f"{prefix}_{kind}_num_rows": nr, f"{prefix}_{kind}_num_cols": nc,
                          f"{prefix}_{kind}_nnz": nnz, f"{prefix}_{kind}_num_TCBlocks": nt,
                          f"{prefix}_{kind}_num_{win}": nw})
            off = "rowWindowOffset" if kind == "bcsr" else "colWindowOffset"
            a2 = "sparseA2B" if kind == "bcsr" else "sparseA2C"
            datas.update({f"{prefix}_{kind}_{off}": wo, f"{prefix}_{kind}_tcOffset": tco,
                          f"{prefix}_{kind}_{a2}": idx, f"{prefix}_{kind}_tcLocalBit": bits,
                          f"{prefix}_{kind}_data": vals})
    coo = gcn.CooData(f_row_indices=blocks[1].edge_dst, f_col_indices=blocks[1].edge_src,
                      s_row_indices=blocks[0].edge_dst, s_col_indices=blocks[0].edge_src)
    return gcn.SparseMatrixSize(**sizes), gcn.SparseMatrixData(**datas), coo


def batch_feature_maps(store, input_ids: torch.Tensor):
    """The batch's cache_search_map and id_map (indexed by the first block's
    local source column) from a FeatureStore over all nodes."""
    idx = input_ids.to(torch.int64)
    return store.cache_search_map[idx].contiguous(), store.id_map[idx].contiguous()
