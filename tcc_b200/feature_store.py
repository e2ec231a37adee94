"""Hot/cold feature store of the mixed first-layer gather.

Rows of the highest-degree nodes ("hot") live in HBM; the rest ("cold") live in
pinned host memory that the GPU reads directly (zero-copy over the host link).
The lookup tables follow the reference's mixed gather
(cnic/src/core/spmm_kernel.cu:129-153, where cnic/ is
TAC_training_backend/spmm_cnic/): for condensed column c,
``g = cache_search_map[c]``; ``g >= 0`` -> row ``g % capacity`` of GPU shard
``g // capacity``; otherwise row ``id_map[c]`` of the host features.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch


def cold_stage_plan(columns: torch.Tensor, cache_search_map: torch.Tensor, id_map: torch.Tensor,
                    num_nodes: int):
    """Which cold rows an aggregation over ``columns`` reads, and where they go
    in a compact staging buffer.  Returns (cold, ids, stage_map): ``cold`` the
    sorted cold column ids among ``columns`` (ids outside [0, num_nodes) are
    padding), ``ids`` their rows in the host cold block (id_map[cold]), and
    ``stage_map`` [num_nodes] int32 with stage_map[cold[i]] = i and -1
    elsewhere -- the id map an aggregation reading the staging buffer uses."""
    c = torch.unique(columns.to(dtype=torch.int64))
    c = c[(c >= 0) & (c < num_nodes)]
    c = c[cache_search_map.to(c.device)[c] < 0]
    ids = id_map.to(c.device)[c].to(torch.int64)
    stage_map = torch.full((num_nodes,), -1, dtype=torch.int32, device=c.device)
    stage_map[c] = torch.arange(c.numel(), dtype=torch.int32, device=c.device)
    return c, ids, stage_map


class FeatureStore:
    """Features X [num_nodes x F] split by degree into an HBM part and a pinned
    host part.  ``hot_fraction`` of the nodes (highest degree first) go to HBM."""

    def __init__(self, X: np.ndarray, degrees: np.ndarray, hot_fraction: float = 0.2,
                 device=None, col_scale: np.ndarray | None = None, shards: int = 1,
                 shard_devices=None):
        """col_scale (optional): a per-node scale folded into the stored rows once,
        so an aggregation over the store computes A·diag(col_scale)·X.

        shards: the hot rows are split into this many GPU shards of
        ``capacity`` rows each, hot row g in shard g // capacity at row
        g % capacity -- the reference's per-GPU feature caches
        (cnic/src/core/spmm_kernel.cu:145-147).  shard_devices: the device of
        each shard (default: all on ``device``); shards on other GPUs are read
        over NVLink with peer access, which the caller enables."""
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        X = np.ascontiguousarray(X, dtype=np.float32)
        if col_scale is not None:
            X = (X * np.asarray(col_scale, dtype=np.float32)[:, None]).astype(np.float32)
        n, F = X.shape
        if F % 4:
            raise ValueError("feature width must be a multiple of 4")
        n_hot = int(round(hot_fraction * n))
        order = np.argsort(-degrees.astype(np.int64), kind="stable")
        hot = np.sort(order[:n_hot])
        is_hot = np.zeros(n, dtype=bool)
        is_hot[hot] = True
        cold = np.nonzero(~is_hot)[0]
        self.num_nodes, self.F = n, F
        shards = max(1, min(int(shards), max(n_hot, 1)))
        self.capacity = max((n_hot + shards - 1) // shards, 1)
        csm = np.full(n, -1, dtype=np.int32)
        csm[hot] = np.arange(n_hot, dtype=np.int32)
        idm = np.full(n, -1, dtype=np.int32)
        idm[cold] = np.arange(cold.size, dtype=np.int32)
        self.cache_search_map = torch.from_numpy(csm).to(device)
        self.id_map = torch.from_numpy(idm).to(device)
        devs = list(shard_devices) if shard_devices is not None else [device] * shards
        if len(devs) != shards:
            raise ValueError("one device per shard")
        hot_rows = X[hot] if n_hot else np.zeros((1, F), np.float32)
        self.gpu_shards = [torch.from_numpy(hot_rows[k * self.capacity:(k + 1) * self.capacity])
                           .to(devs[k]) for k in range(shards)]
        self.cpu_rows = torch.from_numpy(X[cold] if cold.size else np.zeros((1, F), np.float32)) \
            .pin_memory()
        # device array of the shards' base pointers, indexed by g // capacity
        self.gpu_ptrs = torch.tensor([t.data_ptr() for t in self.gpu_shards], dtype=torch.int64,
                                     device=device)
        self.device = torch.device(device)
        self.n_hot, self.n_cold = n_hot, int(cold.size)

    @property
    def gpu_rows(self) -> torch.Tensor:
        """The first hot-row shard (the whole hot block when there is one)."""
        return self.gpu_shards[0]

    def enable_cold_staging(self, budget_bytes: int | None = None, columns: torch.Tensor | None = None,
                            force_gather: bool = False, group=None) -> bool:
        """Allocate an HBM staging buffer for the cold rows an aggregation reads,
        if they fit ``budget_bytes`` (default: a quarter of the device's free
        memory).  ``columns``: the column ids the aggregation gathers (e.g. a
        rank's tile indices; out-of-range ids are padding); only the cold rows
        among them are staged.  The cold rows stay in pinned host memory;
        ``stage_cold`` brings them over PCIe once per call (one crossing per
        row instead of one per gather that touches it) and an aggregation reads
        ``cold_stage`` through ``stage_id_map``.  ``force_gather`` stages through
        the row-gather kernel even when every cold row is needed (tests).

        ``group`` (a process group of the ranks that hold this same store, one
        per GPU): cooperative staging -- the cold block is cut into one
        contiguous chunk per rank, each rank copies only its chunk over PCIe and
        an all-gather over NVLink assembles the whole block on every rank, so
        each cold row crosses the host link once per call for the whole job
        instead of once per rank (the GPUs of a box share the host's memory
        bandwidth).  Returns whether staging is on."""
        if self.n_cold == 0:
            return False
        device = self.device
        self.stage_group = None
        if group is not None and torch.distributed.get_world_size(group) > 1:
            world = torch.distributed.get_world_size(group)
            rank = torch.distributed.get_rank(group)
            chunk = (self.n_cold + world - 1) // world
            if budget_bytes is None:
                free, _ = torch.cuda.mem_get_info(device)
                budget_bytes = free // 4
            if (world + 1) * chunk * self.F * 4 > budget_bytes:
                return False
            self.stage_group = group
            self.cold_stage = torch.empty((world * chunk, self.F), dtype=torch.float32,
                                          device=device)
            self.stage_chunk = torch.empty((chunk, self.F), dtype=torch.float32, device=device)
            r0, r1 = min(rank * chunk, self.n_cold), min((rank + 1) * chunk, self.n_cold)
            self.stage_rows = (r0, r1)
            self.stage_ids = None
            self.stage_id_map = self.id_map  # every cold row, the host block's order
            return True
        ids = stage_map = None
        if columns is not None:
            c, ids, stage_map = cold_stage_plan(columns.to(device), self.cache_search_map, self.id_map,
                                                self.num_nodes)
            if c.numel() == self.n_cold and not force_gather:
                ids = stage_map = None
        n_stage = self.n_cold if ids is None else ids.numel()
        if budget_bytes is None:
            free, _ = torch.cuda.mem_get_info(device)
            budget_bytes = free // 4
        if n_stage * self.F * 4 > budget_bytes:
            return False
        self.cold_stage = torch.empty((max(n_stage, 1), self.F), dtype=torch.float32, device=device)
        if ids is None:  # every cold row: one bulk copy, same row order as the host block
            self.stage_ids = None
            self.stage_id_map = self.id_map
        else:
            self.stage_ids = ids
            self.stage_id_map = stage_map
        return True

    def stage_cold(self, stream: torch.cuda.Stream) -> None:
        """Bring the staged cold rows from pinned host memory into ``cold_stage``
        on ``stream`` (async): one bulk copy when every cold row is staged, else
        the row-gather kernel reading the host rows zero-copy; with cooperative
        staging, this rank's chunk over PCIe and an all-gather of the chunks
        (``stream`` then waits for the all-gather)."""
        if getattr(self, "stage_group", None) is not None:
            r0, r1 = self.stage_rows
            with torch.cuda.stream(stream):
                if r1 > r0:
                    self.stage_chunk[:r1 - r0].copy_(self.cpu_rows[r0:r1], non_blocking=True)
                work = torch.distributed.all_gather_into_tensor(
                    self.cold_stage, self.stage_chunk, group=self.stage_group, async_op=True)
                work.wait()  # the stream waits for the gathered block
            return
        if self.stage_ids is None:
            with torch.cuda.stream(stream):
                self.cold_stage.copy_(self.cpu_rows, non_blocking=True)
            return
        if self.stage_ids.numel() == 0:
            return
        import ctypes as C
        from . import _lib as L
        L.call("tcc_gather_rows", C.c_void_p(self.cpu_rows.data_ptr()), self.F, self.n_cold,
               C.c_void_p(self.stage_ids.data_ptr()), self.stage_ids.numel(),
               C.c_void_p(self.cold_stage.data_ptr()), self.F, self.F, None,
               C.c_void_p(stream.cuda_stream))

    @property
    def cpu_ptr(self) -> int:
        """Device-visible address of the pinned host rows (unified addressing)."""
        return self.cpu_rows.data_ptr()

    def hot_bytes(self) -> int:
        return self.n_hot * self.F * 4

    def cold_bytes(self) -> int:
        return self.n_cold * self.F * 4

    def dense(self) -> torch.Tensor:
        """All rows gathered into one HBM tensor (for checking)."""
        out = torch.empty((self.num_nodes, self.F), dtype=torch.float32, device=self.device)
        hot = self.cache_search_map >= 0
        g = self.cache_search_map[hot].long()
        rows = torch.cat([t.to(self.device) for t in self.gpu_shards])
        out[hot] = rows[g]
        cold = ~hot
        out[cold] = self.cpu_rows.to(out.device)[self.id_map[cold].long()]
        return out
