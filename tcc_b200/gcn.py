"""GCN on the tiled SpMM: the reference's CNICSPMMFunction / GCNConv / GCN
(train/tcgnn_conv_release.py:49-268, train/ = TAC_training_backend/train/) on
tcc_b200's kernels, plus the graph container the trainer uses.

Two entry levels:

* ``CNICSPMMFunction`` keeps the reference's signature and namedtuples
  (SparseMatrixSize / SparseMatrixData / CooData, ``s_*`` tiles for the first
  layer, ``f_*`` for the others).  Forward: X_out = (BCSR + BCSC)·X through
  :mod:`spmm_cnic`, then X_out·W.  Backward replaces the reference's
  ``torch.sparse.mm(A_topo.T, dY)`` (:150-154) by the transposed tile passes:
  a pull over the BCSC part and a push over the BCSR part.
* ``TiledGraph`` + ``GCN`` — one graph tiled once as BCSR (forward, pull) and as
  BCSC (backward Aᵀ, pull), optional GCN scales fused, optional hot/cold
  feature store for the first layer's input rows.
"""
from __future__ import annotations

from collections import namedtuple

import torch

from . import spmm_cnic
from . import tiles as T

CooData = namedtuple("CooData", ["f_row_indices", "f_col_indices",
                                 "s_row_indices", "s_col_indices"])
SparseMatrixSize = namedtuple("SparseMatrixSize", [
    "f_bcsr_num_rows", "f_bcsr_num_cols", "f_bcsr_nnz", "f_bcsr_num_TCBlocks",
    "f_bcsr_num_rowWindows",
    "f_bcsc_num_rows", "f_bcsc_num_cols", "f_bcsc_nnz", "f_bcsc_num_TCBlocks",
    "f_bcsc_num_colWindows",
    "s_bcsr_num_rows", "s_bcsr_num_cols", "s_bcsr_nnz", "s_bcsr_num_TCBlocks",
    "s_bcsr_num_rowWindows",
    "s_bcsc_num_rows", "s_bcsc_num_cols", "s_bcsc_nnz", "s_bcsc_num_TCBlocks",
    "s_bcsc_num_colWindows"])
SparseMatrixData = namedtuple("SparseMatrixData", [
    "f_bcsr_rowWindowOffset", "f_bcsr_tcOffset", "f_bcsr_sparseA2B", "f_bcsr_tcLocalBit",
    "f_bcsr_data",
    "f_bcsc_colWindowOffset", "f_bcsc_tcOffset", "f_bcsc_sparseA2C", "f_bcsc_tcLocalBit",
    "f_bcsc_data",
    "s_bcsr_rowWindowOffset", "s_bcsr_tcOffset", "s_bcsr_sparseA2B", "s_bcsr_tcLocalBit",
    "s_bcsr_data",
    "s_bcsc_colWindowOffset", "s_bcsc_tcOffset", "s_bcsc_sparseA2C", "s_bcsc_tcLocalBit",
    "s_bcsc_data"])


def _layer_parts(prefix, sz, data):
    g = lambda n: getattr(sz, f"{prefix}_{n}")  # noqa: E731
    h = lambda n: getattr(data, f"{prefix}_{n}")  # noqa: E731
    bcsr = (g("bcsr_num_rows"), g("bcsr_num_cols"), g("bcsr_nnz"), g("bcsr_num_TCBlocks"),
            g("bcsr_num_rowWindows"), h("bcsr_rowWindowOffset"), h("bcsr_tcOffset"),
            h("bcsr_sparseA2B"), h("bcsr_tcLocalBit"))
    bcsc = (g("bcsc_num_rows"), g("bcsc_num_cols"), g("bcsc_nnz"), g("bcsc_num_TCBlocks"),
            g("bcsc_num_colWindows"), h("bcsc_colWindowOffset"), h("bcsc_tcOffset"),
            h("bcsc_sparseA2C"), h("bcsc_tcLocalBit"))
    return bcsr, bcsc


def transpose_apply(bcsr: T.Tiles | None, bcsc: T.Tiles | None, G: torch.Tensor,
                    num_cols: int, tc_threshold: int = 0, rs=None, cs=None) -> torch.Tensor:
    """Aᵀ·G for A = BCSR part + BCSC part (the reference's backward SpMM)."""
    F = G.shape[1]
    G = G.contiguous()
    if bcsc is not None:
        Z = T.bcsc_spmm_t(bcsc, G, tc_threshold=tc_threshold, rs=rs, cs=cs)
    else:
        Z = torch.zeros((num_cols, F), dtype=torch.float32, device=G.device)
    if bcsr is not None:
        T.bcsr_spmm_t(bcsr, G, Z, tc_threshold=tc_threshold, rs=rs, cs=cs)
    return Z


class CNICSPMMFunction(torch.autograd.Function):
    """The reference's autograd op (train/tcgnn_conv_release.py:49-166), same
    arguments; every tensor in the namedtuples is a CUDA tensor in the reference
    layouts (index arrays uint32/int32, bitmaps uint64/int64)."""

    @staticmethod
    def forward(ctx, first_layer, sparse_matrix_size, sparse_matrix_data, coo_data,
                cpu_float_feature_len, gpu_node_capacity, feature_dim,
                ids, cpu_feature_cache_ptr, cache_search_map, gpu_feature_cache_ptr,
                x, weights, weight_vertical_axis_dim, device):
        prefix = "s" if first_layer else "f"
        bcsr_args, bcsc_args = _layer_parts(prefix, sparse_matrix_size, sparse_matrix_data)
        F = int(weight_vertical_axis_dim)
        if first_layer and (x is None or x.numel() == 0):
            X_out = spmm_cnic.forward_tensorcore_mixed(
                *bcsr_args, *bcsc_args, cpu_float_feature_len, gpu_node_capacity, feature_dim,
                ids, cpu_feature_cache_ptr, cache_search_map, gpu_feature_cache_ptr)
        else:
            X_out = spmm_cnic.forward_tensorcore(*bcsr_args, *bcsc_args, F,
                                                 x.contiguous().view(-1, F))
        rows = int(bcsr_args[0])
        X_out = X_out.reshape(rows, F)
        X_gat = torch.mm(X_out, weights)
        ctx.save_for_backward(X_out, weights)
        ctx.parts = (T.from_arrays("bcsr", *bcsr_args) if bcsr_args[3] else None,
                     T.from_arrays("bcsc", *bcsc_args) if bcsc_args[3] else None)
        ctx.num_cols = int(bcsr_args[1])
        ctx.x_needs_grad = x is not None and x.requires_grad
        return X_gat

    @staticmethod
    def backward(ctx, d_output):
        X_out, weights = ctx.saved_tensors
        grad_weights = torch.mm(X_out.t(), d_output)
        grad_X = None
        if ctx.x_needs_grad:
            bcsr, bcsc = ctx.parts
            grad_sp = transpose_apply(bcsr, bcsc, d_output.contiguous(), ctx.num_cols)
            grad_X = grad_sp @ weights.t()
        return (None, None, None, None, None, None, None, None, None, None, None,
                grad_X, grad_weights, None, None)


# ----------------------------------------------------- ReLU + dropout --

class ReluDropout(torch.autograd.Function):
    """relu then dropout(p) in one pass (tcc_relu_dropout_forward); the
    backward needs only the output (tcc_relu_dropout_backward).  The reference
    runs torch.relu and F.dropout separately (train/tcgnn_conv_release.py:229-240)."""

    @staticmethod
    def forward(ctx, x, p: float, seed: int):
        import ctypes as C
        from . import _lib as L
        x = x.contiguous()
        out = torch.empty_like(x)
        L.call("tcc_relu_dropout_forward", C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
               x.numel(), float(p), int(seed) & ((1 << 64) - 1),
               C.c_void_p(torch.cuda.current_stream().cuda_stream))
        ctx.p = float(p)
        ctx.save_for_backward(out)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        import ctypes as C
        from . import _lib as L
        (out,) = ctx.saved_tensors
        grad_out = grad_out.contiguous()
        grad_in = torch.empty_like(out)
        L.call("tcc_relu_dropout_backward", C.c_void_p(grad_out.data_ptr()),
               C.c_void_p(out.data_ptr()), C.c_void_p(grad_in.data_ptr()), out.numel(), ctx.p,
               C.c_void_p(torch.cuda.current_stream().cuda_stream))
        return grad_in, None, None


def relu_dropout(x: torch.Tensor, p: float, seed: int, training: bool = True) -> torch.Tensor:
    """dropout(relu(x), p) fused; plain relu when not training or p == 0."""
    if not training or p == 0.0:
        return torch.relu(x)
    return ReluDropout.apply(x, p, seed)


# ------------------------------------------------------------- TiledGraph --

class TiledGraph:
    """A square graph tiled once for both directions: BCSR for the forward
    aggregation, BCSC for Aᵀ in the backward.  rs / cs: optional fused diagonal
    scales (A_hat = diag(rs) A diag(cs))."""

    def __init__(self, rowptr: torch.Tensor, col: torch.Tensor, num_nodes: int, rs=None,
                 cs=None, tc_threshold: int = 12):
        self.n = num_nodes
        self.bcsr = T.from_csr(rowptr, col, num_nodes, num_nodes, kind="bcsr")
        self.bcsc = T.from_csr(rowptr, col, num_nodes, num_nodes, kind="bcsc")
        self.rs, self.cs = rs, cs
        self.tc_threshold = tc_threshold

    def aggregate(self, X: torch.Tensor) -> torch.Tensor:
        return T.bcsr_spmm(self.bcsr, X.contiguous(), tc_threshold=self.tc_threshold,
                           rs=self.rs, cs=self.cs)

    def aggregate_t(self, G: torch.Tensor) -> torch.Tensor:
        return T.bcsc_spmm_t(self.bcsc, G.contiguous(), tc_threshold=self.tc_threshold,
                             rs=self.rs, cs=self.cs)

    def aggregate_store(self, store) -> torch.Tensor:
        """First-layer aggregation gathering from a hot/cold FeatureStore; the
        store's rows already carry the column scale (FeatureStore(col_scale=cs)),
        the row scale is applied here."""
        import ctypes as C
        from . import _lib as L
        F = store.F
        out = torch.empty((self.n, F), dtype=torch.float32, device=store.device)
        W = self.bcsr.num_windows
        full = torch.empty(((W + 1) * 8, F), dtype=torch.float32, device=out.device)
        sc = self.bcsr.scratch()
        s = self.bcsr.struct()
        L.call("tcc_cnic_forward_mixed", C.byref(s), None, C.c_void_p(store.id_map.data_ptr()),
               C.c_void_p(store.cpu_ptr), C.c_void_p(store.cache_search_map.data_ptr()),
               C.c_void_p(store.gpu_ptrs.data_ptr()), store.capacity,
               C.c_void_p(full.data_ptr()), F, self.tc_threshold, C.c_void_p(sc.data_ptr()),
               sc.numel(), C.c_void_p(torch.cuda.current_stream().cuda_stream))
        out.copy_(full[: self.n])
        if self.rs is not None:
            out.mul_(self.rs[:, None])
        return out


class _Aggregate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, graph: TiledGraph, X):
        ctx.graph = graph
        return graph.aggregate(X)

    @staticmethod
    def backward(ctx, dY):
        return None, ctx.graph.aggregate_t(dY)


class GCNConv(torch.nn.Module):
    """Aggregate first, then transform (train/tcgnn_conv_release.py:169-194)."""

    def __init__(self, input_dim, output_dim, first_layer=False):
        super().__init__()
        self.first_layer = first_layer
        self.weights = torch.nn.Parameter(torch.empty(input_dim, output_dim))
        torch.nn.init.xavier_uniform_(self.weights)
        self.weight_vertical_axis_dim = input_dim

    def forward(self, graph: TiledGraph, x):
        if isinstance(x, torch.Tensor):
            agg = _Aggregate.apply(graph, x) if x.requires_grad else graph.aggregate(x)
        else:  # a FeatureStore: the input features need no gradient
            agg = graph.aggregate_store(x)
        return agg @ self.weights


class GCN(torch.nn.Module):
    """Two-layer GCN of train/tcgnn_conv_release.py:196-268."""

    def __init__(self, num_features, hidden_dim, num_classes, dropout=0.5, seed=0):
        super().__init__()
        self.conv1 = GCNConv(num_features, hidden_dim, first_layer=True)
        self.conv_final = GCNConv(hidden_dim, num_classes)
        self.p = dropout
        self._seed = seed
        self._calls = 0

    def forward(self, graph: TiledGraph, x):
        # relu + dropout in one pass; a fresh dropout draw per call
        self._calls += 1
        h = relu_dropout(self.conv1(graph, x), self.p, self._seed * 1_000_003 + self._calls,
                         self.training)
        return self.conv_final(graph, h)
