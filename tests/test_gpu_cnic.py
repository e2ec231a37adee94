"""The spmm_cnic op layer: module mirror vs the reference kernels built from
source, the hot/cold feature store, and the autograd backward (Aᵀ passes)."""
import numpy as np
import pytest
import torch

from gpu_util import csr_dev, dense, rel_fro, rel_inf
from tcc_b200 import feature_store, gcn, spmm_cnic, tiles
from tcc_b200 import graphs as G

pytestmark = pytest.mark.gpu

REF_TOL = 1e-3
FP32_TOL = 1e-5
TF32_TOL = 5e-3


def split_graph(g, frac_hot=0.5, seed=0):
    """Split A's edges into a hot part (BCSR) and a cold part (BCSC), as the
    reference sampler does with its cache split."""
    rng = np.random.default_rng(seed)
    dst, src = g.coo()
    hot = rng.random(dst.size) < frac_hot
    a = G.csr_from_pairs(dst[hot], src[hot], g.rows, g.cols)
    b = G.csr_from_pairs(dst[~hot], src[~hot], g.rows, g.cols)
    return a, b


def tile_args(t):
    return (t.num_rows, t.num_cols, t.nnz, t.num_TCBlocks, t.num_windows, t.windowOffset,
            t.tcOffset, t.sparseIdx, t.tcLocalBit)


# F >= 64: the reference kernels load the 8x8 bitmap with `tid < 64` threads
# (cnic/src/core/spmm_kernel.cu:1632-1649, :1977-1990) but launch F/32 warps, so
# at F = 32 bitmap rows 4-7 are never written and the reference output is wrong.
@pytest.mark.parametrize("F", [64, 128, 256])
def test_forward_tensorcore_vs_reference_kernels(gpu, oracle, F):
    if oracle.ref_lib() is None:
        pytest.fail("oracle/_ref/libtcc_ref.so missing: run `make -C oracle ref`")
    g = G.rmat(12, 16 << 12, seed=31)
    ga, gb = split_graph(g)
    ta = tiles.from_csr(*csr_dev(ga), g.rows, g.cols, kind="bcsr")
    tb = tiles.from_csr(*csr_dev(gb), g.rows, g.cols, kind="bcsc")
    X = G.features(g.cols, F, seed=32)
    out = spmm_cnic.forward_tensorcore(*tile_args(ta), *tile_args(tb), F, dense(X))
    ours = out.view(g.rows, F).cpu().numpy()
    ref, _ = oracle.ref_cnic_spmm(g.rows, g.cols, X, bcsr=oracle.bcsr_from_csr(ga),
                                  bcsc=oracle.bcsc_from_csr(gb))
    assert rel_inf(ours, ref) <= REF_TOL
    want = oracle.csr_spmm(g, X)
    assert rel_fro(ours, want) <= 5e-3  # TF32 on every tile, like the reference


def test_forward_tensorcore_narrow_features(gpu, oracle):
    """F = 32 (where the reference kernels misbehave): ours against the oracle."""
    g = G.rmat(11, 16 << 11, seed=30)
    ga, gb = split_graph(g)
    ta = tiles.from_csr(*csr_dev(ga), g.rows, g.cols, kind="bcsr")
    tb = tiles.from_csr(*csr_dev(gb), g.rows, g.cols, kind="bcsc")
    X = G.features(g.cols, 32, seed=31)
    out = spmm_cnic.forward_tensorcore(*tile_args(ta), *tile_args(tb), 32, dense(X),
                                       tc_threshold=65)
    assert rel_fro(out.view(g.rows, 32).cpu().numpy(), oracle.csr_spmm(g, X)) <= FP32_TOL


@pytest.mark.parametrize("shards", [1, 3])
def test_feature_store_gather_vs_oracle(gpu, oracle, shards):
    """The mixed gather (hot rows from GPU shards, row g % capacity of shard
    g // capacity; cold rows from pinned host memory) against the CPU oracle on
    the dense features, with one shard and with the hot rows split into three
    shards (cnic/src/core/spmm_kernel.cu:145-147)."""
    g = G.rmat(12, 16 << 12, seed=33)
    ga, gb = split_graph(g)
    ta = tiles.from_csr(*csr_dev(ga), g.rows, g.cols, kind="bcsr")
    tb = tiles.from_csr(*csr_dev(gb), g.rows, g.cols, kind="bcsc")
    X = G.features(g.cols, 100, seed=34)
    st = feature_store.FeatureStore(X, g.degrees(), hot_fraction=0.2, shards=shards)
    assert 0 < st.n_hot < g.cols
    assert len(st.gpu_shards) == shards and st.capacity * shards >= st.n_hot
    assert int(st.cache_search_map.max()) // st.capacity == shards - 1
    assert torch.equal(st.dense().cpu(), torch.from_numpy(X))
    want = oracle.csr_spmm(g, X)
    for thr, tol in ((65, FP32_TOL), (12, TF32_TOL)):
        mixed = spmm_cnic.forward_tensorcore_mixed(
            *tile_args(ta), *tile_args(tb), st.n_cold * 100, st.capacity, 100, st.id_map,
            st.cpu_ptr, st.cache_search_map, st.gpu_ptrs, tc_threshold=thr)
        assert rel_fro(mixed.view(g.rows, 100).cpu().numpy(), want) <= tol, thr


def test_space_malloc_and_denseC(gpu):
    g = G.uniform(1000, 8, seed=35)
    ta = tiles.from_csr(*csr_dev(g), g.rows, g.cols, kind="bcsr")
    spmm_cnic.initialize(0)
    bufs = spmm_cnic.space_malloc(0, (ta.num_windows + 1) * 8 * 64)
    X = dense(G.features(g.cols, 64, seed=36))
    out = spmm_cnic.forward_tensorcore(*tile_args(ta), g.rows, g.cols, 0, 0,
                                       (g.cols + 7) // 8, None, None, None, None, 64, X,
                                       denseC=bufs[0])
    assert out.data_ptr() == bufs[0].data_ptr()
    spmm_cnic.finalize(0)


def test_cnic_autograd_backward_matches_sparse_reference(gpu):
    """CNICSPMMFunction (non-first layer): grad_weights and grad_X against
    torch.sparse on the same split matrix, in float64 on the CPU."""
    g = G.rmat(11, 16 << 11, seed=37)
    ga, gb = split_graph(g, seed=1)
    ta = tiles.from_csr(*csr_dev(ga), g.rows, g.cols, kind="bcsr")
    tb = tiles.from_csr(*csr_dev(gb), g.rows, g.cols, kind="bcsc")
    F_in, F_out = 64, 32
    sz = gcn.SparseMatrixSize(*tile_args(ta)[:5], *tile_args(tb)[:5], *tile_args(ta)[:5],
                              *tile_args(tb)[:5])
    data = gcn.SparseMatrixData(*tile_args(ta)[5:], None, *tile_args(tb)[5:], None,
                                *tile_args(ta)[5:], None, *tile_args(tb)[5:], None)
    x = torch.randn((g.cols, F_in), device="cuda", requires_grad=True)
    w = torch.randn((F_in, F_out), device="cuda", requires_grad=True)
    y = gcn.CNICSPMMFunction.apply(False, sz, data, None, 0, 0, F_in, None, None, None, None,
                                   x, w, F_in, "cuda")
    dy = torch.randn_like(y)
    y.backward(dy)
    dst, src = g.coo()
    A = torch.sparse_coo_tensor(np.stack([dst, src]).astype(np.int64),
                                torch.ones(dst.size, dtype=torch.float64), (g.rows, g.cols))
    xd = x.detach().cpu().double().requires_grad_(True)
    wd = w.detach().cpu().double().requires_grad_(True)
    yd = torch.sparse.mm(A, xd) @ wd
    yd.backward(dy.cpu().double())
    assert rel_fro(y.detach().cpu().numpy(), yd.detach().numpy()) <= 5e-3
    assert rel_fro(w.grad.cpu().numpy(), wd.grad.numpy()) <= 5e-3
    assert rel_fro(x.grad.cpu().numpy(), xd.grad.numpy()) <= 5e-3


def test_gcn_training_step_matches_torch_reference(gpu):
    """Two-layer GCN with fused GCN scales and a hot/cold store: loss and weight
    gradients of one step against the same model in torch (float64, CPU)."""
    torch.manual_seed(0)
    g = G.rmat(11, 16 << 11, seed=38)
    rs, cs = G.gcn_scales(g)
    rp, col = csr_dev(g)
    graph = gcn.TiledGraph(rp, col, g.rows, rs=dense(rs), cs=dense(cs), tc_threshold=65)
    X = G.features(g.rows, 100, seed=39)
    store = feature_store.FeatureStore(X, g.degrees(), hot_fraction=0.2, col_scale=cs)
    model = gcn.GCN(100, 64, 7, dropout=0.0).cuda()
    labels = torch.randint(0, 7, (g.rows,), device="cuda")
    out = model(graph, store)
    loss = torch.nn.functional.cross_entropy(out, labels)
    loss.backward()
    dst, src = g.coo()
    vals = rs[dst].astype(np.float64) * cs[src].astype(np.float64)
    A = torch.sparse_coo_tensor(np.stack([dst, src]).astype(np.int64), torch.from_numpy(vals),
                                (g.rows, g.cols))
    W1 = model.conv1.weights.detach().cpu().double().requires_grad_(True)
    W2 = model.conv_final.weights.detach().cpu().double().requires_grad_(True)
    h = torch.relu(torch.sparse.mm(A, torch.from_numpy(X).double()) @ W1)
    o = torch.sparse.mm(A, h) @ W2
    lref = torch.nn.functional.cross_entropy(o, labels.cpu())
    lref.backward()
    assert abs(loss.item() - lref.item()) / abs(lref.item()) < 1e-4
    assert rel_fro(model.conv1.weights.grad.cpu().numpy(), W1.grad.numpy()) <= 1e-4
    assert rel_fro(model.conv_final.weights.grad.cpu().numpy(), W2.grad.numpy()) <= 1e-4
