"""Mini-batch path of the reference's training step: sampled blocks -> BCSR /
BCSC tile sets (all-BCSR, all-BCSC, degree split) -> CNICSPMMFunction for both
layers (layer 1 from the hot/cold feature store), against dense torch on the
same blocks: outputs and weight gradients within the TF32 tolerance (every
tile on the tensor cores, tc_threshold 0)."""
import numpy as np
import pytest
import torch

from gpu_util import csr_dev, rel_fro
from tcc_b200 import graphs as G
from tcc_b200 import minibatch
from tcc_b200.feature_store import FeatureStore
from tcc_b200.gcn import CNICSPMMFunction

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3


def _dense(b, device):
    A = torch.zeros((b.num_dst, b.num_src), dtype=torch.float64, device=device)
    A.index_put_((b.edge_dst, b.edge_src), torch.ones(b.edge_dst.numel(), dtype=torch.float64,
                                                      device=device), accumulate=True)
    return A


def test_sampler_blocks_are_consistent(gpu):
    g = G.rmat(11, 12 << 11, seed=7)
    rp, col = csr_dev(g)
    gen = torch.Generator(device="cuda").manual_seed(3)
    seeds = torch.randperm(g.rows, device="cuda", generator=gen)[:128]
    b1, b2 = minibatch.sample_blocks(rp, col, seeds, (4, 6), generator=gen)
    assert torch.equal(b2.dst_ids, seeds) and torch.equal(b1.dst_ids, b2.src_ids)
    for b, k in ((b1, 4), (b2, 6)):
        assert torch.equal(b.src_ids[:b.num_dst], b.dst_ids)
        per_dst = torch.bincount(b.edge_dst, minlength=b.num_dst)
        deg = (rp[b.dst_ids + 1] - rp[b.dst_ids])
        assert torch.equal(per_dst, torch.minimum(deg, torch.full_like(deg, k)))
        # every sampled edge exists in the graph
        gd, gs = b.dst_ids[b.edge_dst], b.src_ids[b.edge_src]
        keys = rp.new_tensor(np.repeat(np.arange(g.rows), np.diff(g.rowptr.astype(np.int64)))) * \
            (1 << 32) + col.to(torch.int64)
        assert bool(torch.isin(gd * (1 << 32) + gs, keys).all())


@pytest.mark.parametrize("split", ["bcsr", "bcsc", "degree"])
def test_minibatch_cnic_two_layers(gpu, split):
    dev = torch.device("cuda", 0)
    g = G.rmat(11, 12 << 11, seed=8)
    rp, col = csr_dev(g)
    gen = torch.Generator(device="cuda").manual_seed(5)
    seeds = torch.randperm(g.rows, device="cuda", generator=gen)[:200]
    blocks = minibatch.sample_blocks(rp, col, seeds, (5, 10), generator=gen)
    size, data, coo = minibatch.sparse_inputs(blocks, split=split, hub_degree=3)
    if split == "degree":
        assert size.s_bcsr_num_TCBlocks > 0 and size.s_bcsc_num_TCBlocks > 0
    F_in, hidden, classes = 64, 32, 16
    rng = np.random.default_rng(9)
    X = rng.standard_normal((g.rows, F_in)).astype(np.float32)
    store = FeatureStore(X, g.degrees(), hot_fraction=0.3, device=dev)
    csm, idm = minibatch.batch_feature_maps(store, blocks[0].src_ids)
    torch.manual_seed(1)
    W1 = torch.randn(F_in, hidden, device=dev, requires_grad=True)
    W2 = torch.randn(hidden, classes, device=dev, requires_grad=True)
    H1 = CNICSPMMFunction.apply(True, size, data, coo, store.n_cold, store.capacity, F_in, idm,
                                store.cpu_ptr, csm, store.gpu_ptrs, None, W1, F_in, dev)
    out = CNICSPMMFunction.apply(False, size, data, coo, 0, 0, hidden, None, None, None, None,
                                 torch.relu(H1), W2, hidden, dev)
    out.sum().backward()
    # dense reference on the same blocks
    A1, A2 = _dense(blocks[0], dev), _dense(blocks[1], dev)
    Xb = torch.from_numpy(X).to(dev).double()[blocks[0].src_ids]
    V1 = W1.detach().double().requires_grad_(True)
    V2 = W2.detach().double().requires_grad_(True)
    ref = A2 @ torch.relu(A1 @ Xb @ V1) @ V2
    ref.sum().backward()
    assert rel_fro(out.detach().cpu().numpy(), ref.detach().cpu().numpy()) <= TF32_TOL
    assert rel_fro(W2.grad.cpu().numpy(), V2.grad.cpu().numpy()) <= TF32_TOL
    assert rel_fro(W1.grad.cpu().numpy(), V1.grad.cpu().numpy()) <= TF32_TOL
