"""The full-graph GCN trainer (tcc_b200.train_gcn) on one GPU against a dense
fp64 torch GCN on the same seeded graph, features, weights and labels.

Tolerance: the SpMMs run every tile in TF32 (tc_threshold 0), so the
first-epoch loss agrees within 2e-3 relative; training lowers the loss."""
import math

import numpy as np
import pytest
import torch

from tcc_b200 import graphs as G
from tcc_b200 import train_gcn

pytestmark = pytest.mark.gpu


def _dense_loss(cfg, device):
    n = cfg["nodes"]
    scale = max(1, math.ceil(math.log2(n)))
    rowptr, col, _ = G.rmat_gpu(scale, cfg["edges"], seed=cfg["seed"], device=device, n=n)
    deg = torch.diff(rowptr).double()
    rows = torch.repeat_interleave(torch.arange(n, device=device), torch.diff(rowptr))
    A = torch.zeros((n, n), dtype=torch.float64, device=device)
    A[rows, col.long()] = 1.0
    s = deg.rsqrt()
    Ah = s[:, None] * A * s[None, :]
    rng = np.random.Generator(np.random.PCG64(cfg["seed"]))
    X = torch.from_numpy(rng.standard_normal((n, cfg["F_in"]), dtype=np.float32)).to(device).double()
    lab_rng = np.random.Generator(np.random.PCG64(cfg["seed"] + 1))
    labeled = lab_rng.random(n) < cfg["label_fraction"]
    labels = lab_rng.integers(0, cfg["classes"], size=n)
    torch.manual_seed(cfg["seed"])
    W1 = torch.empty(cfg["F_in"], cfg["hidden"], device=device)
    W2 = torch.empty(cfg["hidden"], cfg["classes"], device=device)
    torch.nn.init.xavier_uniform_(W1)
    torch.nn.init.xavier_uniform_(W2)
    H1 = torch.relu(Ah @ X @ W1.double())
    logits = Ah @ H1 @ W2.double()
    idx = torch.from_numpy(np.nonzero(labeled)[0]).to(device)
    y = torch.from_numpy(labels[np.nonzero(labeled)[0]]).to(device)
    return float(torch.nn.functional.cross_entropy(logits[idx], y, reduction="sum") / labeled.sum())


@pytest.mark.parametrize("transform_first,cold_staging,gather", [
    (False, True, False), (True, True, False), (False, False, False), (True, True, True)])
def test_gcn_trainer_matches_dense_reference(gpu, transform_first, cold_staging, gather):
    """Cold rows through the HBM staging buffer (bulk copy, or the row-gather
    kernel reading the pinned host rows) and zero-copy."""
    cfg = train_gcn.config(shrink=10)
    cfg["dropout"] = 0.0
    cfg["epochs"] = 6
    cfg["cold_staging"] = cold_staging
    cfg["cold_stage_gather"] = gather
    dev = torch.device("cuda", 0)
    r = train_gcn.train(cfg, dev, 1, 0, transform_first=transform_first)
    assert r["cold_staging"] == cold_staging
    want = _dense_loss(cfg, dev)
    assert abs(r["losses"][0] - want) / want <= 2e-3, (r["losses"][0], want)
    assert r["losses"][-1] < r["losses"][0]


def test_gcn_checkpoint_resume_continues_the_run(gpu, tmp_path):
    """6 epochs in one go == 3 epochs, checkpoint, 3 more from the checkpoint
    (dropout off, so the runs are deterministic up to kernel rounding)."""
    cfg = train_gcn.config(shrink=10)
    cfg["dropout"] = 0.0
    dev = torch.device("cuda", 0)
    full = train_gcn.train(dict(cfg, epochs=6), dev, 1, 0)
    ck = str(tmp_path / "gcn.pt")
    first = train_gcn.train(dict(cfg, epochs=3, save=ck), dev, 1, 0)
    rest = train_gcn.train(dict(cfg, epochs=6, resume=ck), dev, 1, 0)
    assert len(rest["losses"]) == 3
    got = first["losses"] + rest["losses"]
    assert max(abs(a - b) / b for a, b in zip(got, full["losses"])) < 1e-4


def test_gcn_trainer_full_size_config4_first_loss(gpu):
    """Config 4 at full size (2,449,029 nodes, ~119 M nonzeros): the trainer's
    first-epoch loss (dropout off) against the same forward pass in fp64 with
    torch.sparse on the device (cuSPARSE), within the TF32 tolerance."""
    cfg = train_gcn.config()
    cfg["dropout"] = 0.0
    cfg["epochs"] = 2
    dev = torch.device("cuda", 0)
    r = train_gcn.train(cfg, dev, 1, 0)
    n = cfg["nodes"]
    scale = max(1, math.ceil(math.log2(n)))
    rowptr, col, _ = G.rmat_gpu(scale, cfg["edges"], seed=cfg["seed"], device=dev, n=n)
    s = torch.diff(rowptr).double().rsqrt()
    rows = torch.repeat_interleave(torch.arange(n, device=dev), torch.diff(rowptr))
    vals = s[rows] * s[col.long()]
    Ah = torch.sparse_csr_tensor(rowptr, col.long(), vals, size=(n, n))
    del rows, vals
    rng = np.random.Generator(np.random.PCG64(cfg["seed"]))
    X = torch.from_numpy(rng.standard_normal((n, cfg["F_in"]), dtype=np.float32)).to(dev).double()
    lab_rng = np.random.Generator(np.random.PCG64(cfg["seed"] + 1))
    labeled = lab_rng.random(n) < cfg["label_fraction"]
    labels = lab_rng.integers(0, cfg["classes"], size=n)
    torch.manual_seed(cfg["seed"])
    W1 = torch.empty(cfg["F_in"], cfg["hidden"], device=dev)
    W2 = torch.empty(cfg["hidden"], cfg["classes"], device=dev)
    torch.nn.init.xavier_uniform_(W1)
    torch.nn.init.xavier_uniform_(W2)
    H1 = torch.relu((Ah @ X) @ W1.double())
    logits = Ah @ (H1 @ W2.double())
    idx = torch.from_numpy(np.nonzero(labeled)[0]).to(dev)
    y = torch.from_numpy(labels[np.nonzero(labeled)[0]]).to(dev)
    want = float(torch.nn.functional.cross_entropy(logits[idx], y, reduction="sum") / labeled.sum())
    assert abs(r["losses"][0] - want) / want <= 2e-3, (r["losses"][0], want)
    assert r["nnz"] > 100_000_000
