"""Host logic of the hot/cold feature store's cold-row staging plan (CPU)."""
import numpy as np
import torch

from tcc_b200.feature_store import cold_stage_plan


def _maps(n, hot):
    csm = np.full(n, -1, np.int32)
    csm[hot] = np.arange(len(hot), dtype=np.int32)
    cold = np.setdiff1d(np.arange(n), hot)
    idm = np.full(n, -1, np.int32)
    idm[cold] = np.arange(cold.size, dtype=np.int32)
    return torch.from_numpy(csm), torch.from_numpy(idm), cold


def test_plan_maps_each_read_cold_row_once():
    n = 50
    hot = np.array([0, 3, 7, 20, 41])
    csm, idm, cold = _maps(n, hot)
    # tile indices: repeats, hot ids, padding (-1 as int32, and out of range)
    cols = torch.tensor([5, 3, 5, 49, -1, 7, 12, 60, 12, 0, 33], dtype=torch.int32)
    c, ids, stage_map = cold_stage_plan(cols, csm, idm, n)
    assert c.tolist() == [5, 12, 33, 49]
    assert ids.tolist() == [int(idm[k]) for k in (5, 12, 33, 49)]
    for i, k in enumerate(c.tolist()):
        assert int(stage_map[k]) == i
    others = np.setdiff1d(np.arange(n), c.numpy())
    assert (stage_map[torch.from_numpy(others)] == -1).all()


def test_plan_rows_read_through_the_stage_equal_the_host_rows():
    """stage[stage_map[c]] == host_cold[id_map[c]] for every cold column read."""
    rng = np.random.default_rng(3)
    n, F = 300, 8
    hot = np.sort(rng.choice(n, 60, replace=False))
    csm, idm, cold = _maps(n, hot)
    host_cold = torch.from_numpy(rng.standard_normal((cold.size, F)).astype(np.float32))
    cols = torch.from_numpy(rng.integers(0, n, 500).astype(np.int32))
    c, ids, stage_map = cold_stage_plan(cols, csm, idm, n)
    stage = host_cold[ids]  # what the row-gather kernel writes
    for k in cols.tolist():
        if int(csm[k]) < 0:
            assert torch.equal(stage[int(stage_map[k])], host_cold[int(idm[k])])


def test_plan_empty_when_every_column_is_hot():
    n = 10
    csm, idm, _ = _maps(n, np.arange(n))
    c, ids, stage_map = cold_stage_plan(torch.arange(n, dtype=torch.int32), csm, idm, n)
    assert c.numel() == 0 and ids.numel() == 0 and (stage_map == -1).all()
