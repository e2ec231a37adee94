"""HostPipeline (tcc_b200.hostio): steps whose inputs come from pinned host
memory and whose outputs return there, with uploads, passes and downloads
overlapped across steps on three streams and two device buffer sets.  Every
step's outputs must equal the same passes run on device-resident inputs, for
several steps in flight at once (each step with its own host buffers)."""
import numpy as np
import pytest
import torch

from gpu_util import csr_dev, dense
from tcc_b200 import graphs as G
from tcc_b200 import tiles
from tcc_b200.hostio import HostPipeline

pytestmark = pytest.mark.gpu


def test_host_pipeline_matches_device_passes(gpu):
    g = G.rmat(13, 16 << 13, seed=51)
    rp, col = csr_dev(g)
    fwd_t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    bwd_t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    rs, cs = G.gcn_scales(g)
    rs_d, cs_d = dense(rs), dense(cs)
    F = 128

    def fwd(X, Y):
        tiles.bcsr_spmm(fwd_t, X, Y, tc_threshold=65, rs=rs_d, cs=cs_d)

    def bwd(Gm, Z):
        tiles.bcsc_spmm_t(bwd_t, Gm, Z, tc_threshold=65, rs=rs_d, cs=cs_d)

    pipe = HostPipeline(fwd, bwd, (g.cols, F), (g.rows, F), (g.rows, F), (g.cols, F))
    steps = 5
    hX = [torch.from_numpy(G.features(g.cols, F, seed=60 + i)).pin_memory() for i in range(steps)]
    hG = [torch.from_numpy(G.features(g.rows, F, seed=70 + i)).pin_memory() for i in range(steps)]
    hY = [torch.full((g.rows, F), float("nan")).pin_memory() for _ in range(steps)]
    hZ = [torch.full((g.cols, F), float("nan")).pin_memory() for _ in range(steps)]
    for i in range(steps):
        pipe.submit(hX[i], hG[i], hY[i], hZ[i])
    pipe.synchronize()
    assert pipe.h2d_bytes == steps * (hX[0].numel() + hG[0].numel()) * 4
    assert pipe.d2h_bytes == steps * (hY[0].numel() + hZ[0].numel()) * 4
    for i in range(steps):
        Y = tiles.bcsr_spmm(fwd_t, hX[i].cuda(), tc_threshold=65, rs=rs_d, cs=cs_d)
        Z = tiles.bcsc_spmm_t(bwd_t, hG[i].cuda(), tc_threshold=65, rs=rs_d, cs=cs_d)
        # split windows reduce in any order: equal to fp32 rounding
        np.testing.assert_allclose(hY[i].numpy(), Y.cpu().numpy(), rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(hZ[i].numpy(), Z.cpu().numpy(), rtol=1e-5, atol=1e-5)
