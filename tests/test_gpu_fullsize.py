"""Parity at the benchmark configurations' full sizes, on the graphs bench.py times.

Config 2 is the bench's own graph (R-MAT 2^20, 16 M directed edges symmetrised,
deduplicated, self-loops added, GCN scales; the bench's GPU generator and seed),
checked at F = 128 through the kernels the bench runs:
  * BCSR / BCSC / SWTCF tiles byte for byte against the canonical oracle, and
    the reference converter's output (canonicalised) against ours;
  * the forward pull (BCSR) and the transposed pull (BCSC) on random N(0,1)
    inputs against the oracle's fp64-accumulated CSR products (relative
    Frobenius <= 5e-3 at tc_threshold 12, <= 1e-5 with fp32-accurate tiles);
  * the forward against the reference launchSWTCFSpMM on the same graph, with X
    pre-scaled by the column scales and the output post-scaled by the row scales
    (||a - b||_inf / ||b||_inf <= 1e-3).
A directed R-MAT 2^20 (config 5's generator at scale 20, row-normalised)
checks forward and transposed passes where A != A^T, and config 3 at half size
(SBM, 116,482 nodes) checks the 602 -> 256 projection followed by the F = 256
SpMM.
"""
import numpy as np
import pytest
import torch

from gpu_util import SWTCF_KEYS, dense, rel_fro, rel_inf
from tcc_b200 import graphs as G
from tcc_b200 import swtcf, tiles

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3
FP32_TOL = 1e-5
REF_TOL = 1e-3


def host_csr(rowptr, col, cols):
    return G.Csr(rowptr.numel() - 1, cols, rowptr.cpu().numpy().astype(np.uint64),
                 col.cpu().numpy().view(np.uint32))


def randn(shape, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(shape, generator=gen, device="cuda")


def tiles_equal(dev, ref, kind):
    off, idx, nwin = (("rowWindowOffset", "sparseA2B", "num_rowWindows") if kind == "bcsr" else
                      ("colWindowOffset", "sparseA2C", "num_colWindows"))
    h = dev.to_host()
    T = ref["num_TCBlocks"]
    assert h["num_TCBlocks"] == T and h[nwin] == ref[nwin]
    assert np.array_equal(h[off], ref[off])
    assert np.array_equal(h["tcOffset"][:T + 1], ref["tcOffset"])
    assert np.array_equal(h[idx][:8 * T], ref[idx])
    assert np.array_equal(h["tcLocalBit"][:T], ref["tcLocalBit"])


@pytest.fixture(scope="module")
def config2(gpu):
    rp, col, _ = G.rmat_gpu(20, 16 << 20, seed=1, device="cuda")
    g = host_csr(rp, col, rp.numel() - 1)
    rs, cs = G.gcn_scales(g)
    bcsr = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    bcsc = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    return dict(g=g, rp=rp, col=col, rs=rs, cs=cs, bcsr=bcsr, bcsc=bcsc)


def test_config2_tiles_bit_exact(config2, oracle):
    g = config2["g"]
    assert g.nnz > 30_000_000
    tiles_equal(config2["bcsr"], oracle.bcsr_from_csr(g), "bcsr")
    tiles_equal(config2["bcsc"], oracle.bcsc_from_csr(g), "bcsc")


def test_config2_forward_and_transposed_vs_oracle(config2, oracle, monkeypatch):
    g, rs, cs = config2["g"], config2["rs"], config2["cs"]
    rs_d, cs_d = dense(rs), dense(cs)
    X = randn((g.cols, 128), 1000)
    Gm = randn((g.rows, 128), 1001)
    Xh, Gh = X.cpu().numpy(), Gm.cpu().numpy()
    want = oracle.csr_spmm(g, Xh, rs, cs)
    want_t = oracle.csr_spmm_t(g, Gh, rs, cs)
    monkeypatch.delenv("TCC_PULL_KERNEL", raising=False)  # the bench's kernel (bulk-copy)
    for thr, tol in ((12, TF32_TOL), (65, FP32_TOL)):
        Y = tiles.bcsr_spmm(config2["bcsr"], X, tc_threshold=thr, rs=rs_d, cs=cs_d)
        Z = tiles.bcsc_spmm_t(config2["bcsc"], Gm, tc_threshold=thr, rs=rs_d, cs=cs_d)
        assert tiles.pull_device_error(config2["bcsr"]) == 0
        assert tiles.pull_device_error(config2["bcsc"]) == 0
        e, et = rel_fro(Y.cpu().numpy(), want), rel_fro(Z.cpu().numpy(), want_t)
        assert e <= tol and et <= tol, (thr, e, et)
    # the register-gather kernel on the same inputs
    monkeypatch.setenv("TCC_PULL_KERNEL", "ldg")
    Y = tiles.bcsr_spmm(config2["bcsr"], X, tc_threshold=65, rs=rs_d, cs=cs_d)
    assert rel_fro(Y.cpu().numpy(), want) <= FP32_TOL


def test_config2_vs_reference_kernel(config2, oracle):
    """The bench's forward (GCN scales fused) against the reference's own
    launchSWTCFSpMM, which is pattern-only: fed cs * X, post-scaled by rs."""
    if oracle.ref_lib() is None:
        pytest.fail("oracle/_ref/libtcc_ref.so missing: run `make -C oracle ref` before shipping")
    g, rs, cs = config2["g"], config2["rs"], config2["cs"]
    X = randn((g.cols, 128), 1000)
    Y = tiles.bcsr_spmm(config2["bcsr"], X, tc_threshold=12, rs=dense(rs), cs=dense(cs))
    dst, src = g.coo()
    ref, _ = oracle.ref_swtcf_spmm(g.rows, g.cols, dst, src, X.cpu().numpy() * cs[:, None],
                                   tc_threshold=12)
    ref *= rs[:, None]
    assert rel_inf(Y.cpu().numpy(), ref) <= REF_TOL
    assert rel_fro(Y.cpu().numpy(), ref) <= TF32_TOL


def test_config2_swtcf_bit_exact_and_reference_converter(config2, oracle):
    g = config2["g"]
    m = swtcf.SWTCFMatrix(g.rows, g.cols, g.nnz, 16)
    ws = swtcf.SWTCFConvertWorkspace(g.nnz, g.cols, 16)
    swtcf.convert_csr(config2["rp"], config2["col"], m, ws)
    assert ws.device_error() == 0
    ws.free()
    ours = m.to_host()
    dst, src = g.coo()
    want = oracle.swtcf_convert(g.rows, g.cols, dst, src)
    for k in SWTCF_KEYS:
        assert np.array_equal(ours[k], want[k]), k
    if oracle.ref_lib() is not None:
        ref = oracle.swtcf_canonicalize(oracle.ref_swtcf_convert(g.rows, g.cols, dst, src))
        assert ref["device_error"] == 0
        for k in SWTCF_KEYS:
            assert np.array_equal(ours[k], ref[k]), k
    # the reference-named forward on the converted tiles: Y accumulates
    X = randn((g.cols, 128), 1002)
    Y = torch.zeros((g.rows, 128), device="cuda")
    swtcf.spmm(m, X, Y, tc_threshold=12)
    assert rel_fro(Y.cpu().numpy(), oracle.csr_spmm(g, X.cpu().numpy())) <= TF32_TOL
    m.free()


def test_directed_rmat_forward_and_transposed(gpu, oracle):
    """A != A^T: config 5's generator (directed, deduplicated, no self-loops,
    row-normalised) at scale 20."""
    rp, col, _ = G.rmat_gpu(20, 16 << 20, seed=4, device="cuda", symmetric=False, loops=False)
    g = host_csr(rp, col, rp.numel() - 1)
    rs, _ = G.row_scales(g)
    bcsr = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    bcsc = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    X = randn((g.cols, 128), 4000)
    Gm = randn((g.rows, 128), 4001)
    Y = tiles.bcsr_spmm(bcsr, X, tc_threshold=12, rs=dense(rs))
    assert rel_fro(Y.cpu().numpy(), oracle.csr_spmm(g, X.cpu().numpy(), rs)) <= TF32_TOL
    Z = tiles.bcsc_spmm_t(bcsc, Gm, tc_threshold=65, rs=dense(rs))
    # Z = A^T diag(rs) G: the transposed pass scales its gathered rows by rs
    want_t = oracle.csr_spmm_t(g, Gm.cpu().numpy(), rs, None)
    assert rel_fro(Z.cpu().numpy(), want_t) <= FP32_TOL


def test_config3_half_projection_then_spmm(gpu, oracle):
    """Config 3 at half size: H = X W (602 -> 256, fp32 GEMM), then
    Y = D^-1/2 (A+I) D^-1/2 H at F = 256 through the default pull kernel, and
    the transposed pass at the same width."""
    n = 232_965 // 2
    rp, col = G.sbm_gpu(n, 50, 114_600_000 // 2, 40.0, 1.2, seed=2, device="cuda")
    g = host_csr(rp, col, n)
    rs, cs = G.gcn_scales(g)
    bcsr = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    tiles_equal(bcsr, oracle.bcsr_from_csr(g), "bcsr")
    gen = torch.Generator(device="cuda").manual_seed(2)
    X = torch.rand((n, 602), generator=gen, device="cuda") * 2 - 1
    W = torch.randn((602, 256), generator=gen, device="cuda") / 602 ** 0.5
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        H = X @ W
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    Hh = H.cpu().numpy()
    assert rel_fro(Hh, X.cpu().double().numpy() @ W.cpu().double().numpy()) <= FP32_TOL
    Y = tiles.bcsr_spmm(bcsr, H, tc_threshold=12, rs=dense(rs), cs=dense(cs))
    want = oracle.csr_spmm(g, Hh, rs, cs)
    assert rel_fro(Y.cpu().numpy(), want) <= TF32_TOL
    bcsc = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    Z = tiles.bcsc_spmm_t(bcsc, H, tc_threshold=65, rs=dense(rs), cs=dense(cs))
    assert rel_fro(Z.cpu().numpy(), oracle.csr_spmm_t(g, Hh, rs, cs)) <= FP32_TOL
