"""GPU SpMM passes against the CPU oracle, the reference's known-answer test and
the reference kernels built from source.

Tolerances (stated per north star): fp32 tiles (tc_threshold 65) against the
fp64 CSR oracle: relative Frobenius <= 1e-5; TF32 tiles: <= 5e-3; against the
reference swtcf_spmm on the same inputs: ||a-b||_inf / ||b||_inf <= 1e-3.
"""
import numpy as np
import pytest
import torch

from gpu_util import csr_dev, dense, edge_case_graphs, rel_fro, rel_inf, u32
from tcc_b200 import graphs as G
from tcc_b200 import swtcf, tiles

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
TF32_TOL = 5e-3
REF_TOL = 1e-3

CASES = edge_case_graphs()


def make_swtcf(g, S=16):
    m = swtcf.SWTCFMatrix(g.rows, g.cols, g.nnz, S)
    ws = swtcf.SWTCFConvertWorkspace(g.nnz, g.cols, S)
    dst, src = g.coo()
    swtcf.convert_coo(u32(dst), u32(src), m, ws)
    assert ws.device_error() == 0
    return m


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("thr", [12, 65, 0])
def test_swtcf_spmm_reference_semantics(gpu, oracle, name, g, thr):
    """launchSWTCFSpMM: F=128, Y accumulates, pattern-only A."""
    m = make_swtcf(g)
    X = G.features(g.cols, 128, seed=1)
    Y0 = G.features(g.rows, 128, seed=2)
    Yd = dense(Y0)
    swtcf.spmm(m, dense(X), Yd, tc_threshold=thr)
    got = Yd.cpu().numpy()
    host = oracle.swtcf_convert(g.rows, g.cols, *g.coo())
    want = oracle.swtcf_spmm(host, X, tc_threshold=thr, Y=Y0.copy())
    assert rel_fro(got, want) <= FP32_TOL, name
    exact = oracle.csr_spmm(g, X) + Y0
    assert rel_fro(got, exact) <= (FP32_TOL if thr > 64 else TF32_TOL)


def test_swtcf_spmm_known_answer(gpu, oracle):
    """The reference's closed-form X check (src/swtcf_spmm_main.cu:33-112)."""
    g = G.rmat(14, 16 << 14, seed=7)
    m = make_swtcf(g)
    dst, src = g.coo()
    X = oracle.kat_features(g.cols)
    for thr, atol, rtol in ((12, 1e-2, 1e-2), (65, 2e-4, 1e-4)):
        Y = torch.zeros((g.rows, 128), device="cuda")
        swtcf.spmm(m, dense(X), Y, tc_threshold=thr)
        s = src.astype(np.uint32)
        a = ((s * np.uint32(17) + np.uint32(13)) % np.uint32(97)).astype(np.float32) * np.float32(0.001)
        b = ((s * np.uint32(29) + np.uint32(7)) % np.uint32(89)).astype(np.float32) * np.float32(1e-5)
        sa = np.zeros(g.rows)
        sb = np.zeros(g.rows)
        np.add.at(sa, dst, a.astype(np.float64))
        np.add.at(sb, dst, b.astype(np.float64))
        ref = sa[:, None] + sb[:, None] * np.arange(128)[None, :]
        err = np.abs(Y.cpu().numpy() - ref)
        assert np.all(err <= atol + rtol * np.abs(ref)), (thr, err.max())


@pytest.mark.parametrize("name,g", CASES[:5], ids=[c[0] for c in CASES[:5]])
def test_swtcf_spmm_vs_reference_kernel(gpu, oracle, name, g):
    """Our SWTCF SpMM vs the reference launchSWTCFSpMM on the same COO and X."""
    if oracle.ref_lib() is None:
        pytest.fail("oracle/_ref/libtcc_ref.so missing: run `make -C oracle ref` before shipping")
    dst, src = g.coo()
    X = G.features(g.cols, 128, seed=4)
    ref, _ = oracle.ref_swtcf_spmm(g.rows, g.cols, dst, src, X, tc_threshold=12)
    m = make_swtcf(g)
    Y = torch.zeros((g.rows, 128), device="cuda")
    swtcf.spmm(m, dense(X), Y, tc_threshold=12)
    assert rel_inf(Y.cpu().numpy(), ref) <= REF_TOL


@pytest.mark.parametrize("F", [4, 64, 100, 128, 256])
@pytest.mark.parametrize("thr", [12, 65])
def test_swtcf_spmm_ex_scales(gpu, oracle, F, thr):
    g = G.rmat(12, 16 << 12, seed=3)
    rs, cs = G.gcn_scales(g)
    m = make_swtcf(g)
    X = G.features(g.cols, F, seed=5)
    Y = swtcf.spmm_ex(m, dense(X), tc_threshold=thr, row_scale=dense(rs), col_scale=dense(cs))
    want = oracle.csr_spmm(g, X, rs, cs)
    assert rel_fro(Y.cpu().numpy(), want) <= (FP32_TOL if thr > 64 else TF32_TOL)
    # accumulate adds on top
    Y2 = swtcf.spmm_ex(m, dense(X), Y=Y.clone(), tc_threshold=thr, row_scale=dense(rs),
                       col_scale=dense(cs), accumulate=True)
    assert rel_fro(Y2.cpu().numpy(), 2 * want) <= (FP32_TOL if thr > 64 else TF32_TOL)


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("F", [64, 128])
def test_swtcf_transposed(gpu, oracle, name, g, F):
    rs, cs = G.gcn_scales(g) if g.rows == g.cols else (None, None)
    m = make_swtcf(g)
    Gm = G.features(g.rows, F, seed=6)
    Z = swtcf.spmm_t(m, dense(Gm), tc_threshold=65, row_scale=None if rs is None else dense(rs),
                     col_scale=None if cs is None else dense(cs))
    want = oracle.csr_spmm_t(g, Gm, rs, cs)
    assert rel_fro(Z.cpu().numpy(), want) <= FP32_TOL, name
    Z2 = swtcf.spmm_t(m, dense(Gm), tc_threshold=12)
    assert rel_fro(Z2.cpu().numpy(), oracle.csr_spmm_t(g, Gm)) <= TF32_TOL


PULL_KERNELS = ["default", "ldg", "tma", "tma-bulk", "umma"]


@pytest.fixture(params=PULL_KERNELS)
def pull_kernel(request, monkeypatch):
    """Run a pull test on each pull kernel: the default dispatch (bulk-copy
    kernel for F a multiple of 128, register-gather kernel otherwise), the
    register-gather kernel (TCC_PULL_KERNEL=ldg), the TMA gather kernel (=tma)
    with its tile::gather4 copies and with per-row bulk copies
    (TCC_PULL_COPY=bulk), and the tcgen05 kernel (=umma; tc_threshold 0, F a
    multiple of 128).  Shapes a kernel does not take fall back to the
    register-gather kernel."""
    monkeypatch.delenv("TCC_PULL_COPY", raising=False)
    if request.param == "default":
        monkeypatch.delenv("TCC_PULL_KERNEL", raising=False)
    elif request.param == "tma-bulk":
        monkeypatch.setenv("TCC_PULL_KERNEL", "tma")
        monkeypatch.setenv("TCC_PULL_COPY", "bulk")
    else:
        monkeypatch.setenv("TCC_PULL_KERNEL", request.param)
    return request.param


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("F,thr", [(128, 65), (128, 12), (128, 0), (4, 65), (32, 65), (64, 65),
                                   (100, 12), (256, 12), (512, 65), (48, 0), (8, 0), (384, 12)])
def test_bcsr_pull(gpu, oracle, pull_kernel, name, g, F, thr):
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    rs, cs = G.gcn_scales(g) if g.rows == g.cols else G.row_scales(g)
    X = G.features(g.cols, F, seed=8)
    Y = tiles.bcsr_spmm(t, dense(X), tc_threshold=thr, rs=dense(rs),
                        cs=None if cs is None else dense(cs))
    want = oracle.csr_spmm(g, X, rs, cs)
    assert rel_fro(Y.cpu().numpy(), want) <= (FP32_TOL if thr > 64 else TF32_TOL), name
    # the plan is reused on the second call; accumulate adds
    Y2 = tiles.bcsr_spmm(t, dense(X), C_out=Y.clone(), tc_threshold=thr, rs=dense(rs),
                         cs=None if cs is None else dense(cs), accumulate=True)
    assert rel_fro(Y2.cpu().numpy(), 2 * want) <= (FP32_TOL if thr > 64 else TF32_TOL)


@pytest.mark.parametrize("kernel", ["ldg", "tma", "tma-bulk", "umma"])
def test_bcsr_pull_matches_tile_arithmetic(gpu, oracle, monkeypatch, kernel):
    """TF32 on every tile (tc_threshold 0) against its exact restatement: the
    register-gather and bulk-copy kernels round X like cvt.rna (the oracle's
    tile emulation); the tcgen05 kernel hands the tensor core raw fp32 bits
    and it drops the low 13 mantissa bits, i.e. A.trunc(X) summed in fp32.
    The device error word stays clear."""
    monkeypatch.setenv("TCC_PULL_KERNEL", kernel.split("-")[0])
    if kernel == "tma-bulk":
        monkeypatch.setenv("TCC_PULL_COPY", "bulk")
    else:
        monkeypatch.delenv("TCC_PULL_COPY", raising=False)
    g = G.sbm(2000, 20, 120000, 40.0, 1.2, seed=12)
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    X = G.features(g.cols, 128, seed=9)
    Y = tiles.bcsr_spmm(t, dense(X), tc_threshold=0)
    if kernel in ("ldg", "tma", "tma-bulk"):
        want = oracle.bcsr_spmm(oracle.bcsr_from_csr(g), X, tc_threshold=0)
    else:
        want = oracle.csr_spmm(g, oracle.tf32_trunc(X))
    assert rel_fro(Y.cpu().numpy(), want) <= FP32_TOL
    Y65 = tiles.bcsr_spmm(t, dense(X), tc_threshold=65)
    assert rel_fro(Y65.cpu().numpy(), oracle.csr_spmm(g, X)) <= FP32_TOL
    assert tiles.pull_device_error(t) == 0


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("F,thr", [(128, 65), (128, 0), (64, 12), (256, 65)])
def test_bcsc_push_and_transposed(gpu, oracle, pull_kernel, name, g, F, thr):
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    X = G.features(g.cols, F, seed=10)
    C0 = G.features(g.rows, F, seed=11)
    Cd = dense(C0)
    tiles.bcsc_spmm(t, dense(X), Cd, tc_threshold=thr)
    want = oracle.csr_spmm(g, X) + C0
    tol = FP32_TOL if thr > 64 else TF32_TOL
    assert rel_fro(Cd.cpu().numpy(), want) <= tol, name
    Gm = G.features(g.rows, F, seed=12)
    Z = tiles.bcsc_spmm_t(t, dense(Gm), tc_threshold=thr)
    assert rel_fro(Z.cpu().numpy(), oracle.csr_spmm_t(g, Gm)) <= tol, name


def test_full_size_properties(gpu):
    """Config-2 size: A.1 = degree exactly (pattern-only, fp32 exact integers),
    linearity, and <A X, G> = <X, A^T G>."""
    rp, col, _ = G.rmat_gpu(20, 16 << 20, seed=1, device="cuda")  # the bench's config-2 graph
    g = G.Csr(rp.numel() - 1, rp.numel() - 1, rp.cpu().numpy().astype(np.uint64),
              col.cpu().numpy().view(np.uint32))
    bcsr = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsr")
    bcsc = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    ones = torch.ones((g.cols, 128), device="cuda")
    deg = torch.from_numpy(g.degrees().astype(np.float32)).cuda()
    Y = tiles.bcsr_spmm(bcsr, ones, tc_threshold=65)
    assert torch.equal(Y, deg[:, None].expand(-1, 128))
    Yt = tiles.bcsr_spmm(bcsr, ones, tc_threshold=0)  # TF32 of 1.0 is exact
    assert torch.equal(Yt, deg[:, None].expand(-1, 128))
    Z = tiles.bcsc_spmm_t(bcsc, ones, tc_threshold=65)
    assert torch.equal(Z, deg[:, None].expand(-1, 128))  # symmetric graph
    gen = torch.Generator(device="cuda").manual_seed(0)
    X1 = torch.randn((g.cols, 128), device="cuda", generator=gen)
    X2 = torch.randn((g.cols, 128), device="cuda", generator=gen)
    a, b = 0.75, -1.5
    L = tiles.bcsr_spmm(bcsr, a * X1 + b * X2, tc_threshold=65)
    R = a * tiles.bcsr_spmm(bcsr, X1, tc_threshold=65) + b * tiles.bcsr_spmm(bcsr, X2, tc_threshold=65)
    assert (torch.linalg.norm(L - R) / torch.linalg.norm(R)).item() < 1e-5
    Gm = torch.randn((g.rows, 128), device="cuda", generator=gen)
    lhs = torch.sum(tiles.bcsr_spmm(bcsr, X1, tc_threshold=65).double() * Gm.double())
    rhs = torch.sum(X1.double() * tiles.bcsc_spmm_t(bcsc, Gm, tc_threshold=65).double())
    assert abs((lhs - rhs) / rhs).item() < 1e-5


@pytest.mark.parametrize("name,g", CASES[:6], ids=[c[0] for c in CASES[:6]])
@pytest.mark.parametrize("thr", [12, 0, 65])
def test_swtcf_spmm_quantized(gpu, oracle, name, g, thr):
    """launchSWTCFSpMMQuantized: source column c reads the int8 row of global node
    src_global[c] times its scale; against the oracle on the dequantized rows
    (the same fp32 values) and, where the reference build is present, against
    the reference kernel."""
    m = make_swtcf(g)
    rng = np.random.default_rng(21)
    n_global = g.cols + 37
    q = rng.integers(-128, 128, size=(n_global, 128), dtype=np.int8)
    scales = (rng.random(n_global, dtype=np.float32) * 0.05).astype(np.float32)
    src_global = rng.permutation(n_global)[:g.cols].astype(np.uint32)
    Xd = (q[src_global].astype(np.float32) * scales[src_global][:, None]).astype(np.float32)
    Y = torch.zeros((g.rows, 128), dtype=torch.float32, device="cuda")
    swtcf.spmm_quantized(m, torch.from_numpy(q).cuda(), torch.from_numpy(scales).cuda(),
                         torch.from_numpy(src_global.view(np.int32)).cuda(), Y, tc_threshold=thr)
    got = Y.cpu().numpy()
    want = oracle.csr_spmm(g, Xd)
    assert rel_fro(got, want) <= (FP32_TOL if thr > 64 else TF32_TOL), name
    if oracle.ref_lib() is not None and g.nnz > 0:
        dst, src = g.coo()
        ref = oracle.ref_swtcf_spmm_quantized(g.rows, g.cols, dst, src, q, scales, src_global, thr)
        assert rel_inf(got, ref) <= REF_TOL, name


@pytest.mark.parametrize("thr", [65, 12])
def test_push_heavy_hub_window(gpu, oracle, thr):
    """A 40,000-node star: the hub's column window holds ~5,000 tiles, so the
    push pass shares it among many warps and splits its super-window over
    several CTAs (each flushing the repeat-cache rows it touched).  SWTCF
    forward (reference semantics: Y accumulates) and the BCSC push against
    the oracle, and against the reference kernel where it is built."""
    n = 40000
    u = np.zeros(n - 1, np.uint32)
    v = np.arange(1, n, dtype=np.uint32)
    g = G._symmetrise_with_loops(u, v, n)
    X = G.features(g.cols, 128, seed=31)
    Y0 = G.features(g.rows, 128, seed=32)
    want = oracle.csr_spmm(g, X) + Y0
    tol = FP32_TOL if thr > 64 else TF32_TOL
    m = make_swtcf(g)
    Yd = dense(Y0)
    swtcf.spmm(m, dense(X), Yd, tc_threshold=thr)
    assert rel_fro(Yd.cpu().numpy(), want) <= tol
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind="bcsc")
    Cd = dense(Y0)
    tiles.bcsc_spmm(t, dense(X), Cd, tc_threshold=thr)
    assert rel_fro(Cd.cpu().numpy(), want) <= tol
    if thr == 12:
        if oracle.ref_lib() is None:
            pytest.fail("oracle/_ref/libtcc_ref.so missing: run `make -C oracle ref` before shipping")
        dst, src = g.coo()
        ref, _ = oracle.ref_swtcf_spmm(g.rows, g.cols, dst, src, X, tc_threshold=12)
        Yz = torch.zeros((g.rows, 128), device="cuda")
        swtcf.spmm(m, dense(X), Yz, tc_threshold=12)
        assert rel_inf(Yz.cpu().numpy(), ref) <= REF_TOL


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
def test_swtcf_spmm_prepared_pull(gpu, oracle, name, g):
    """tcc_swtcf_prepare_pull: the forward product as a pull over a row-window
    tiling of the converted matrix.  Against the oracle (fp32 tiles at
    tc_threshold 65, TF32 at 12; Y accumulates like the reference), the
    reference kernel, and the general form with scales; a new conversion
    drops the tiling and the push runs again."""
    m = make_swtcf(g)
    X = G.features(g.cols, 128, seed=41)
    Y0 = G.features(g.rows, 128, seed=42)
    swtcf.prepare_pull(m)
    assert m.c.fwd_ready == 1
    want = oracle.csr_spmm(g, X) + Y0
    for thr, tol in ((65, FP32_TOL), (12, TF32_TOL)):
        Yd = dense(Y0)
        swtcf.spmm(m, dense(X), Yd, tc_threshold=thr)
        assert rel_fro(Yd.cpu().numpy(), want) <= tol, (name, thr)
    if oracle.ref_lib() is None:
        pytest.fail("oracle/_ref/libtcc_ref.so missing: run `make -C oracle ref` before shipping")
    dst, src = g.coo()
    ref, _ = oracle.ref_swtcf_spmm(g.rows, g.cols, dst, src, X, tc_threshold=12)
    Yz = torch.zeros((g.rows, 128), device="cuda")
    swtcf.spmm(m, dense(X), Yz, tc_threshold=12)
    assert rel_inf(Yz.cpu().numpy(), ref) <= REF_TOL, name
    rs, cs = G.gcn_scales(g) if g.rows == g.cols else G.row_scales(g)
    Ys = swtcf.spmm_ex(m, dense(X), tc_threshold=65, row_scale=dense(rs),
                       col_scale=None if cs is None else dense(cs))
    assert rel_fro(Ys.cpu().numpy(), oracle.csr_spmm(g, X, rs, cs)) <= FP32_TOL, name
    ws = swtcf.SWTCFConvertWorkspace(g.nnz, g.cols, 16)
    swtcf.convert_coo(u32(dst), u32(src), m, ws)
    assert m.c.fwd_ready == 0
    Yd = dense(Y0)
    swtcf.spmm(m, dense(X), Yd, tc_threshold=65)
    assert rel_fro(Yd.cpu().numpy(), want) <= FP32_TOL, name
