"""GPU converters against the CPU oracle (bit-exact) and against the reference
converter built from source (canonicalised, bit-exact)."""
import numpy as np
import pytest
import torch

from gpu_util import SWTCF_KEYS, csr_dev, edge_case_graphs, u32
from tcc_b200 import graphs as G
from tcc_b200 import swtcf, tiles

pytestmark = pytest.mark.gpu

CASES = edge_case_graphs()


def gpu_swtcf(g, S=16, via="coo"):
    m = swtcf.SWTCFMatrix(g.rows, g.cols, g.nnz, S)
    ws = swtcf.SWTCFConvertWorkspace(g.nnz, g.cols, S)
    if via == "coo":
        dst, src = g.coo()
        swtcf.convert_coo(u32(dst), u32(src), m, ws)
    else:
        rp, col = csr_dev(g)
        swtcf.convert_csr(rp, col, m, ws)
    assert ws.device_error() == 0
    return m.to_host()


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("S", [16, 1, 7, 32])
@pytest.mark.parametrize("via", ["coo", "csr"])
def test_swtcf_bit_exact_vs_oracle(gpu, oracle, name, g, S, via):
    """Both entry points: COO (full key sort) and CSR (rows in order, so only
    the window digits are sorted)."""
    dst, src = g.coo()
    want = oracle.swtcf_convert(g.rows, g.cols, dst, src, S=S)
    got = gpu_swtcf(g, S, via=via)
    assert got["T"] == want["T"] and got["R"] == want["R"]
    for k in SWTCF_KEYS:
        np.testing.assert_array_equal(got[k], want[k], err_msg=f"{name} S={S} {k}")


def test_swtcf_csr_entry_and_determinism(gpu):
    g = G.rmat(13, 16 << 13, seed=11)
    a = gpu_swtcf(g, via="coo")
    b = gpu_swtcf(g, via="csr")
    c = gpu_swtcf(g, via="coo")
    for k in SWTCF_KEYS:
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)
        np.testing.assert_array_equal(a[k], c[k], err_msg=k)


def test_swtcf_shuffled_coo(gpu, oracle):
    """COO edges in random order give the same canonical tiles."""
    g = G.rmat(14, 16 << 14, seed=12)
    dst, src = g.coo()
    perm = np.random.default_rng(3).permutation(dst.size)
    m = swtcf.SWTCFMatrix(g.rows, g.cols, g.nnz, 16)
    ws = swtcf.SWTCFConvertWorkspace(g.nnz, g.cols, 16)
    swtcf.convert_coo(u32(dst[perm]), u32(src[perm]), m, ws)
    assert ws.device_error() == 0
    got = m.to_host()
    want = oracle.swtcf_convert(g.rows, g.cols, dst, src)
    for k in SWTCF_KEYS:
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)


def test_swtcf_device_errors(gpu):
    # duplicate edge -> code 1 (the reference's bad-degree error, src/swtcf_convert.cu:186-195)
    dst = np.array([0, 1, 1, 2], np.uint32)
    src = np.array([0, 2, 2, 3], np.uint32)
    m = swtcf.SWTCFMatrix(4, 4, 4)
    ws = swtcf.SWTCFConvertWorkspace(4, 4)
    swtcf.convert_coo(u32(dst), u32(src), m, ws)
    assert ws.device_error() == 1
    # out-of-range index -> code 5, and the call stays in bounds
    swtcf.convert_coo(u32(np.array([0, 9], np.uint32)), u32(np.array([1, 1], np.uint32)), m, ws)
    assert ws.device_error() == 5
    # a clean conversion clears the word
    swtcf.convert_coo(u32(np.array([0, 1], np.uint32)), u32(np.array([1, 1], np.uint32)), m, ws)
    assert ws.device_error() == 0
    # host-side argument errors, as the reference's runtime_error
    from tcc_b200._lib import TccError
    with pytest.raises(TccError):
        swtcf.SWTCFMatrix(4, 0, 4)
    with pytest.raises(TccError):
        swtcf.convert_coo(u32(np.zeros(5, np.uint32)), u32(np.zeros(5, np.uint32)), m, ws)


@pytest.mark.parametrize("name,g", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("kind", ["bcsr", "bcsc"])
def test_tiles_bit_exact_vs_oracle(gpu, oracle, name, g, kind):
    rp, col = csr_dev(g)
    t = tiles.from_csr(rp, col, g.rows, g.cols, kind=kind)
    got = t.to_host()
    want = oracle.bcsr_from_csr(g) if kind == "bcsr" else oracle.bcsc_from_csr(g)
    assert got["num_TCBlocks"] == want["num_TCBlocks"]
    T = want["num_TCBlocks"]
    for k in want:
        if isinstance(want[k], np.ndarray):
            n = want[k].size
            if k in ("sparseA2B", "sparseA2C"):
                n = 8 * T
            elif k == "tcLocalBit":
                n = T
            np.testing.assert_array_equal(got[k][:n], want[k][:n], err_msg=f"{name} {kind} {k}")


def test_tiles_reject_duplicates(gpu):
    rp = torch.tensor([0, 2, 3], dtype=torch.int64, device="cuda")
    col = u32(np.array([1, 1, 0], np.uint32))
    from tcc_b200._lib import TccError
    with pytest.raises(TccError, match="duplicate"):
        tiles.from_csr(rp, col, 2, 2)


@pytest.mark.parametrize("name,g", [c for c in CASES if c[1].nnz < (1 << 20)],
                         ids=[c[0] for c in CASES if c[1].nnz < (1 << 20)])
def test_swtcf_vs_reference_converter(gpu, oracle, name, g):
    """Reference convertCOOToSWTCF (built from source) -> canonical form == ours."""
    if oracle.ref_lib() is None:
        pytest.fail("oracle/_ref/libtcc_ref.so missing: run `make -C oracle ref` before shipping")
    dst, src = g.coo()
    ref = oracle.ref_swtcf_convert(g.rows, g.cols, dst, src)
    assert ref["device_error"] == 0
    ok, why = oracle.swtcf_validate(ref, dst, src)
    assert ok, why
    canon = oracle.swtcf_canonicalize(ref)
    got = gpu_swtcf(g)
    for k in SWTCF_KEYS:
        np.testing.assert_array_equal(got[k], canon[k], err_msg=f"{name} {k}")
