"""The CPU oracle against the reference's own checks (CPU only).

Pins: the reference's closed-form known-answer SpMM test
(src/swtcf_spmm_main.cu:33-112) and its layout validators
(src/swtcf_convert_main.cu:36-310), both restated in oracle/tcc_oracle.c.  The
golden vectors produced by the reference build itself (tests/golden/) are
checked in tests/test_golden.py.
"""
import numpy as np
import pytest

from tcc_b200 import graphs as G


def small_graphs():
    yield "uniform-512", G.uniform(512, 16, seed=0)
    yield "uniform-4096", G.config(1)["graph"]
    yield "rmat-2^12", G.rmat(12, 16 << 12, seed=1)
    yield "sbm-1456", G.sbm(1456, 50, 40000, 40.0, 1.2, seed=2)
    yield "rmat-2^10-odd", G.rmat(10, 4000, seed=5, n=1003)


@pytest.mark.parametrize("name,g", list(small_graphs()))
@pytest.mark.parametrize("S", [16, 1, 32])
def test_oracle_layout_passes_reference_validators(oracle, name, g, S):
    dst, src = g.coo()
    m = oracle.swtcf_convert(g.rows, g.cols, dst, src, S=S)
    ok, why = oracle.swtcf_validate(m, dst, src)
    assert ok, why
    # every tile is non-empty and T/R are consistent with the offsets
    assert m["T"] == m["colWindowOffset"][-1]
    assert m["R"] == m["superWindowRowOffset"][-1]
    assert np.all(m["tileLocalBit"] != 0)


def _kat_expected(dst, src, rows, F=128):
    """validateOutput of src/swtcf_spmm_main.cu:58-112, in double."""
    s = src.astype(np.uint32)
    a = ((s * np.uint32(17) + np.uint32(13)) % np.uint32(97)).astype(np.float32) * np.float32(0.001)
    b = ((s * np.uint32(29) + np.uint32(7)) % np.uint32(89)).astype(np.float32) * np.float32(1e-5)
    sa = np.zeros(rows)
    sb = np.zeros(rows)
    np.add.at(sa, dst, a.astype(np.float64))
    np.add.at(sb, dst, b.astype(np.float64))
    return sa[:, None] + sb[:, None] * np.arange(F)[None, :]


@pytest.mark.parametrize("thr,atol,rtol", [(12, 1e-2, 1e-2), (65, 2e-4, 1e-4), (0, 1e-2, 1e-2)])
def test_oracle_spmm_known_answer(oracle, thr, atol, rtol):
    g = G.rmat(12, 16 << 12, seed=1)
    dst, src = g.coo()
    m = oracle.swtcf_convert(g.rows, g.cols, dst, src)
    X = oracle.kat_features(g.cols)
    Y = oracle.swtcf_spmm(m, X, tc_threshold=thr)
    ref = _kat_expected(dst, src, g.rows)
    assert np.all(np.abs(Y - ref) <= atol + rtol * np.abs(ref))


def test_oracle_tile_spmm_matches_csr(oracle):
    g = G.rmat(11, 16 << 11, seed=3)
    X = G.features(g.cols, 64, seed=3)
    Yc = oracle.csr_spmm(g, X)
    dst, src = g.coo()
    m = oracle.swtcf_convert(g.rows, g.cols, dst, src)
    Ys = oracle.swtcf_spmm(m, X, tc_threshold=65)
    b = oracle.bcsr_from_csr(g)
    Yb = oracle.bcsr_spmm(b, X, tc_threshold=65)
    c = oracle.bcsc_from_csr(g)
    Yp = oracle.bcsc_spmm(c, X, tc_threshold=65)
    for Y in (Ys, Yb, Yp):
        assert np.linalg.norm(Y - Yc) / np.linalg.norm(Yc) < 1e-6
    # TF32 on every tile stays inside the stated TF32 bound
    Yt = oracle.bcsr_spmm(b, X, tc_threshold=0)
    assert np.linalg.norm(Yt - Yc) / np.linalg.norm(Yc) < 5e-3


def test_oracle_transposed(oracle):
    g = G.rmat(10, 4000, seed=6, n=1000)
    g = G.csr_from_pairs(*[a for a in g.coo()][::-1], 1000, 1000)  # any matrix
    X = G.features(g.rows, 16, seed=1)
    Z = oracle.csr_spmm_t(g, X)
    gt = g.transpose()
    Z2 = oracle.csr_spmm(gt, X)
    np.testing.assert_allclose(Z, Z2, rtol=1e-6, atol=1e-6)


def test_oracle_bcsr_bcsc_decode(oracle):
    rng = np.random.default_rng(0)
    r = rng.integers(0, 77, 900).astype(np.uint32)
    c = rng.integers(0, 53, 900).astype(np.uint32)
    g = G.csr_from_pairs(r, c, 77, 53)
    b = oracle.bcsr_from_csr(g)
    got = set()
    for w in range(b["num_rowWindows"]):
        for t in range(b["rowWindowOffset"][w], b["rowWindowOffset"][w + 1]):
            bm = int(b["tcLocalBit"][t])
            for i in range(8):
                for k in range(8):
                    if bm >> (i * 8 + k) & 1:
                        got.add((w * 8 + i, int(b["sparseA2B"][8 * t + k])))
    dst, src = g.coo()
    assert got == set(zip(dst.tolist(), src.tolist()))
    c = oracle.bcsc_from_csr(g)
    got = set()
    for w in range(c["num_colWindows"]):
        for t in range(c["colWindowOffset"][w], c["colWindowOffset"][w + 1]):
            bm = int(c["tcLocalBit"][t])
            for n in range(8):
                for k in range(8):
                    if bm >> (n * 8 + k) & 1:
                        got.add((int(c["sparseA2C"][8 * t + n]), w * 8 + k))
    assert got == set(zip(dst.tolist(), src.tolist()))
    # condensed indices ascending within each window; padding 0xFFFFFFFF
    idx = b["sparseA2B"].reshape(-1, 8)
    for w in range(b["num_rowWindows"]):
        seq = idx[b["rowWindowOffset"][w]:b["rowWindowOffset"][w + 1]].ravel()
        seq = seq[seq != 0xFFFFFFFF]
        assert np.all(np.diff(seq.astype(np.int64)) > 0)


def test_oracle_rejects_bad_input(oracle):
    dst = np.array([0, 1, 1], np.uint32)
    src = np.array([0, 2, 2], np.uint32)  # duplicate (1,2)
    with pytest.raises(oracle.OracleError) as e:
        oracle.swtcf_convert(4, 4, dst, src)
    assert e.value.code == 7
    with pytest.raises(oracle.OracleError) as e:
        oracle.swtcf_convert(4, 4, np.array([0], np.uint32), np.array([4], np.uint32))
    assert e.value.code == 8
    with pytest.raises(oracle.OracleError) as e:
        oracle.swtcf_convert(4, 4, np.zeros(0, np.uint32), np.zeros(0, np.uint32))
    assert e.value.code == 1


def _shuffle_ties(m, seed):
    """Emulate the reference's atomic tie orders on a canonical layout."""
    rng = np.random.default_rng(seed)
    m = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in m.items()}
    S, W, SW = m["S"], m["numColWindows"], m["numSuperWindows"]
    off, swo = m["colWindowOffset"], m["superWindowRowOffset"]
    for s in range(SW):
        rb, re_ = int(swo[s]), int(swo[s + 1])
        perm = rng.permutation(re_ - rb)           # new slot of old slot
        inv = np.argsort(perm)
        rows = m["superWindowRows"][rb:re_].copy()
        m["superWindowRows"][rb:re_] = rows[inv]
        cache = m["superWindowRowCacheSlot"][rb:re_].copy()
        m["superWindowRowCacheSlot"][rb:re_] = cache[inv]
        for c in range(32):
            v = m["superWindowCachedRowSlot"][32 * s + c]
            if v != 0xFFFFFFFF:
                m["superWindowCachedRowSlot"][32 * s + c] = perm[v]
        for w in range(s * S, min(W, (s + 1) * S)):
            tb, te = int(off[w]), int(off[w + 1])
            slots = m["tileRowSlot"][8 * tb:8 * te].copy()
            bits = m["tileLocalBit"][tb:te].view(np.uint8).reshape(-1).copy()
            valid = slots != 0xFFFFFFFF
            slots[valid] = perm[slots[valid]]
            # permute rows inside each equal-degree run
            deg = np.array([bin(x).count("1") for x in bits])
            order = np.arange(slots.size)
            n = int(valid.sum())
            i = 0
            while i < n:
                j = i
                while j < n and deg[j] == deg[i]:
                    j += 1
                order[i:j] = i + rng.permutation(j - i)
                i = j
            m["tileRowSlot"][8 * tb:8 * te] = slots[order]
            m["tileLocalBit"][tb:te] = bits[order].view(np.uint64)
    return m


def test_canonicalize_undoes_reference_tie_orders(oracle):
    g = G.rmat(11, 16 << 11, seed=9)
    dst, src = g.coo()
    m = oracle.swtcf_convert(g.rows, g.cols, dst, src)
    shuffled = _shuffle_ties(m, seed=3)
    assert not np.array_equal(shuffled["tileRowSlot"], m["tileRowSlot"])
    ok, why = oracle.swtcf_validate(shuffled, dst, src)
    assert ok, why
    c = oracle.swtcf_canonicalize(shuffled)
    for k in ("colWindowOffset", "tileLocalBit", "tileRowSlot", "superWindowRowOffset",
              "superWindowRows", "superWindowRowCacheSlot", "superWindowCachedRowSlot",
              "superWindowCachedCount"):
        np.testing.assert_array_equal(c[k], m[k], err_msg=k)
