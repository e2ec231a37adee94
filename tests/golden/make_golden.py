"""Generates the golden fixtures of tests/test_golden.py from the reference itself.

Runs the UNMODIFIED reference build (oracle/_ref/libtcc_ref.so: the reference's
convertCOOToSWTCF, launchSWTCFSpMM and the spmm_cnic BCSR / BCSC kernels
compiled from the reference sources for sm_100a) on small seeded graphs and
saves its inputs and outputs as compressed .npz files.  Needs a GPU and the
reference build; the committed fixtures let the CPU-only tests pin the oracle
against the reference without either.

    python tests/golden/make_golden.py OUT_DIR
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
from tcc_b200 import graphs as G  # noqa: E402

SWTCF_KEYS = ("colWindowOffset", "tileLocalBit", "tileRowSlot", "superWindowRowOffset",
              "superWindowRows", "superWindowRowCacheSlot", "superWindowCachedRowSlot",
              "superWindowCachedCount")


def cases():
    yield "rmat-2^8", G.rmat(8, 16 << 8, seed=11)
    yield "uniform-300", G.uniform(300, 12, seed=12)
    # a hub: one heavy column window and a cached repeat row
    n = 200
    u = np.zeros(n - 1, np.uint32)
    v = np.arange(1, n, dtype=np.uint32)
    yield "star-200", G._symmetrise_with_loops(u, v, n)


def main(out):
    os.makedirs(out, exist_ok=True)
    assert O.ref_lib() is not None, "reference build oracle/_ref/libtcc_ref.so missing"
    for name, g in cases():
        dst, src = g.coo()
        ref = O.ref_swtcf_convert(g.rows, g.cols, dst, src)
        assert ref["device_error"] == 0, name
        canon = O.swtcf_canonicalize(ref)
        X = G.features(g.cols, 128, seed=5)
        # the reference SpMM on the canonical tiling (which tiles run TF32
        # depends on the tiling, and the reference converter orders rows by
        # atomic arrival), so the oracle can be compared on the same tiles
        Y = O.ref_swtcf_spmm_tiles(canon, X, tc_threshold=12)
        Y65 = O.ref_swtcf_spmm_tiles(canon, X, tc_threshold=65)
        Xc = G.features(g.cols, 64, seed=6)
        bcsr = O.bcsr_from_csr(g)
        Cr, _ = O.ref_cnic_spmm(g.rows, g.cols, Xc, bcsr=bcsr)
        bcsc = O.bcsc_from_csr(g)
        Cc, _ = O.ref_cnic_spmm(g.rows, g.cols, Xc, bcsc=bcsc)
        np.savez_compressed(
            os.path.join(out, f"{name}.npz"), rows=g.rows, cols=g.cols, rowptr=g.rowptr,
            col=g.col, X=X, Xc=Xc, swtcf_Y_thr12=Y, swtcf_Y_thr65=Y65, cnic_bcsr_C=Cr,
            cnic_bcsc_C=Cc, **{f"swtcf_{k}": canon[k] for k in SWTCF_KEYS},
            swtcf_T=canon["T"], swtcf_R=canon["R"])
        print(name, g.rows, g.nnz, "tiles", canon["T"])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
