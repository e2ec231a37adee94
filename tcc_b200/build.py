"""Build tcc_b200/libtcc_b200.so (sm_100a) in-tree with nvcc.

    python -m tcc_b200.build [--verbose-ptxas]

Objects go to tcc_b200/_build/ and are rebuilt only when a source or header is
newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtcc_b200.so")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         f"-I{os.path.join(ROOT, 'include')}", "--expt-relaxed-constexpr"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(ROOT, "include", "tcc_b200.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    if not force and not verbose_ptxas and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        results = list(ex.map(compile_one, _sources()))
    if verbose_ptxas:
        for _, err in results:
            sys.stderr.write(err)
    objs = [o for o, _ in results]
    tmp = LIB + ".tmp"
    r = subprocess.run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--exclude-libs,ALL", "-o", tmp, *objs],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="--verbose-ptxas" in sys.argv, force="--force" in sys.argv))
