"""The ctypes mirrors in tcc_b200._lib match the C structs of include/tcc_b200.h
field for field: the header is compiled with gcc (CPU only) and every
sizeof / offsetof is compared with ctypes."""
import ctypes as C
import os
import shutil
import subprocess

import pytest

from tcc_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_INC = "/usr/local/cuda/include"
MIRRORS = [(_lib.Swtcf, "tcc_swtcf"), (_lib.Bcsr, "tcc_bcsr"), (_lib.Bcsc, "tcc_bcsc"),
           (_lib.IpcHandle, "tcc_ipc_handle"), (_lib.HaloPushArgs, "tcc_halo_push_args"),
           (_lib.DistOperand, "tcc_dist_operand"), (_lib.DistStepArgs, "tcc_dist_step_args")]


def test_ctypes_structs_match_the_header(tmp_path):
    if shutil.which("gcc") is None or not os.path.exists(os.path.join(CUDA_INC, "cuda_runtime_api.h")):
        pytest.skip("gcc or the CUDA runtime header is not available")
    lines = ['#include <stdio.h>', '#include "tcc_b200.h"', "int main(void) {"]
    for cls, cname in MIRRORS:
        lines.append(f'    printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for name, _ in cls._fields_:
            lines.append(f'    printf("{cname} {name} %zu\\n", offsetof({cname}, {name}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), "-I", CUDA_INC,
                    str(src), "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    got = {}
    for line in out.splitlines():
        cname, field, value = line.split()
        got[(cname, field)] = int(value)
    for cls, cname in MIRRORS:
        assert got[(cname, "sizeof")] == C.sizeof(cls), cname
        for name, _ in cls._fields_:
            assert got[(cname, name)] == getattr(cls, name).offset, (cname, name)
