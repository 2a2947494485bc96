"""Build libpentanet_b200.so in place (sm_100a only).

    python pentanet-v1.0_b200/build.py

Compiles csrc/pn_lib.cu (one translation unit holding every kernel and the C
ABI) with nvcc for sm_100a.  The .so lands next to this file, so it travels
with the source tree; nothing is installed anywhere else.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "libpentanet_b200.so")
SOURCES = ["csrc/pn_lib.cu"]
DEPS = ["csrc/pn_common.cuh", "csrc/pn_internal.h", "csrc/pn_pack.cu", "csrc/pn_act.cu", "csrc/pn_norm.cu",
        "csrc/pn_dqmm.cu", "csrc/pn_simt.cu", "csrc/pn_gemv.cu", "csrc/pn_capi.cu", "csrc/pn_static_ws.cu", "csrc/pn_peer.cu", "csrc/pn_i8w.cu", "csrc/pn_ternary2.cu",
        "csrc/pn_lib.cu", "../include/pentanet_b200.h"]

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(os.path.join(HERE, d)) <= t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-o", tmp,
           *[os.path.join(HERE, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=HERE)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
