"""Builds libsdpa_b200.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python tf-custom-flash-attention_b200/build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libsdpa_b200.so")
SOURCES = [os.path.join(HERE, "csrc", f) for f in ("api.cu",)]
DEPS = SOURCES + [os.path.join(HERE, "csrc", f) for f in ("common.cuh", "ptx.cuh", "simt.cuh", "fwd_tc.cuh",
                                                          "bwd_tc.cuh")] + [
    os.path.join(os.path.dirname(HERE), "include", "sdpa_b200.h")]
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
FLAGS = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-Xcompiler", "-fPIC",
         "-shared", "-Xptxas", "-v"]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in DEPS if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *FLAGS, "-o", LIB + ".tmp", *SOURCES, "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libsdpa_b200.so")
    os.replace(LIB + ".tmp", LIB)
    with open(os.path.join(HERE, "ptxas_info.txt"), "w") as f:
        f.write(r.stderr)
    if verbose:
        print(r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
