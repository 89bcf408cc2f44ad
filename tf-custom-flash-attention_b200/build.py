"""Builds libsdpa_b200.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python tf-custom-flash-attention_b200/build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libsdpa_b200.so")
SOURCES = [os.path.join(HERE, "csrc", f) for f in ("simt_bwd_f32.cu", "simt_bwd_f16.cu", "simt_fwd_f32.cu", "simt_fwd_f16.cu",
                                                   "bwd_tc.cu", "fwd_tc.cu", "tf32_tc.cu", "api.cu")]
DEPS = SOURCES + [os.path.join(HERE, "csrc", f) for f in ("common.cuh", "ptx.cuh", "simt.cuh", "fwd_tc.cuh",
                                                          "bwd_tc.cuh", "tf32_fwd.cuh", "tf32_bwd.cuh", "tf32_gemm.cuh", "tf32_scores.cuh", "host.cuh", "simt_launch.cuh")] + [
    os.path.join(os.path.dirname(HERE), "include", "sdpa_b200.h")]
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
FLAGS = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-Xcompiler", "-fPIC",
         "-Xptxas", "-v"]
OBJ_DIR = os.path.join(HERE, "_build")


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in DEPS if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    objs = [os.path.join(OBJ_DIR, os.path.basename(src) + ".o") for src in SOURCES]
    procs = [subprocess.Popen([NVCC, *FLAGS, "-c", src, "-o", obj], stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                              text=True) for src, obj in zip(SOURCES, objs)]  # translation units in parallel
    logs = []
    for pr, src in zip(procs, SOURCES):
        out, err = pr.communicate()
        logs.append(err)
        if pr.returncode != 0:
            sys.stderr.write(out + err)
            raise RuntimeError(f"nvcc failed on {src}")
    r = subprocess.run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB + ".tmp", *objs,
                        "-lcudart"], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed linking libsdpa_b200.so")
    os.replace(LIB + ".tmp", LIB)
    with open(os.path.join(HERE, "ptxas_info.txt"), "w") as f:
        f.write("".join(logs))
    if verbose:
        print("".join(logs))
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
