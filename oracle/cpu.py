"""ctypes driver for sdpa_oracle.c (test infrastructure only).

The C file restates the reference's GPU algorithm (sdpa/sdpa_fwd.cu.cc,
sdpa/sdpa_bwd.cu.cc, RNG of sdpa/sdpa_utils.cuh:13-19); see its header.
Arrays are numpy float16 / float32, C-contiguous [B, S, D].
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")

_lib = None


def build() -> None:
    subprocess.run(["bash", os.path.join(HERE, "build.sh")], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB):
        build()
    L = ctypes.CDLL(LIB)
    vp, i64, u64, f32, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_int
    L.oracle_set_threads.argtypes = [ci]
    L.oracle_rng_uniform.argtypes = [u64] * 7
    L.oracle_rng_uniform.restype = f32
    L.oracle_dropout_mask.argtypes = [u64, u64, i64, i64, i64, f32, vp]
    L.oracle_fwd_tile_kv.argtypes = [i64, i64]
    L.oracle_fwd_tile_kv.restype = ci
    L.oracle_sdpa_fwd.argtypes = [ci, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, f32, ci, u64, u64, ci]
    L.oracle_sdpa_bwd.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, f32, ci,
                                  u64, u64]
    L.oracle_set_threads(os.cpu_count() or 1)
    _lib = L
    return L


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float16:
        return 0
    if a.dtype == np.float32:
        return 1
    raise TypeError(a.dtype)


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def rng_uniform(seed, offset, b, i, j, S_q, S_kv) -> float:
    m = (1 << 64) - 1
    return float(lib().oracle_rng_uniform(seed & m, offset & m, b, i, j, S_q, S_kv))


def dropout_mask(seed, offset, B, S_q, S_kv, rate) -> np.ndarray:
    """uint8 [B,S_q,S_kv], 1 where the element is dropped."""
    m = np.zeros((B, S_q, S_kv), dtype=np.uint8)
    M = (1 << 64) - 1
    lib().oracle_dropout_mask(seed & M, offset & M, B, S_q, S_kv, float(rate), _p(m))
    return m


def fwd_tile_kv(D_qk, D_v) -> int:
    return int(lib().oracle_fwd_tile_kv(D_qk, D_v))


def sdpa(q, k, v, seed, offset, *, scale=1.0, dropout=0.0, causal_mask=False, tile_kv=0):
    """(output [B,S_q,D_v], stats [B,S_q] float32) per the reference GPU forward."""
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    o = np.zeros((B, S_q, D_v), dtype=q.dtype)
    s = np.zeros((B, S_q), dtype=np.float32)
    M = (1 << 64) - 1
    lib().oracle_sdpa_fwd(_dt(q), _p(q), _p(k), _p(v), _p(o), _p(s), B, S_q, S_kv, D_qk, D_v, float(scale),
                          float(dropout), int(bool(causal_mask)), seed & M, offset & M, int(tile_kv))
    return o, s


def sdpa_grad(q, k, v, out, stats, d_o, seed, offset, *, dropout=0.0, scale=1.0, causal_mask=False):
    """(dq, dk, dv) per the reference GPU backward (dK/dV kernel + dQ kernel)."""
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    stats = np.ascontiguousarray(stats, dtype=np.float32)
    M = (1 << 64) - 1
    lib().oracle_sdpa_bwd(_dt(q), _p(q), _p(k), _p(v), _p(out), _p(stats), _p(d_o), _p(dq), _p(dk), _p(dv), B, S_q,
                          S_kv, D_qk, D_v, float(scale), float(dropout), int(bool(causal_mask)), seed & M, offset & M)
    return dq, dk, dv
