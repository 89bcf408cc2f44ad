"""Float64 dense attention with the reference's dropout mask (test infrastructure).

Restates the semantics of the reference's dense check ``manual_attention``
(test.py:65-88) and its Python RNG ``get_random_float`` (test.py:33-46), and
adds the exact backward of the reference's forward (the dS formulas of
sdpa/sdpa_bwd.cu.cc:131-157 without the p <= 1e-6 skip).  Used as the
ground truth that both the C oracle and the CUDA kernels are compared with.
"""
from __future__ import annotations

import numpy as np

_A = 6364136223846793005
_C = 1442695040888963407
_M64 = (1 << 64) - 1


def get_random_float(seed, offset, b, i, j, stride_m, stride_n) -> float:
    """Pure-Python big-int LCG of test.py:33-46 (used for small known-answer checks)."""
    idx = b * stride_m * stride_n + i * stride_n + j
    state = (int(seed) + int(offset) + idx) & _M64
    state = (state * _A + _C) & _M64
    return float(np.float32((state >> 32) & 0xFFFFFFFF) / np.float32(4294967296.0))


def uniform_tensor(seed, offset, B, S_q, S_kv) -> np.ndarray:
    """Vectorised RNG: float32 [B,S_q,S_kv] identical to get_random_float."""
    with np.errstate(over="ignore"):
        idx = np.arange(B * S_q * S_kv, dtype=np.uint64).reshape(B, S_q, S_kv)
        state = idx + np.uint64((int(seed) + int(offset)) & _M64)
        state = state * np.uint64(_A) + np.uint64(_C)
    hi = (state >> np.uint64(32)).astype(np.uint32)
    return hi.astype(np.float32) / np.float32(4294967296.0)


def keep_mask(seed, offset, B, S_q, S_kv, rate) -> np.ndarray:
    """float64 1.0 where kept; dropout active iff rate > 1e-6 (GPU rule)."""
    if not rate > 1e-6:
        return np.ones((B, S_q, S_kv))
    u = uniform_tensor(seed, offset, B, S_q, S_kv)
    return (~(u < np.float32(rate))).astype(np.float64)


def forward(q, k, v, seed, offset, *, scale=1.0, dropout=0.0, causal_mask=False):
    """(o, stats, P, keep) in float64.  stats = m + ln(l + 1e-6) as in the reference."""
    q64, k64, v64 = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    B, S_q, _ = q64.shape
    S_kv = k64.shape[1]
    s = np.einsum("bid,bjd->bij", q64, k64) * scale
    if causal_mask:
        s = np.where(np.triu(np.ones((S_q, S_kv), dtype=bool), 1)[None], -np.inf, s)
    m = s.max(-1, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(-1, keepdims=True)
    P = e / l
    keep = keep_mask(seed, offset, B, S_q, S_kv, dropout)
    inv = 1.0 / (1.0 - dropout) if dropout > 1e-6 else 1.0
    o = np.einsum("bij,bjd->bid", P * keep * inv, v64)
    stats = (m + np.log(l + 1e-6))[..., 0]
    return o, stats, P, keep


def backward(q, k, v, d_o, seed, offset, *, scale=1.0, dropout=0.0, causal_mask=False):
    """Exact (dq, dk, dv) of the reference forward, float64."""
    q64, k64, v64, do64 = (np.asarray(x, dtype=np.float64) for x in (q, k, v, d_o))
    o, _, P, keep = forward(q, k, v, seed, offset, scale=scale, dropout=dropout, causal_mask=causal_mask)
    inv = 1.0 / (1.0 - dropout) if dropout > 1e-6 else 1.0
    Pt = P * keep * inv
    dv = np.einsum("bij,bid->bjd", Pt, do64)
    dP = np.einsum("bid,bjd->bij", do64, v64) * keep * inv
    delta = (do64 * o).sum(-1, keepdims=True)
    dS = P * (dP - delta) * scale
    dq = np.einsum("bij,bjd->bid", dS, k64)
    dk = np.einsum("bij,bid->bjd", dS, q64)
    return dq, dk, dv
