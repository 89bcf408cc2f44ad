"""Seeded random shapes against the oracle (needs a B200).

Sweeps the dispatch space the hand-picked cases do not all reach: both
dtypes, every kernel family (fp16 paired / one-tile tcgen05, fp32 3xTF32 with
narrow and wide values, SIMT), ragged and tiny sequence lengths, head dims
from 4 to 128, causal and not, dropout on and off, folded and [B, S, H, D]
layouts.  Tolerances as everywhere: fp16 2e-3, fp32 1e-5 of max|ref|.
"""
import importlib
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu  # noqa: E402

pytestmark = pytest.mark.gpu

fa = importlib.import_module("tf-custom-flash-attention_b200")
TOL = {np.float16: 2e-3, np.float32: 1e-5}


def draw(i):
    r = np.random.default_rng(1000 + i)
    dt = (np.float16, np.float32)[i % 2]
    B = int(r.integers(1, 4))
    H = int(r.choice([1, 1, 2, 3]))
    causal = bool(r.random() < 0.4)
    S_q = int(r.choice([1, 7, 64, 127, 128, 129, 200, 256, 383, 520]))
    S_kv = S_q if causal else int(r.choice([1, 33, 64, 128, 130, 300, 640]))
    dims = [4, 8, 12, 16, 32, 40, 48, 64, 72, 96, 100, 128]
    D_qk, D_v = int(r.choice(dims)), int(r.choice(dims))
    p = float(r.choice([0.0, 0.0, 0.1, 0.5]))
    if S_kv == 1:
        # one key: dS = p (kf dP - D) cancels exactly (P = 1, D = kf dO.v), so dQ
        # and dK are pure rounding noise of either implementation, not results;
        # without dropout both sides produce exact zeros and are still compared.
        p = 0.0
    return dt, B, H, S_q, S_kv, D_qk, D_v, causal, p


# SDPA_B200_RANDOM_CASES widens the sweep (40 by default), SDPA_B200_RANDOM_FIRST moves it.
_FIRST = int(os.environ.get("SDPA_B200_RANDOM_FIRST", "0"))
CASES = [draw(i) for i in range(_FIRST, _FIRST + int(os.environ.get("SDPA_B200_RANDOM_CASES", "40")))]


def ident(c):
    dt, B, H, S_q, S_kv, D_qk, D_v, causal, p = c
    return f"{np.dtype(dt).name}-B{B}H{H}-{S_q}x{S_kv}-d{D_qk}v{D_v}-{'c' if causal else 'n'}-p{p}"


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("case", CASES, ids=[ident(c) for c in CASES])
def test_random_shape_matches_oracle(case):
    dt, B, H, S_q, S_kv, D_qk, D_v, causal, p = case
    rng = np.random.default_rng(S_q * 131 + S_kv * 7 + D_qk + D_v)
    std = 1.0 if dt == np.float16 else 0.5
    q = (rng.standard_normal((B * H, S_q, D_qk)) * std).astype(dt)
    k = (rng.standard_normal((B * H, S_kv, D_qk)) * std).astype(dt)
    v = (rng.standard_normal((B * H, S_kv, D_v)) * std).astype(dt)
    do = rng.standard_normal((B * H, S_q, D_v)).astype(dt)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 3, 77, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 3, 77, **kw)
    tq, tk, tv, to, ts, tdo = (torch.from_numpy(np.ascontiguousarray(x)).cuda()
                               for x in (q, k, v, o_ref, s_ref, do))
    if H == 1:
        o, s = fa.sdpa(tq, tk, tv, 3, 77, **kw)
        g = fa.sdpa_grad(tq, tk, tv, to, ts, tdo, 3, 77, **kw)
    else:  # the same rows in the [B, S, H, D] layout (row b*H + h is head h of batch b)
        def bshd(x):
            return x.reshape(B, H, x.shape[1], x.shape[2]).permute(0, 2, 1, 3).contiguous()

        def back(x):
            return x.permute(0, 2, 1, 3).reshape(B * H, x.shape[1], x.shape[3])

        o4, s3 = fa.sdpa_bshd(bshd(tq), bshd(tk), bshd(tv), 3, 77, **kw)  # stats [B, H, S_q]
        o, s = back(o4), s3.reshape(B * H, S_q)
        g4 = fa.sdpa_grad_bshd(bshd(tq), bshd(tk), bshd(tv), bshd(to), ts.reshape(B, H, S_q), bshd(tdo), 3, 77,
                               **kw)
        g = tuple(back(x) for x in g4)
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in (o, s, *g)]
    tol = TOL[dt]
    for name, a, b in zip(("o", "stats", "dq", "dk", "dv"), got, (o_ref, s_ref, *g_ref)):
        if not b.size:
            continue
        if np.abs(b).max() == 0:  # e.g. dQ with one key: exactly zero in the oracle's order of operations
            assert np.abs(a).max() <= 1e-4, (name, np.abs(a).max())
        elif name == "stats":  # log-sum-exp values: compared on the scale of 1 when all are tiny
            err = float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1.0))
            assert err <= tol, (name, err)
        else:
            assert rel(a, b) <= tol, (name, rel(a, b))
    assert fa.device_status() == 0
