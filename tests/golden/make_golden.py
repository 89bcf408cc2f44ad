"""Generates the committed golden vectors in tests/golden/ from the reference itself.

  python tests/golden/make_golden.py            # CPU op  -> ref_cpu_<case>.npz, rng_kat.npz
  python tests/golden/make_golden.py --gpu      # GPU op  -> ref_gpu_<case>.npz (run on a B200 box)

Outputs come from the reference's OWN op sources (sdpa/sdpa_cpu.cc and, with
--gpu, sdpa/sdpa_fwd.cu.cc + sdpa/sdpa_bwd.cu.cc for sm_100a), built
unmodified by oracle/build_ref.sh and driven through their registered
OpKernels.  RNG known answers follow test.py:33-46 with Python big integers.
Inputs are stored in the fixtures, so the files are self-contained.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import dense, ref  # noqa: E402

# name: (dtype, B, S_q, S_kv, D_qk, D_v, causal, dropout, scale, seed, offset, std, loss)
CASES = {
    # BASELINE configs[0] shrunk in B and S: fp32, D_v=4, dropout .2, loss = sum(max(o,-1))
    "cfg1_small": ("f32", 2, 64, 64, 32, 4, False, 0.2, 32 ** -0.5, 42, 1000, 1.0, "summax"),
    "f16_causal_d64": ("f16", 2, 80, 80, 64, 64, True, 0.0, 1 / 8, 0, 0, 1.0, "normal"),
    "f16_causal_dropout_d128": ("f16", 2, 96, 96, 128, 128, True, 0.1, 128 ** -0.5, 7, 0, 1.0, "normal"),
    "f32_cross_d64_dv128": ("f32", 2, 40, 136, 64, 128, False, 0.05, 1 / 8, 3, 77, 0.5, "normal"),
    "f16_ragged_wrap": ("f16", 3, 17, 33, 40, 24, False, 0.3, 0.2, (1 << 64) - 3, (1 << 63) + 5, 1.0, "normal"),
    "f16_single": ("f16", 1, 1, 1, 8, 8, False, 0.0, 1.0, 0, 0, 1.0, "normal"),
    "f32_odd_d5_dv3": ("f32", 2, 50, 50, 5, 3, True, 0.25, 0.4, 11, 12, 1.0, "normal"),
    "f16_nondiv_d100": ("f16", 1, 130, 130, 100, 72, True, 0.0, 0.1, 0, 0, 1.0, "normal"),
}


def make_inputs(name):
    dt, B, S_q, S_kv, D_qk, D_v, causal, p, scale, seed, offset, std, loss = CASES[name]
    npdt = np.float16 if dt == "f16" else np.float32
    rng = np.random.default_rng(sum(map(ord, name)))
    q = (rng.standard_normal((B, S_q, D_qk)) * std).astype(npdt)
    k = (rng.standard_normal((B, S_kv, D_qk)) * std).astype(npdt)
    v = (rng.standard_normal((B, S_kv, D_v)) * std).astype(npdt)
    return q, k, v


def d_out(name, o):
    loss = CASES[name][-1]
    if loss == "summax":
        # d/dO of sum(reduce_max(o, -1)): one-hot at each row's first argmax
        g = np.zeros_like(o)
        idx = np.argmax(o, axis=-1)
        np.put_along_axis(g, idx[..., None], 1, axis=-1)
        return g
    rng = np.random.default_rng(1 + sum(map(ord, name)))
    return rng.standard_normal(o.shape).astype(o.dtype)


def rng_kat():
    pts = []
    for seed, offset in [(42, 1000), (7, 0), (0, 0), ((1 << 64) - 3, (1 << 63) + 5), (123456789, 987654321)]:
        for (b, i, j, S_q, S_kv) in [(0, 0, 0, 400, 400), (19, 399, 399, 400, 400), (3, 5, 7, 17, 33),
                                     (31, 8191, 8190, 8192, 8192), (127, 511, 4095, 512, 4096)]:
            pts.append((seed, offset, b, i, j, S_q, S_kv))
    arr = np.array(pts, dtype=np.uint64)
    u = np.array([dense.get_random_float(*p) for p in pts], dtype=np.float32)
    return arr, u


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpu", action="store_true")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    if not a.gpu:
        pts, u = rng_kat()
        np.savez_compressed(os.path.join(a.out, "rng_kat.npz"), points=pts, u=u)
    for name, c in CASES.items():
        dt, B, S_q, S_kv, D_qk, D_v, causal, p, scale, seed, offset, std, loss = c
        q, k, v = make_inputs(name)
        kw = dict(scale=scale, dropout=p, causal_mask=causal)
        if a.gpu:
            import torch

            tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
            o, s = ref.ref_sdpa(tq, tk, tv, seed, offset, device="GPU", **kw)
            do = d_out(name, o.cpu().numpy())
            g = ref.ref_sdpa_grad(tq, tk, tv, o, s, torch.from_numpy(do).cuda(), seed, offset, device="GPU", **kw)
            torch.cuda.synchronize()
            o, s = o.cpu().numpy(), s.cpu().numpy()
            dq, dk, dv = (x.cpu().numpy() for x in g)
            fn = f"ref_gpu_{name}.npz"
        else:
            o, s = ref.ref_sdpa(q, k, v, seed, offset, **kw)
            do = d_out(name, o)
            dq, dk, dv = ref.ref_sdpa_grad(q, k, v, o, s, do, seed, offset, **kw)
            fn = f"ref_cpu_{name}.npz"
        np.savez_compressed(os.path.join(a.out, fn), q=q, k=k, v=v, d_o=do, o=o, stats=s, dq=dq, dk=dk, dv=dv,
                            causal=causal, dropout=np.float32(p), scale=np.float32(scale),
                            seed=np.uint64(seed), offset=np.uint64(offset))
        print("wrote", fn)


if __name__ == "__main__":
    main()
