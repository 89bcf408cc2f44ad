"""Parity at the exact shapes of the benchmark configurations, and the MHA layer's
dropout offset across training steps (needs a B200).

* cfg1: the reference's own example (test.py:141-179): fp32 q/k [20,400,32],
  v [20,400,4], dropout 0.2, seed 42, offset 1000, scale 1/sqrt(32), loss
  sum(reduce_max(o, -1)), whose gradient dO is one-hot at each row's argmax.
* cfg5: fp32 q[*,512,64], k[*,4096,64], v[*,4096,128] ~N(0, 0.5), dropout 0.05,
  scale 1/8, on a batch subset (every batch row is independent work).
* MHA in training mode: the second call's masks start where the first call's
  ended (mha.py:162-165: offset += B*H*S_q*S_kv).

Tolerances (north star): fp32 max|new - ref| <= 1e-5 * max|ref|, fp16 2e-3.
"""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu, ref  # noqa: E402

pytestmark = pytest.mark.gpu

fa = importlib.import_module("tf-custom-flash-attention_b200")
needs_ref_gpu = pytest.mark.skipif(not ref.available("GPU"), reason="oracle/_ref GPU build missing")


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def cuda(*xs):
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in xs]


def host(*xs):
    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in xs]


def argmax_onehot(o):
    """d sum(reduce_max(o, -1)) / d o: 1 at each row's maximum (first index on ties)."""
    g = np.zeros_like(o)
    idx = o.argmax(-1)
    np.put_along_axis(g, idx[..., None], 1, axis=-1)
    return g


def cfg1_inputs():
    rng = np.random.default_rng(141)
    q = rng.standard_normal((20, 400, 32)).astype(np.float32)
    k = rng.standard_normal((20, 400, 32)).astype(np.float32)
    v = rng.standard_normal((20, 400, 4)).astype(np.float32)
    return q, k, v, dict(scale=32 ** -0.5, dropout=0.2, causal_mask=False), 42, 1000


def test_cfg1_exact_shape_matches_oracle():
    q, k, v, kw, seed, offset = cfg1_inputs()
    o_ref, s_ref = cpu.sdpa(q, k, v, seed, offset, **kw)
    o, s = host(*fa.sdpa(*cuda(q, k, v), seed, offset, **kw))
    assert rel(o, o_ref) <= 1e-5, rel(o, o_ref)
    assert rel(s, s_ref) <= 1e-5, rel(s, s_ref)
    do = argmax_onehot(o_ref)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, seed, offset, **kw)
    g = host(*fa.sdpa_grad(*cuda(q, k, v, o_ref, s_ref, do), seed, offset, **kw))
    for name, a, b in zip(("dq", "dk", "dv"), g, g_ref):
        assert rel(a, b) <= 1e-5, (name, rel(a, b))


@needs_ref_gpu
def test_cfg1_exact_shape_matches_reference_gpu_op():
    q, k, v, kw, seed, offset = cfg1_inputs()
    tq, tk, tv = cuda(q, k, v)
    o_r, s_r = ref.ref_sdpa(tq, tk, tv, seed, offset, device="GPU", **kw)
    o, s = fa.sdpa(tq, tk, tv, seed, offset, **kw)
    do = torch.from_numpy(argmax_onehot(host(o_r)[0])).cuda()
    g_r = ref.ref_sdpa_grad(tq, tk, tv, o_r, s_r, do, seed, offset, device="GPU", **kw)
    g = fa.sdpa_grad(tq, tk, tv, o_r, s_r, do, seed, offset, **kw)
    for name, a, b in zip(("o", "stats", "dq", "dk", "dv"), host(o, s, *g), host(o_r, s_r, *g_r)):
        assert rel(a, b) <= 1e-5, (name, rel(a, b))


def cfg5_inputs(B=2):
    rng = np.random.default_rng(5)
    q = (rng.standard_normal((B, 512, 64)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, 4096, 64)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, 4096, 128)) * 0.5).astype(np.float32)
    do = rng.standard_normal((B, 512, 128)).astype(np.float32)
    return q, k, v, do, dict(scale=0.125, dropout=0.05, causal_mask=False)


@needs_ref_gpu
def test_cfg5_full_rows_match_reference_gpu_op():
    q, k, v, do, kw = cfg5_inputs()
    tq, tk, tv, tdo = cuda(q, k, v, do)
    o_r, s_r = ref.ref_sdpa(tq, tk, tv, 0, 0, device="GPU", **kw)
    g_r = ref.ref_sdpa_grad(tq, tk, tv, o_r, s_r, tdo, 0, 0, device="GPU", **kw)
    o, s = fa.sdpa(tq, tk, tv, 0, 0, **kw)
    g = fa.sdpa_grad(tq, tk, tv, o_r, s_r, tdo, 0, 0, **kw)
    errs = {name: rel(a, b) for name, a, b in zip(("o", "stats", "dq", "dk", "dv"), host(o, s, *g),
                                                   host(o_r, s_r, *g_r))}
    assert all(e <= 1e-5 for e in errs.values()), errs


def test_cfg5_full_rows_match_oracle():
    q, k, v, do, kw = cfg5_inputs(B=1)
    o_ref, s_ref = cpu.sdpa(q, k, v, 0, 0, **kw)
    o, s = host(*fa.sdpa(*cuda(q, k, v), 0, 0, **kw))
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 0, 0, **kw)
    g = host(*fa.sdpa_grad(*cuda(q, k, v, o_ref, s_ref, do), 0, 0, **kw))
    errs = {name: rel(a, b) for name, a, b in zip(("o", "stats", "dq", "dk", "dv"), (o, s, *g), (o_ref, s_ref, *g_ref))}
    assert all(e <= 1e-5 for e in errs.values()), errs


@pytest.mark.parametrize("layout", ["bsf", "bsxf"])
def test_mha_training_offset_advances_between_calls(layout):
    """Two training-mode calls: call n uses offset0 + n*B*H*S_q*S_kv (mha.py:162-165),
    checked bit for bit against the op called directly with that offset."""
    torch.manual_seed(2)
    H, p = 2, 0.2
    if layout == "bsf":
        shape, seq_axis, feature_axis = (2, 128, 128), -2, -1
    else:
        shape, seq_axis, feature_axis = (2, 96, 3, 64), 1, 3
    q, k, v = (torch.randn(*shape, device="cuda").half() for _ in range(3))
    m = fa.MHA(num_heads=H, dropout=p, seq_axis=seq_axis, feature_axis=feature_axis).cuda().train()
    m.seed, m.offset = 17, 1000
    outs = [m(q, k, v).detach() for _ in range(2)]
    # fold heads exactly as the layer does and call the op with each step's offset
    s_ax, f_ax = m._axes(q.dim())
    q3, _, dh = m._split(q, s_ax, f_ax)
    k3, _, _ = m._split(k, s_ax, f_ax)
    v3, _, _ = m._split(v, s_ax, f_ax)
    Bf, S = q3.shape[0], q3.shape[1]
    assert m.offset == 1000 + 2 * Bf * S * S
    for n, out in enumerate(outs):
        o3, _ = fa.sdpa(q3, k3, v3, 17, 1000 + n * Bf * S * S, scale=dh ** -0.5, dropout=p)
        if layout == "bsf":
            expect = o3.view(shape[0], H, S, dh).transpose(1, 2).reshape(shape)
        else:
            expect = o3.view(shape[0], shape[2], H, S, dh).permute(0, 3, 1, 2, 4).reshape(shape)
        assert torch.equal(out, expect), n


def test_fp32_runs_on_the_tensor_core_kernels():
    """cfg5's fp32 shapes take the 3xTF32 tcgen05 kernels (one forward launch;
    backward: D, the score pass and the dQ / dK / dV GEMMs), not the SIMT fallback."""
    assert fa.kernel_path(torch.float32, 64, 128) == "tcgen05-3xtf32"
    assert fa.kernel_path(torch.float32, 64, 128, backward=True) == "tcgen05-3xtf32"
    q, k, v, do, kw = cfg5_inputs(B=1)
    tq, tk, tv, tdo = cuda(q, k, v, do)
    o, s = fa.sdpa(tq, tk, tv, 0, 0, **kw)
    assert fa.last_launch_count() == 1
    fa.sdpa_grad(tq, tk, tv, o, s, tdo, 0, 0, **kw)
    assert fa.last_launch_count() == 5
    torch.cuda.synchronize()
