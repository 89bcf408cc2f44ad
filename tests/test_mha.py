"""The MHA layer (mirror of the reference's Keras layer, mha.py:32-178)."""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
fa = importlib.import_module("tf-custom-flash-attention_b200")


def test_split_is_heads_innermost_and_round_trips():
    m = fa.MHA(num_heads=4)
    x = torch.randn(2, 3, 10, 32)  # (batch, batch2, S, H*Dh)
    x3, bshape, hd = m._split(x, 2, 3)
    assert x3.shape == (2 * 3 * 4, 10, 8) and tuple(bshape) == (2, 3) and hd == 8
    # folded row (b, b2, h) holds head h of x[b, b2]
    assert torch.equal(x3[(1 * 3 + 2) * 4 + 3], x[1, 2, :, 24:32])


def test_offset_advances_only_in_training():
    m = fa.MHA(num_heads=2, dropout=0.1)
    m.offset = 5
    m.eval()
    assert m.offset == 5
    assert fa.sharding.advance_offset(5, 6, 7, 8) == 5 + 6 * 7 * 8


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["bsf", "bsxf"])
def test_mha_matches_dense_torch(layout):
    torch.manual_seed(0)
    H = 2
    if layout == "bsf":  # (B, S, F), seq_axis=-2, feature_axis=-1
        shape, seq_axis, feature_axis = (2, 256, 128), -2, -1
    else:                # (B, S, X, F), seq_axis=1, feature_axis=3
        shape, seq_axis, feature_axis = (2, 192, 3, 64), 1, 3
    q, k, v = (torch.randn(*shape, device="cuda").half().requires_grad_() for _ in range(3))
    m = fa.MHA(num_heads=H, seq_axis=seq_axis, feature_axis=feature_axis, causal_mask=True).cuda().eval()
    out = m(q, k, v)
    assert out.shape == q.shape
    out.float().square().sum().backward()

    qs, ks, vs = (x.detach().float().requires_grad_() for x in (q, k, v))

    def to_heads(x):  # -> (..., H, S, Dh)
        if layout == "bsf":
            B, S, F = x.shape
            return x.view(B, S, H, F // H).transpose(1, 2)
        B, S, X, F = x.shape
        return x.view(B, S, X, H, F // H).permute(0, 2, 3, 1, 4)

    def from_heads(o):
        if layout == "bsf":
            B, _, S, Dh = o.shape
            return o.transpose(1, 2).reshape(B, S, H * Dh)
        B, X, _, S, Dh = o.shape
        return o.permute(0, 3, 1, 2, 4).reshape(B, S, X, H * Dh)

    Q, K, V = to_heads(qs), to_heads(ks), to_heads(vs)
    S = Q.shape[-2]
    att = (Q @ K.transpose(-1, -2)) / Q.shape[-1] ** 0.5
    att = att.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    ref_out = from_heads(att.softmax(-1) @ V)
    ref_out.square().sum().backward()
    assert float((out.detach().float() - ref_out.detach()).abs().max() / ref_out.detach().abs().max()) < 2e-3
    for a, r in ((q.grad, qs.grad), (k.grad, ks.grad), (v.grad, vs.grad)):
        err = float((a.float() - r).abs().max() / r.abs().max())
        assert err < 2e-3, err


@pytest.mark.gpu
@pytest.mark.parametrize("p,dtype", [(0.0, torch.float16), (0.2, torch.float16), (0.2, torch.float32)])
def test_stats_gradient_extension(p, dtype):
    """d(loss on stats and o)/d(q,k,v) with differentiable_stats=True vs dense float64 autograd
    (fp16 within 2e-3, fp32 -- the 3xTF32 path -- within 1e-5)."""
    from oracle import dense

    torch.manual_seed(1)
    B, S, D = 2, 128, 64
    q, k, v = (torch.randn(B, S, D, device="cuda").to(dtype).requires_grad_() for _ in range(3))
    w = torch.randn(B, S, device="cuda")
    o, s = fa.autograd.sdpa_with_stats(q, k, v, 3, 4, p, 0.125, True, differentiable_stats=True)
    (o.float().sum() + (s * w).sum()).backward()
    keep = torch.from_numpy(dense.keep_mask(3, 4, B, S, S, p)).cuda()
    qd, kd, vd = (x.detach().double().requires_grad_() for x in (q, k, v))
    sc = (qd @ kd.transpose(1, 2)) * 0.125
    sc = sc.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    P = sc.softmax(-1)
    inv = 1 / (1 - p) if p > 1e-6 else 1.0
    od = (P * keep * inv) @ vd
    sd = torch.logsumexp(sc, -1)
    (od.sum() + (sd * w.double()).sum()).backward()
    for a, r in ((q.grad, qd.grad), (k.grad, kd.grad), (v.grad, vd.grad)):
        err = float((a.double() - r).abs().max() / r.abs().max())
        assert err < (2e-3 if dtype == torch.float16 else 1e-5), err
