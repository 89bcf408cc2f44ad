"""Head-strided [B, S, H, D] entry points (needs a B200).

sdpa_b200_fwd_bshd / _bwd_bshd read and write the multi-head layout in place.
They run the same kernels and arithmetic as the folded [B*H, S, D] calls, so
every output must equal, bit for bit, a folded call on the tensors the
reference's MHA builds by transposing (mha.py:103-129, heads innermost),
including the dropout masks.
"""
import importlib

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

fa = importlib.import_module("tf-custom-flash-attention_b200")


def fold(x):  # [B, S, H, D] -> [B*H, S, D]
    B, S, H, D = x.shape
    return x.permute(0, 2, 1, 3).reshape(B * H, S, D).contiguous()


def unfold(x, B, H):  # [B*H, S, D] -> [B, S, H, D]
    return x.reshape(B, H, x.shape[1], x.shape[2]).permute(0, 2, 1, 3)


@pytest.mark.parametrize("dtype,B,H,S_q,S_kv,D_qk,D_v,causal,p", [
    (torch.float16, 2, 4, 256, 256, 128, 128, True, 0.1),    # tcgen05 path
    (torch.float16, 3, 2, 200, 200, 64, 64, True, 0.0),      # ragged rows, causal edge
    (torch.float16, 2, 3, 130, 333, 64, 128, False, 0.2),    # D_qk != D_v, S_q != S_kv
    (torch.float16, 1, 5, 96, 96, 32, 32, False, 0.1),       # tcgen05 path, D = 32 (zero-filled to 64)
    (torch.float16, 1, 3, 64, 64, 12, 20, False, 0.1),       # SIMT path (rows not 16-byte multiples)
    (torch.float32, 2, 2, 70, 150, 64, 64, False, 0.05),     # fp32, 3xTF32 tensor-core path
    (torch.float32, 1, 2, 96, 96, 100, 36, True, 0.1),       # fp32, D_qk > 64: 3xTF32 forward, GEMM-route backward
    (torch.float32, 1, 2, 40, 40, 6, 10, False, 0.0),        # fp32 SIMT path
])
def test_bshd_equals_folded_bitwise(dtype, B, H, S_q, S_kv, D_qk, D_v, causal, p):
    g = torch.Generator(device="cuda").manual_seed(B * 100 + H)
    q = torch.randn(B, S_q, H, D_qk, generator=g, device="cuda").to(dtype)
    k = torch.randn(B, S_kv, H, D_qk, generator=g, device="cuda").to(dtype)
    v = torch.randn(B, S_kv, H, D_v, generator=g, device="cuda").to(dtype)
    do = torch.randn(B, S_q, H, D_v, generator=g, device="cuda").to(dtype)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o4, s4 = fa.sdpa_bshd(q, k, v, 11, 77, **kw)
    o3, s3 = fa.sdpa(fold(q), fold(k), fold(v), 11, 77, **kw)
    assert torch.equal(o4, unfold(o3, B, H))
    assert torch.equal(s4.reshape(B * H, S_q), s3)
    g4 = fa.sdpa_grad_bshd(q, k, v, o4, s4, do, 11, 77, dropout=p, scale=D_qk ** -0.5, causal_mask=causal)
    g3 = fa.sdpa_grad(fold(q), fold(k), fold(v), o3, s3, fold(do), 11, 77, dropout=p, scale=D_qk ** -0.5,
                      causal_mask=causal)
    for a, b in zip(g4, g3):
        assert torch.equal(a, unfold(b, B, H))


def test_bshd_stats_gradient_matches_folded():
    B, H, S, D = 2, 2, 128, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v, do = (torch.randn(B, S, H, D, generator=g, device="cuda").half() for _ in range(4))
    ds = torch.randn(B, H, S, generator=g, device="cuda")
    o4, s4 = fa.sdpa_bshd(q, k, v, 1, 2, scale=0.125)
    g4 = fa.sdpa_grad_bshd(q, k, v, o4, s4, do, 1, 2, scale=0.125, d_stats=ds)
    o3, s3 = fa.sdpa(fold(q), fold(k), fold(v), 1, 2, scale=0.125)
    g3 = fa.sdpa_grad(fold(q), fold(k), fold(v), o3, s3, fold(do), 1, 2, scale=0.125,
                      d_stats=ds.reshape(B * H, S))
    for a, b in zip(g4, g3):
        assert torch.equal(a, unfold(b, B, H))


def test_mha_strided_path_equals_transposing_path():
    """MHA on [B, S, F] (strided kernels) equals autograd.sdpa on the transposed heads, forward and backward."""
    B, S, H, Dh = 2, 192, 4, 64
    torch.manual_seed(5)
    x = [torch.randn(B, S, H * Dh, device="cuda").half().requires_grad_() for _ in range(3)]
    m = fa.MHA(num_heads=H, dropout=0.1, seed=9, causal_mask=True).cuda().train()
    out = m(*x)
    torch.cuda.synchronize()
    assert fa.device_status() == 0
    assert m.offset == fa.sharding.advance_offset(0, B * H, S, S)
    go = torch.randn_like(out)
    out.backward(go)
    grads = [t.grad.clone() for t in x]
    y = [t.detach().clone().requires_grad_() for t in x]
    f = [fold(t.reshape(B, S, H, Dh)) for t in y]
    o3 = fa.autograd.sdpa(*f, 9, 0, 0.1, Dh ** -0.5, True)
    ref = unfold(o3, B, H).reshape(B, S, H * Dh)
    ref.backward(go)
    assert torch.equal(out, ref)
    for a, t in zip(grads, y):
        assert torch.equal(a, t.grad)
