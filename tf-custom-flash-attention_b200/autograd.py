"""Autograd binding: the gradient registration of the reference's Python layer.

Mirrors ``@tf.RegisterGradient("Sdpa")`` (mha.py:10-21): the backward of
``sdpa`` calls ``sdpa_grad`` with the forward's inputs, outputs and attrs;
seed and offset get no gradient, and the gradient reaching ``stats`` is
ignored (the reference drops it via ``*args``) unless the caller asks for
it with ``sdpa_with_stats(..., differentiable_stats=True)`` (an extension).
"""
from __future__ import annotations

import torch

from . import ops


class SdpaFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seed, offset, dropout, scale, causal_mask, differentiable_stats=False):
        o, s = ops.sdpa(q, k, v, seed, offset, scale=scale, dropout=dropout, causal_mask=causal_mask)
        ctx.save_for_backward(q, k, v, o, s)
        ctx.attrs = (int(ops._scalar_u64(seed, "seed")), int(ops._scalar_u64(offset, "offset")), dropout, scale,
                     causal_mask)
        ctx.stats_grad = bool(differentiable_stats)
        if not ctx.stats_grad:
            ctx.mark_non_differentiable(s)
        return o, s

    @staticmethod
    def backward(ctx, d_o, d_stats):
        q, k, v, o, s = ctx.saved_tensors
        seed, offset, dropout, scale, causal = ctx.attrs
        if d_o is None:
            d_o = torch.zeros_like(o)
        dq, dk, dv = ops.sdpa_grad(q, k, v, o, s, d_o.contiguous(), seed, offset, dropout=dropout, scale=scale,
                                   causal_mask=causal, d_stats=d_stats if ctx.stats_grad else None)
        return dq, dk, dv, None, None, None, None, None, None


class SdpaBSHDFunction(torch.autograd.Function):
    """Same gradient registration over head-strided [B,S,H,D] tensors (ops.sdpa_bshd)."""

    @staticmethod
    def forward(ctx, q, k, v, seed, offset, dropout, scale, causal_mask):
        o, s = ops.sdpa_bshd(q, k, v, seed, offset, scale=scale, dropout=dropout, causal_mask=causal_mask)
        ctx.save_for_backward(q, k, v, o, s)
        ctx.attrs = (int(ops._scalar_u64(seed, "seed")), int(ops._scalar_u64(offset, "offset")), dropout, scale,
                     causal_mask)
        return o

    @staticmethod
    def backward(ctx, d_o):
        q, k, v, o, s = ctx.saved_tensors
        seed, offset, dropout, scale, causal = ctx.attrs
        dq, dk, dv = ops.sdpa_grad_bshd(q, k, v, o, s, d_o.contiguous(), seed, offset, dropout=dropout, scale=scale,
                                        causal_mask=causal)
        return dq, dk, dv, None, None, None, None, None


def sdpa_bshd(q, k, v, seed, offset, dropout: float = 0.0, scale: float = 1.0, causal_mask: bool = False):
    """Differentiable attention over [B,S,H,D] tensors (no head transposes); returns [B,S_q,H,D_v]."""
    return SdpaBSHDFunction.apply(q, k, v, seed, offset, dropout, scale, causal_mask)


def sdpa(q, k, v, seed, offset, dropout: float = 0.0, scale: float = 1.0, causal_mask: bool = False):
    """Differentiable attention, like mha.py:24-29 ``sdpa`` (returns the output only)."""
    o, _ = SdpaFunction.apply(q, k, v, seed, offset, dropout, scale, causal_mask)
    return o


def sdpa_with_stats(q, k, v, seed, offset, dropout: float = 0.0, scale: float = 1.0, causal_mask: bool = False,
                    differentiable_stats: bool = False):
    """Differentiable attention returning (o, stats) like test.py:14-17; with
    differentiable_stats=True a loss on stats also reaches q and k."""
    return SdpaFunction.apply(q, k, v, seed, offset, dropout, scale, causal_mask, differentiable_stats)
