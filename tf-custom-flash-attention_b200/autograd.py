"""Autograd binding: the gradient registration of the reference's Python layer.

Mirrors ``@tf.RegisterGradient("Sdpa")`` (mha.py:10-21): the backward of
``sdpa`` calls ``sdpa_grad`` with the forward's inputs, outputs and attrs;
seed and offset get no gradient, and the gradient reaching ``stats`` is
ignored (the reference drops it via ``*args``).
"""
from __future__ import annotations

import torch

from . import ops


class SdpaFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seed, offset, dropout, scale, causal_mask):
        o, s = ops.sdpa(q, k, v, seed, offset, scale=scale, dropout=dropout, causal_mask=causal_mask)
        ctx.save_for_backward(q, k, v, o, s)
        ctx.attrs = (int(ops._scalar_u64(seed, "seed")), int(ops._scalar_u64(offset, "offset")), dropout, scale,
                     causal_mask)
        ctx.mark_non_differentiable(s)
        return o, s

    @staticmethod
    def backward(ctx, d_o, _d_stats):
        q, k, v, o, s = ctx.saved_tensors
        seed, offset, dropout, scale, causal = ctx.attrs
        dq, dk, dv = ops.sdpa_grad(q, k, v, o, s, d_o.contiguous(), seed, offset, dropout=dropout, scale=scale,
                                   causal_mask=causal)
        return dq, dk, dv, None, None, None, None, None


def sdpa(q, k, v, seed, offset, dropout: float = 0.0, scale: float = 1.0, causal_mask: bool = False):
    """Differentiable attention, like mha.py:24-29 ``sdpa`` (returns the output only)."""
    o, _ = SdpaFunction.apply(q, k, v, seed, offset, dropout, scale, causal_mask)
    return o


def sdpa_with_stats(q, k, v, seed, offset, dropout: float = 0.0, scale: float = 1.0, causal_mask: bool = False):
    """Differentiable attention returning (o, stats) like test.py:14-17."""
    return SdpaFunction.apply(q, k, v, seed, offset, dropout, scale, causal_mask)
