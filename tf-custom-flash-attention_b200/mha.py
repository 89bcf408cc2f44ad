"""Multi-head attention layer over the sdpa op (torch mirror of the reference's Keras `MHA`).

Follows mha.py:32-178 of the reference: the feature axis is split into
`num_heads` heads, the (batch..., head) axes are folded into the op's batch
axis with heads innermost (so the dropout counter of folded row b*H + h is the
reference's), `scale = 1/sqrt(head_dim)`, and while training the dropout
offset advances by B*H*S_q*S_kv per call (mha.py:162-165) so successive steps
draw fresh masks; evaluation uses dropout 0 and offset 0 (mha.py:150-155).

Where the sequence axis is second to last and the feature axis last (the usual
[..., S, d_model]), splitting the features into heads is a free view
[B, S, H, Dh] and the layer calls the head-strided kernels (autograd.sdpa_bshd)
directly: no transposes in either direction.  Other axis orders take the
transposing path above.  Both give the same results and dropout masks.
"""
from __future__ import annotations

import torch

from . import autograd, sharding


class MHA(torch.nn.Module):
    def __init__(self, num_heads: int = 1, seq_axis: int = -2, feature_axis: int = -1, dropout: float = 0.0,
                 seed: int = 42, causal_mask: bool = False):
        super().__init__()
        self.num_heads = num_heads
        self.seq_axis = seq_axis
        self.feature_axis = feature_axis
        self.dropout = dropout
        self.seed = seed
        self.causal_mask = causal_mask
        self.offset = 0  # uint64 counter, advanced per training call

    def _axes(self, rank: int):
        s_ax = self.seq_axis % rank
        f_ax = self.feature_axis % rank
        if s_ax == f_ax:
            raise ValueError("seq_axis and feature_axis must differ")
        return s_ax, f_ax

    def _split(self, x: torch.Tensor, s_ax: int, f_ax: int):
        """[..., S, ..., H*Dh, ...] -> [prod(batch)*H, S, Dh] (heads innermost), plus the batch shape."""
        d_model = x.shape[f_ax]
        if d_model % self.num_heads:
            raise ValueError(f"num_heads {self.num_heads} does not divide the feature size {d_model}")
        head_dim = d_model // self.num_heads
        x = x.unflatten(f_ax, (self.num_heads, head_dim))          # rank + 1
        s_ax2 = s_ax if s_ax < f_ax else s_ax + 1
        h_ax, d_ax = f_ax, f_ax + 1
        batch = [i for i in range(x.dim()) if i not in (s_ax2, h_ax, d_ax)]
        x = x.permute(*batch, h_ax, s_ax2, d_ax)                   # (batch..., H, S, Dh)
        bshape = x.shape[:-3]
        return x.reshape(-1, x.shape[-2], x.shape[-1]).contiguous(), bshape, head_dim

    def _forward_strided(self, q, k, v):
        """[..., S, H*Dh] inputs viewed as [B, S, H, Dh]: no copies."""
        def view(x):
            if x.shape[-1] % self.num_heads:
                raise ValueError(f"num_heads {self.num_heads} does not divide the feature size {x.shape[-1]}")
            x = x.contiguous()
            return x.reshape(-1, x.shape[-2], self.num_heads, x.shape[-1] // self.num_heads)
        q4, k4, v4 = view(q), view(k), view(v)
        scale = 1.0 / float(q4.shape[-1]) ** 0.5
        if self.training:
            dropout, offset = self.dropout, self.offset
        else:
            dropout, offset = 0.0, 0
        o4 = autograd.sdpa_bshd(q4, k4, v4, self.seed, offset, dropout, scale, self.causal_mask)
        if self.training:
            self.offset = sharding.advance_offset(self.offset, q4.shape[0] * self.num_heads, q4.shape[1], k4.shape[1])
        return o4.reshape(*q.shape[:-1], o4.shape[2] * o4.shape[3])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        if not (q.dim() == k.dim() == v.dim()):
            raise ValueError("q, k, v should have the same rank")
        rank = q.dim()
        s_ax, f_ax = self._axes(rank)
        if s_ax == rank - 2 and f_ax == rank - 1 and q.shape[:-2] == k.shape[:-2] == v.shape[:-2]:
            return self._forward_strided(q, k, v)
        q3, bshape, head_dim = self._split(q, s_ax, f_ax)
        k3, _, _ = self._split(k, s_ax, f_ax)
        v3, _, head_dim_v = self._split(v, s_ax, f_ax)
        scale = 1.0 / float(head_dim) ** 0.5
        if self.training:
            dropout, offset = self.dropout, self.offset
        else:
            dropout, offset = 0.0, 0
        o3 = autograd.sdpa(q3, k3, v3, self.seed, offset, dropout, scale, self.causal_mask)
        if self.training:
            self.offset = sharding.advance_offset(self.offset, q3.shape[0], q3.shape[1], k3.shape[1])
        # (B*H, S_q, Dv) -> (batch..., H, S_q, Dv) -> original axis order with features merged
        o = o3.reshape(*bshape, self.num_heads, q3.shape[1], head_dim_v)
        nb = len(bshape)
        # current axes: batch (0..nb-1), H (nb), S (nb+1), Dv (nb+2); rebuild the input order
        order_in = []  # for each output axis of the unsplit rank, the source axis
        b_iter = iter(range(nb))
        for ax in range(rank):
            if ax == s_ax:
                order_in.append(nb + 1)
            elif ax == f_ax:
                order_in.append(-1)  # placeholder for (H, Dv)
            else:
                order_in.append(next(b_iter))
        perm = []
        for src in order_in:
            perm.extend([nb, nb + 2] if src == -1 else [src])
        o = o.permute(*perm)
        return o.flatten(f_ax, f_ax + 1)
