"""Batch sharding across ranks with dropout masks identical to the unsharded run.

The dropout counter of element (b, i, j) is seed + offset + (b*S_q + i)*S_kv + j
(sdpa/sdpa_utils.cuh:13-19), affine in b.  A rank that owns batch rows
[b0, b1) and indexes them locally from 0 passes
offset' = offset + b0*S_q*S_kv (mod 2^64) and gets bit-identical masks.
"""
from __future__ import annotations

M64 = (1 << 64) - 1


def shard_rows(B: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [b0, b1) of B rows for `rank` of `world` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    b0 = B * rank // world
    b1 = B * (rank + 1) // world
    return b0, b1


def shard_offset(offset: int, b0: int, S_q: int, S_kv: int) -> int:
    """Dropout offset for a shard whose first (local 0) row is global row b0."""
    return (int(offset) + int(b0) * int(S_q) * int(S_kv)) & M64


def advance_offset(offset: int, B: int, S_q: int, S_kv: int) -> int:
    """Offset for the next training step, as mha.py:162-165 advances it (+ B*S_q*S_kv)."""
    return (int(offset) + int(B) * int(S_q) * int(S_kv)) & M64
