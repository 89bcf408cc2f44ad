"""Host-buffer forward + backward with copies overlapped with the kernels.

`train_step_host` takes q, k, v, d_o in pinned host memory and returns
o, stats, dq, dk, dv in pinned host memory.  The batch is cut into chunks;
chunk c+1 is copied in (one stream) while chunk c is computed (another) and
chunk c-1 is copied out (a third), so PCIe traffic in both directions hides
behind the attention kernels.  Device buffers for three chunks are allocated
once per shape and reused (nothing is allocated inside the pipeline, so no
allocator call can serialise the streams).  Dropout masks equal an unchunked
call: each chunk passes the offset rebased to its first batch row
(sharding.shard_offset), as the reference's counter is affine in b.
"""
from __future__ import annotations

import threading

import torch

from . import _lib, ops, sharding

_buffers: dict = {}
_SETS = 3  # chunks in flight: copy-in, compute, copy-out


def _chunk_buffers(dev, dtype, nb, S_q, S_kv, D_qk, D_v):
    # per thread: calls from two threads (on their own streams) must not share device buffers
    key = (str(dev), dtype, nb, S_q, S_kv, D_qk, D_v, threading.get_ident())
    if key not in _buffers:
        def e(*shape, dt=dtype):
            return torch.empty(shape, dtype=dt, device=dev)

        dt_code = _lib.F16 if dtype == torch.float16 else _lib.F32
        ws_words = (max(_lib.lib().sdpa_b200_bwd_workspace_bytes(dt_code, nb, S_q, S_kv, D_qk, D_v), 4) + 3) // 4
        _buffers[key] = [dict(q=e(nb, S_q, D_qk), k=e(nb, S_kv, D_qk), v=e(nb, S_kv, D_v), do=e(nb, S_q, D_v),
                              o=e(nb, S_q, D_v), s=e(nb, S_q, dt=torch.float32), dq=e(nb, S_q, D_qk),
                              dk=e(nb, S_kv, D_qk), dv=e(nb, S_kv, D_v), ws=e(ws_words, dt=torch.float32))
                         for _ in range(_SETS)]
    return _buffers[key]


def train_step_host(q, k, v, d_o, seed, offset, *, scale=1.0, dropout=0.0, causal_mask=False, chunks=8,
                    device=None, out=None, synchronize=False):
    """(o, stats, dq, dk, dv) on pinned host memory; q, k, v, d_o pinned host [B, S, D] tensors.

    `out` may pass preallocated pinned host tensors (o, stats, dq, dk, dv) to reuse across calls.
    The call returns once the work is queued: the copies back to host memory
    complete in stream order, and the caller's current stream waits for them.
    Synchronize that stream (or pass synchronize=True) before reading the
    returned tensors on the host.  Calls from one thread reuse one set of
    device buffers, so they must be ordered on one stream (as they are when
    made from the same thread without switching streams); calls from other
    threads get their own buffers.
    """
    dev = torch.device(device or "cuda")
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    if out is None:
        out = (torch.empty((B, S_q, D_v), dtype=q.dtype, pin_memory=True),
               torch.empty((B, S_q), dtype=torch.float32, pin_memory=True),
               torch.empty_like(q, pin_memory=True), torch.empty_like(k, pin_memory=True),
               torch.empty_like(v, pin_memory=True))
    ho, hs, hdq, hdk, hdv = out
    n = max(1, min(int(chunks), B))
    bounds = [sharding.shard_rows(B, n, c) for c in range(n)]
    nb_max = max(b1 - b0 for b0, b1 in bounds)
    sets = _chunk_buffers(dev, q.dtype, nb_max, S_q, S_kv, D_qk, D_v)
    h2d, comp, d2h = (torch.cuda.Stream(device=dev) for _ in range(3))
    main = torch.cuda.current_stream(dev)
    start = torch.cuda.Event()
    start.record(main)
    for st in (h2d, comp, d2h):
        st.wait_event(start)
    copied_out = []
    for c, (b0, b1) in enumerate(bounds):
        nb = b1 - b0
        buf = sets[c % _SETS]
        view = {name: t[:nb] for name, t in buf.items() if name != "ws"}
        loaded = torch.cuda.Event()
        with torch.cuda.stream(h2d):
            if c >= _SETS:  # chunk c-3 used this buffer set: wait until its results left
                h2d.wait_event(copied_out[c - _SETS])
            for name, x in (("q", q), ("k", k), ("v", v), ("do", d_o)):
                view[name].copy_(x[b0:b1], non_blocking=True)
            loaded.record(h2d)
        computed = torch.cuda.Event()
        with torch.cuda.stream(comp):
            comp.wait_event(loaded)
            off = sharding.shard_offset(offset, b0, S_q, S_kv)
            ops.sdpa(view["q"], view["k"], view["v"], seed, off, scale=scale, dropout=dropout,
                     causal_mask=causal_mask, _out=(view["o"], view["s"]))
            ops.sdpa_grad(view["q"], view["k"], view["v"], view["o"], view["s"], view["do"], seed, off,
                          dropout=dropout, scale=scale, causal_mask=causal_mask,
                          _out=(view["dq"], view["dk"], view["dv"]), _ws=buf["ws"])
            computed.record(comp)
        done = torch.cuda.Event()
        with torch.cuda.stream(d2h):
            d2h.wait_event(computed)
            for hbuf, name in ((ho, "o"), (hs, "s"), (hdq, "dq"), (hdk, "dk"), (hdv, "dv")):
                hbuf[b0:b1].copy_(view[name], non_blocking=True)
            done.record(d2h)
        copied_out.append(done)
    main.wait_event(copied_out[-1])
    if synchronize:
        copied_out[-1].synchronize()
    return out
