"""Host-side mirror of the reference's ``Sdpa`` / ``SdpaGrad`` ops for torch CUDA tensors.

``sdpa`` and ``sdpa_grad`` take the reference ops' inputs and attrs (names,
meaning, defaults: sdpa/sdpa_ops.cc:7-63), run the reference OpKernels'
validation with the same messages and order (SdpaFwdOp::Compute
sdpa/sdpa_cpu.cc:29-87, SdpaBwdOp::Compute sdpa/sdpa_cpu.cc:105-192), allocate
the outputs like ``allocate_output`` does, and launch the sm_100a kernels
through the C ABI on the current CUDA stream.

Failed checks raise ``InvalidArgumentError`` (TensorFlow's
``errors::InvalidArgument``).  Inputs must be CUDA tensors: there is no CPU
path (the reference's CPU kernels are not part of this library).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class InvalidArgumentError(ValueError):
    """Raised where the reference's OP_REQUIRES fails with errors::InvalidArgument."""


class KernelError(RuntimeError):
    """A non-validation failure reported by the C ABI (CUDA error, timeout)."""


_DTYPES = {torch.float16: _lib.F16, torch.float32: _lib.F32}


def _scalar_u64(x, name: str) -> int:
    if isinstance(x, torch.Tensor):
        if x.dim() != 0:
            raise InvalidArgumentError(f"{name} must be scalar")
        x = int(x.item())
    return int(x) & 0xFFFFFFFFFFFFFFFF


def _rank3(t: torch.Tensor, idx: int):
    if t.dim() != 3:
        raise InvalidArgumentError(f"Shape must be rank 3 but is rank {t.dim()} for input {idx}")


def _prep(ts):
    dt = ts[0].dtype
    if dt not in _DTYPES:
        raise InvalidArgumentError(f"T must be half or float, got {dt}")
    for t in ts:
        if not t.is_cuda:
            raise InvalidArgumentError("sdpa_b200 runs on CUDA tensors only (no CPU kernel is registered)")
        if t.dtype != dt:
            raise InvalidArgumentError("all floating-point inputs must share dtype T")
    return [t.contiguous() for t in ts], _DTYPES[dt]


def _check(rc: int):
    if rc == _lib.OK:
        return
    if rc in (_lib.EINVAL, _lib.EUNSUPPORTED, _lib.EWORKSPACE):
        raise InvalidArgumentError(_lib.strerror(rc))
    detail = _lib.lib().sdpa_b200_last_error_detail().decode() if rc == _lib.ECUDA else ""
    raise KernelError(_lib.strerror(rc) + (f" [{detail}]" if detail else ""))


_FEATURE_MSG = ("CUDA kernel does not support feature size over 128. Set smaller feature size or use more heads")


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seed, offset, scale: float = 1.0, dropout: float = 0.0,
         causal_mask: bool = False, *, _out=None):
    """The ``Sdpa`` op: returns (output [B,S_q,D_v] T, stats [B,S_q] float32).

    ``_out`` (internal): preallocated (output, stats) to write into."""
    for i, t in enumerate((q, k, v)):
        _rank3(t, i)
    seed_v = _scalar_u64(seed, "seed")
    offset_v = _scalar_u64(offset, "offset")
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    if k.shape[0] != B:
        raise InvalidArgumentError("K batch size mismatch")
    if k.shape[2] != D_qk:
        raise InvalidArgumentError("K feature size mismatch")
    if v.shape[0] != B:
        raise InvalidArgumentError("V batch size mismatch")
    if v.shape[1] != S_kv:
        raise InvalidArgumentError("V seq size mismatch")
    if causal_mask and S_q != S_kv:
        raise InvalidArgumentError("seq size Q != K while causal_mask = True")
    if max(D_qk, D_v) > 128:
        raise InvalidArgumentError(_FEATURE_MSG)
    (q, k, v), dt = _prep([q, k, v])
    if _out is not None:
        out, stats = _out
    else:
        out = torch.empty((B, S_q, D_v), dtype=q.dtype, device=q.device)
        stats = torch.empty((B, S_q), dtype=torch.float32, device=q.device)
    if B * S_q == 0 or D_v == 0:
        return out, stats
    with torch.cuda.device(q.device):
        st = torch.cuda.current_stream().cuda_stream
        rc = _lib.lib().sdpa_b200_fwd(dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                      stats.data_ptr(), B, S_q, S_kv, D_qk, D_v, float(scale), float(dropout),
                                      int(bool(causal_mask)), seed_v, offset_v, st)
    _check(rc)
    return out, stats


def sdpa_grad(q, k, v, out, stats, do, seed, offset, dropout: float = 0.0, scale: float = 1.0,
              causal_mask: bool = False, *, d_stats=None, _out=None, _ws=None):
    """The ``SdpaGrad`` op: returns (dq, dk, dv) shaped like (q, k, v).

    ``d_stats`` (extension, not in the reference): a float32 [B, S_q] gradient
    reaching ``stats``; it is propagated as the log-sum-exp it is.
    ``_out`` / ``_ws`` (internal): preallocated (dq, dk, dv) and float32 workspace."""
    for i, t in enumerate((q, k, v)):
        _rank3(t, i)
    seed_v = _scalar_u64(seed, "seed")
    offset_v = _scalar_u64(offset, "offset")
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    checks = [
        (k.shape[0] == B, "K batch size mismatch"),
        (k.shape[2] == D_qk, "K feature size mismatch"),
        (v.shape[0] == B, "V batch size mismatch"),
        (v.shape[1] == S_kv, "V seq size mismatch"),
        (out.dim() == 3 and out.shape[0] == B, "O batch size mismatch"),
        (out.dim() == 3 and out.shape[1] == S_q, "O seq size mismatch"),
        (out.dim() == 3 and out.shape[2] == D_v, "O feature size mismatch"),
        (do.dim() == 3 and do.shape[0] == B, "dO batch size mismatch"),
        (do.dim() == 3 and do.shape[1] == S_q, "dO seq size mismatch"),
        (do.dim() == 3 and do.shape[2] == D_v, "dO feature size mismatch"),
        (stats.dim() >= 1 and stats.shape[0] == B, "S batch size mismatch"),
        (stats.dim() >= 2 and stats.shape[1] == S_q, "S seq size mismatch"),
        (not causal_mask or S_q == S_kv, "seq size Q != K while causal_mask = True"),
        (max(D_qk, D_v) <= 128, _FEATURE_MSG),
    ]
    for ok, msg in checks:
        if not ok:
            raise InvalidArgumentError(msg)
    (q, k, v, out, do), dt = _prep([q, k, v, out, do])
    if stats.dtype != torch.float32 or not stats.is_cuda:
        raise InvalidArgumentError("stats must be a float32 CUDA tensor")
    stats = stats.contiguous()
    dq, dk, dv = _out if _out is not None else (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))
    L = _lib.lib()
    ws_bytes = L.sdpa_b200_bwd_workspace_bytes(dt, B, S_q, S_kv, D_qk, D_v)
    if _ws is not None and _ws.numel() * 4 >= ws_bytes:
        ws = _ws
    else:
        ws = torch.empty((max(ws_bytes, 4) + 3) // 4, dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        st = torch.cuda.current_stream().cuda_stream
        if d_stats is None:
            rc = L.sdpa_b200_bwd(dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), stats.data_ptr(),
                                 do.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S_q, S_kv, D_qk, D_v,
                                 float(scale), float(dropout), int(bool(causal_mask)), seed_v, offset_v,
                                 ws.data_ptr(), ws_bytes, st)
        else:
            d_stats = d_stats.to(torch.float32).contiguous()
            if tuple(d_stats.shape) != (B, S_q):
                raise InvalidArgumentError("d_stats must be [B, S_q]")
            rc = L.sdpa_b200_bwd_dstats(dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        stats.data_ptr(), d_stats.data_ptr(), do.data_ptr(), dq.data_ptr(),
                                        dk.data_ptr(), dv.data_ptr(), B, S_q, S_kv, D_qk, D_v, float(scale),
                                        float(dropout), int(bool(causal_mask)), seed_v, offset_v, ws.data_ptr(),
                                        ws_bytes, st)
    _check(rc)
    return dq, dk, dv


def _bshd_dims(q, k, v):
    for i, t in enumerate((q, k, v)):
        if t.dim() != 4:
            raise InvalidArgumentError(f"Shape must be rank 4 ([B, S, H, D]) but is rank {t.dim()} for input {i}")
    B, S_q, H, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[3]
    if k.shape[0] != B or v.shape[0] != B:
        raise InvalidArgumentError("K/V batch size mismatch")
    if k.shape[2] != H or v.shape[2] != H:
        raise InvalidArgumentError("K/V head count mismatch")
    if k.shape[3] != D_qk:
        raise InvalidArgumentError("K feature size mismatch")
    if v.shape[1] != S_kv:
        raise InvalidArgumentError("V seq size mismatch")
    if max(D_qk, D_v) > 128:
        raise InvalidArgumentError(_FEATURE_MSG)
    return B, H, S_q, S_kv, D_qk, D_v


def sdpa_bshd(q, k, v, seed, offset, scale: float = 1.0, dropout: float = 0.0, causal_mask: bool = False):
    """Attention over head-strided tensors (extension for the MHA layer, no reference op).

    q [B,S_q,H,D_qk], k [B,S_kv,H,D_qk], v [B,S_kv,H,D_v] -> (output [B,S_q,H,D_v],
    stats [B,H,S_q] float32), read and written in place.  Equal to ``sdpa`` on the
    [B*H,S,D] tensors mha.py:103-129 builds by transposing (heads innermost in the
    folded batch index, so the dropout masks agree too)."""
    B, H, S_q, S_kv, D_qk, D_v = _bshd_dims(q, k, v)
    if causal_mask and S_q != S_kv:
        raise InvalidArgumentError("seq size Q != K while causal_mask = True")
    (q, k, v), dt = _prep([q, k, v])
    out = torch.empty((B, S_q, H, D_v), dtype=q.dtype, device=q.device)
    stats = torch.empty((B, H, S_q), dtype=torch.float32, device=q.device)
    if B * H * S_q == 0:
        return out, stats
    with torch.cuda.device(q.device):
        st = torch.cuda.current_stream().cuda_stream
        rc = _lib.lib().sdpa_b200_fwd_bshd(dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                           stats.data_ptr(), B, H, S_q, S_kv, D_qk, D_v, float(scale),
                                           float(dropout), int(bool(causal_mask)), _scalar_u64(seed, "seed"),
                                           _scalar_u64(offset, "offset"), st)
    _check(rc)
    return out, stats


def sdpa_grad_bshd(q, k, v, out, stats, do, seed, offset, dropout: float = 0.0, scale: float = 1.0,
                   causal_mask: bool = False, *, d_stats=None):
    """Gradients (dq, dk, dv) of ``sdpa_bshd``, shaped like (q, k, v) ([B,S,H,D])."""
    B, H, S_q, S_kv, D_qk, D_v = _bshd_dims(q, k, v)
    if tuple(out.shape) != (B, S_q, H, D_v) or tuple(do.shape) != (B, S_q, H, D_v):
        raise InvalidArgumentError("O / dO must be [B, S_q, H, D_v]")
    if tuple(stats.shape) != (B, H, S_q) or stats.dtype != torch.float32:
        raise InvalidArgumentError("stats must be float32 [B, H, S_q]")
    if causal_mask and S_q != S_kv:
        raise InvalidArgumentError("seq size Q != K while causal_mask = True")
    (q, k, v, out, do), dt = _prep([q, k, v, out, do])
    stats = stats.contiguous()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    if d_stats is not None:
        d_stats = d_stats.to(torch.float32).contiguous()
        if tuple(d_stats.shape) != (B, H, S_q):
            raise InvalidArgumentError("d_stats must be [B, H, S_q]")
    L = _lib.lib()
    ws_bytes = L.sdpa_b200_bwd_workspace_bytes(dt, B * H, S_q, S_kv, D_qk, D_v)
    ws = torch.empty((max(ws_bytes, 4) + 3) // 4, dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        st = torch.cuda.current_stream().cuda_stream
        rc = L.sdpa_b200_bwd_bshd(dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), stats.data_ptr(),
                                  d_stats.data_ptr() if d_stats is not None else None, do.data_ptr(),
                                  dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, S_q, S_kv, D_qk, D_v,
                                  float(scale), float(dropout), int(bool(causal_mask)), _scalar_u64(seed, "seed"),
                                  _scalar_u64(offset, "offset"), ws.data_ptr(), ws_bytes, st)
    _check(rc)
    return dq, dk, dv


def dropout_mask(seed, offset, B: int, S_q: int, S_kv: int, dropout: float, device=None) -> torch.Tensor:
    """uint8 [B,S_q,S_kv], 1 where the kernels drop (b,i,j): the device RNG itself."""
    m = torch.empty((B, S_q, S_kv), dtype=torch.uint8, device=device or "cuda")
    if m.numel():
        st = torch.cuda.current_stream(m.device).cuda_stream
        _check(_lib.lib().sdpa_b200_dropout_mask(_scalar_u64(seed, "seed"), _scalar_u64(offset, "offset"), B, S_q,
                                                 S_kv, float(dropout), m.data_ptr(), st))
    return m


def device_status(device=None) -> int:
    """Reads and clears the device status word (bit 0: a bounded wait timed out)."""
    w = ctypes.c_uint(0)
    with torch.cuda.device(device or torch.cuda.current_device()):
        rc = _lib.lib().sdpa_b200_device_status(ctypes.byref(w), torch.cuda.current_stream().cuda_stream)
    if rc not in (_lib.OK, _lib.ETIMEOUT):
        _check(rc)
    return int(w.value)


def kernel_path(dtype: torch.dtype, D_qk: int, D_v: int, backward: bool = False) -> str:
    """'tcgen05' (fp16), 'tcgen05-3xtf32' (fp32) or 'simt': which kernel family serves this shape."""
    return {1: "tcgen05", 2: "tcgen05-3xtf32"}.get(_lib.lib().sdpa_b200_path(_DTYPES[dtype], D_qk, D_v, int(backward)),
                                                   "simt")


def last_launch_count() -> int:
    return int(_lib.lib().sdpa_b200_last_launch_count())
