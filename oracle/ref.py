"""ctypes driver for the reference's own op, built unmodified by oracle/build_ref.sh.

TEST INFRASTRUCTURE ONLY (parity oracle + CPU baseline): used by tests/,
bench.py's reference arm / cpu_baseline leg and __graft_entry__.smoke().

  ref_sdpa(...)       -> runs the reference's registered ``Sdpa`` OpKernel
                         (SdpaFwdOp, sdpa/sdpa_cpu.cc:29-87) on "CPU" or "GPU"
  ref_sdpa_grad(...)  -> runs ``SdpaGrad`` (SdpaBwdOp, sdpa/sdpa_cpu.cc:105-192)

CPU arrays are numpy; GPU arrays are torch CUDA tensors (the GPU library runs
the reference kernels of sdpa/sdpa_fwd.cu.cc and sdpa/sdpa_bwd.cu.cc, compiled
for sm_100a).  Errors raised by the reference's validation come back as
``RefOpError`` with the reference's exact message.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_DT_FLOAT, _DT_HALF = 1, 19


class RefOpError(RuntimeError):
    """The reference OpKernel rejected its inputs (OP_REQUIRES failure)."""


_libs: dict[str, ctypes.CDLL] = {}


def _lib(device: str) -> ctypes.CDLL:
    name = "libsdpa_ref_gpu.so" if device == "GPU" else "libsdpa_ref_cpu.so"
    if name in _libs:
        return _libs[name]
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing: run oracle/build_ref.sh")
    lib = ctypes.CDLL(path)
    lib.ref_run.restype = ctypes.c_int
    lib.ref_run.argtypes = [
        ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_long), ctypes.POINTER(ctypes.c_long),
        ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_long),
        ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int,
    ]
    lib.ref_set_num_threads.argtypes = [ctypes.c_int]
    lib.ref_get_num_threads.restype = ctypes.c_int
    lib.ref_num_kernels.restype = ctypes.c_int
    lib.ref_kernel_info.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_int)]
    _libs[name] = lib
    return lib


def available(device: str = "CPU") -> bool:
    name = "libsdpa_ref_gpu.so" if device == "GPU" else "libsdpa_ref_cpu.so"
    return os.path.exists(os.path.join(REF_DIR, name))


def set_num_threads(n: int, device: str = "CPU") -> None:
    _lib(device).ref_set_num_threads(int(n))


def get_num_threads(device: str = "CPU") -> int:
    return int(_lib(device).ref_get_num_threads())


def registered_kernels(device: str = "CPU") -> list[tuple[str, str, int]]:
    lib = _lib(device)
    out = []
    for i in range(lib.ref_num_kernels()):
        op = ctypes.create_string_buffer(64)
        dev = ctypes.create_string_buffer(16)
        dt = ctypes.c_int()
        lib.ref_kernel_info(i, op, 64, dev, 16, ctypes.byref(dt))
        out.append((op.value.decode(), dev.value.decode(), dt.value))
    return out


def _ptr_shape(x):
    """(pointer, shape, dtype-code) of a numpy array or torch tensor."""
    if isinstance(x, np.ndarray):
        assert x.flags["C_CONTIGUOUS"]
        dt = {np.dtype(np.float16): _DT_HALF, np.dtype(np.float32): _DT_FLOAT}.get(x.dtype)
        return x.ctypes.data, tuple(x.shape), dt
    import torch  # noqa: PLC0415

    assert x.is_contiguous()
    dt = {torch.float16: _DT_HALF, torch.float32: _DT_FLOAT}.get(x.dtype)
    return x.data_ptr(), tuple(x.shape), dt


def _run(op, device, tensors, seed, offset, outs, scale, dropout, causal):
    lib = _lib(device)
    seed_a = np.array(np.uint64(seed & 0xFFFFFFFFFFFFFFFF))
    off_a = np.array(np.uint64(offset & 0xFFFFFFFFFFFFFFFF))
    ptrs, ranks, dims = [], [], []
    dtype = None
    for t in tensors:
        p, s, dt = _ptr_shape(t)
        if dtype is None:
            dtype = dt
        ptrs.append(p)
        ranks.append(len(s))
        dims.extend(s)
    for a in (seed_a, off_a):
        ptrs.append(a.ctypes.data)
        ranks.append(0)
    out_ptrs = [_ptr_shape(o)[0] for o in outs]
    n_in, n_out = len(ptrs), len(out_ptrs)
    c_in = (ctypes.c_void_p * n_in)(*ptrs)
    c_ranks = (ctypes.c_long * n_in)(*ranks)
    c_dims = (ctypes.c_long * max(1, len(dims)))(*dims)
    c_out = (ctypes.c_void_p * n_out)(*out_ptrs)
    c_odims = (ctypes.c_long * (3 * n_out))()
    err = ctypes.create_string_buffer(512)
    stream = None
    if device == "GPU" and not isinstance(tensors[0], np.ndarray):
        import torch  # noqa: PLC0415

        stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ref_run(op.encode(), device.encode(), dtype, n_in, c_in, c_ranks, c_dims, n_out, c_out, c_odims,
                     float(scale), float(dropout), int(bool(causal)), stream, err, 512)
    if rc == 1:
        raise RefOpError(err.value.decode())
    if rc != 0:
        raise RuntimeError(f"reference op failed ({rc}): {err.value.decode()}")
    return [tuple(int(v) for v in c_odims[3 * i:3 * i + 3] if v >= 0) for i in range(n_out)]


def _empty_like_shape(proto, shape, dtype=None):
    if isinstance(proto, np.ndarray):
        return np.zeros(shape, dtype=dtype or proto.dtype)
    import torch  # noqa: PLC0415

    return torch.zeros(shape, dtype=dtype or proto.dtype, device=proto.device)


def ref_sdpa(q, k, v, seed, offset, *, scale=1.0, dropout=0.0, causal_mask=False, device="CPU"):
    """The reference ``Sdpa`` op: returns (output [B,S_q,D_v] T, stats [B,S_q] f32)."""
    f32 = np.float32 if isinstance(q, np.ndarray) else __import__("torch").float32
    B, S_q = q.shape[0], q.shape[1]
    o = _empty_like_shape(q, (B, S_q, v.shape[2]))
    s = _empty_like_shape(q, (B, S_q), f32)
    shapes = _run("Sdpa", device, [q, k, v], seed, offset, [o, s], scale, dropout, causal_mask)
    assert shapes[0] == tuple(o.shape) and shapes[1] == tuple(s.shape), shapes
    return o, s


def ref_sdpa_grad(q, k, v, out, stats, d_o, seed, offset, *, dropout=0.0, scale=1.0, causal_mask=False,
                  device="CPU"):
    """The reference ``SdpaGrad`` op: returns (dq, dk, dv) shaped like q, k, v."""
    dq = _empty_like_shape(q, tuple(q.shape))
    dk = _empty_like_shape(k, tuple(k.shape))
    dv = _empty_like_shape(v, tuple(v.shape))
    _run("SdpaGrad", device, [q, k, v, out, stats, d_o], seed, offset, [dq, dk, dv], scale, dropout, causal_mask)
    return dq, dk, dv
