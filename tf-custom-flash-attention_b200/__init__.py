"""sdpa_b200: Blackwell (sm_100a) attention behind the reference's Sdpa / SdpaGrad ops.

    import importlib; fa = importlib.import_module("tf-custom-flash-attention_b200")
    o, stats = fa.sdpa(q, k, v, seed, offset, scale=..., dropout=..., causal_mask=...)
    dq, dk, dv = fa.sdpa_grad(q, k, v, o, stats, d_o, seed, offset, dropout=..., scale=..., causal_mask=...)

Kernels live in csrc/ and are reached through the C ABI of include/sdpa_b200.h
(libsdpa_b200.so, built in-tree by build.py).
"""
from .ops import (InvalidArgumentError, KernelError, device_status, dropout_mask, kernel_path, last_launch_count,
                  sdpa, sdpa_bshd, sdpa_grad, sdpa_grad_bshd)
from . import autograd, pipeline, sharding  # noqa: F401
from .mha import MHA  # noqa: F401
from ._lib import LIB_PATH  # noqa: F401

__all__ = ["sdpa", "sdpa_grad", "sdpa_bshd", "sdpa_grad_bshd", "dropout_mask", "device_status", "kernel_path", "last_launch_count",
           "InvalidArgumentError", "KernelError", "autograd", "pipeline", "sharding", "MHA"]
