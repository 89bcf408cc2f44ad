"""CPU-only checks of the host side: the C ABI library loads and exports every
declared symbol, header and binding agree, sharding arithmetic, no compute."""
import importlib
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
fa = importlib.import_module("tf-custom-flash-attention_b200")


def header_symbols():
    src = open(os.path.join(ROOT, "include", "sdpa_b200.h")).read()
    return sorted(set(re.findall(r"\b(sdpa_b200_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = fa._lib.lib()
    syms = header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(fa._lib.EXPORTS) == syms


def test_version_and_strerror():
    L = fa._lib.lib()
    assert L.sdpa_b200_version() >= 100
    assert fa._lib.strerror(0) == "ok"
    assert "128" in fa._lib.strerror(2)


def test_path_selection():
    import torch

    assert fa.kernel_path(torch.float16, 128, 128) == "tcgen05"
    assert fa.kernel_path(torch.float16, 64, 40) == "tcgen05"
    assert fa.kernel_path(torch.float16, 5, 3) == "simt"
    assert fa.kernel_path(torch.float16, 8, 64) == "simt"      # too few dims: the reference's product rounding
    assert fa.kernel_path(torch.float16, 16, 8) == "tcgen05"
    assert fa.kernel_path(torch.float32, 64, 128) == "tcgen05-3xtf32"
    assert fa.kernel_path(torch.float32, 32, 4, backward=True) == "tcgen05-3xtf32"
    assert fa.kernel_path(torch.float32, 128, 64) == "tcgen05-3xtf32"
    assert fa.kernel_path(torch.float32, 128, 128) == "tcgen05-3xtf32"  # Q lo in shared memory
    assert fa.kernel_path(torch.float32, 128, 128, backward=True) == "tcgen05-3xtf32"  # GEMM route, V lo in smem
    assert fa.kernel_path(torch.float32, 128, 64, backward=True) == "tcgen05-3xtf32"  # GEMM route
    assert fa.kernel_path(torch.float32, 5, 3) == "simt"


def test_argument_errors_without_gpu():
    L = fa._lib.lib()
    # invalid dtype, D > 128, causal with S_q != S_kv: rejected before any CUDA call
    assert L.sdpa_b200_fwd(7, None, None, None, None, None, 1, 1, 1, 8, 8, 1.0, 0.0, 0, 0, 0, None) == 1
    assert L.sdpa_b200_fwd(0, None, None, None, None, None, 1, 1, 1, 200, 8, 1.0, 0.0, 0, 0, 0, None) == 2
    assert L.sdpa_b200_fwd(0, None, None, None, None, None, 1, 2, 3, 8, 8, 1.0, 0.0, 1, 0, 0, None) == 1
    # empty problem: nothing to do
    assert L.sdpa_b200_fwd(0, None, None, None, None, None, 0, 4, 4, 8, 8, 1.0, 0.0, 0, 0, 0, None) == 0
    # workspace checks
    assert L.sdpa_b200_bwd_workspace_bytes(0, 2, 10, 10, 8, 8) == 80
    assert L.sdpa_b200_bwd(0, *([None] * 9), 2, 10, 10, 8, 8, 1.0, 0.0, 0, 0, 0, None, 0, None) == 5


def test_shard_offsets_reproduce_global_counter():
    from oracle import dense

    B, S_q, S_kv, seed, off = 5, 7, 9, 3, 11
    u = dense.uniform_tensor(seed, off, B, S_q, S_kv)
    for world in (1, 2, 3):
        for r in range(world):
            b0, b1 = fa.sharding.shard_rows(B, world, r)
            o2 = fa.sharding.shard_offset(off, b0, S_q, S_kv)
            assert np.array_equal(dense.uniform_tensor(seed, o2, b1 - b0, S_q, S_kv), u[b0:b1])
    assert fa.sharding.advance_offset(off, B, S_q, S_kv) == off + B * S_q * S_kv


def test_host_validation_messages():
    import torch

    x = torch.zeros(2, 4, 8)
    with pytest.raises(fa.InvalidArgumentError, match="^K batch size mismatch$"):
        fa.sdpa(x, torch.zeros(1, 4, 8), x, 0, 0)
    with pytest.raises(fa.InvalidArgumentError, match="rank 3"):
        fa.sdpa(torch.zeros(4, 8), x, x, 0, 0)
    with pytest.raises(fa.InvalidArgumentError, match="CUDA tensors only"):
        fa.sdpa(x, x, x, 0, 0)  # no CPU kernel: fails loudly


def test_bshd_validation_on_host():
    """sdpa_bshd checks ranks and head counts before touching a device."""
    torch = pytest.importorskip("torch")
    q = torch.zeros(2, 8, 4, 16)
    with pytest.raises(fa.InvalidArgumentError, match="rank 4"):
        fa.sdpa_bshd(q[0], q, q, 0, 0)
    with pytest.raises(fa.InvalidArgumentError, match="head count"):
        fa.sdpa_bshd(q, torch.zeros(2, 8, 3, 16), q, 0, 0)
