"""The allocation-free backward entry point, checked against the regular one.

sdpa_b200_bwd_noalloc exists for callers that cannot allocate device memory
per call -- a memory-planned graph executor, a real-time loop, an embedded
host -- so it takes no workspace and uses a fixed scratch array inside the
library instead.  This file is collected last so that a run stopping at the
first failure has already run every other test.
"""
import ctypes
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

fa = importlib.import_module("tf-custom-flash-attention_b200")
TOL = {torch.float16: 2e-3, torch.float32: 1e-5}


def _bwd(noalloc, q, k, v, o, s, do, kw):
    L = fa._lib.lib()
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    dt = fa._lib.F16 if q.dtype == torch.float16 else fa._lib.F32
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    st = torch.cuda.current_stream().cuda_stream
    common = (dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), s.data_ptr(), do.data_ptr(),
              dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S_q, S_kv, D_qk, D_v, kw["scale"], kw["dropout"],
              int(kw["causal"]), 7, 11)
    if noalloc:
        rc = L.sdpa_b200_bwd_noalloc(*common, st)
    else:
        n = L.sdpa_b200_bwd_workspace_bytes(dt, B, S_q, S_kv, D_qk, D_v)
        ws = torch.empty(max(n, 4) // 4, dtype=torch.float32, device="cuda")
        rc = L.sdpa_b200_bwd(*common, ws.data_ptr(), n, st)
    assert rc == 0, fa._lib.strerror(rc)
    return dq, dk, dv


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("dtype,B,S,D,causal,p", [
    (torch.float16, 2, 512, 128, True, 0.1),
    (torch.float16, 3, 200, 64, False, 0.0),
    (torch.float32, 2, 96, 40, True, 0.2),
])
def test_noalloc_matches_regular_backward_twice(dtype, B, S, D, causal, p):
    kw = dict(scale=D ** -0.5, dropout=p, causal=causal)
    for call in range(2):  # the second call runs over the first call's leftover scratch
        g = torch.Generator(device="cuda").manual_seed(100 * call + D)
        q, k, v, do = (torch.randn(B, S, D, generator=g, device="cuda").to(dtype) for _ in range(4))
        o, s = fa.sdpa(q, k, v, 7, 11, scale=kw["scale"], dropout=p, causal_mask=causal)
        ref = _bwd(False, q, k, v, o, s, do, kw)
        got = _bwd(True, q, k, v, o, s, do, kw)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert _rel(a, b) <= TOL[dtype]


def test_noalloc_rejects_problems_beyond_its_scratch():
    L = fa._lib.lib()
    rows = fa._lib.NOALLOC_MAX_ROWS + 1
    rc = L.sdpa_b200_bwd_noalloc(0, *([None] * 9), 1, rows, rows, 8, 8, 1.0, 0.0, 0, 0, 0, None)
    assert rc == fa._lib.ESCRATCH
    assert "scratch" in fa._lib.strerror(rc)
