"""The two routes of the fp32 (3xTF32) backward, both against the oracle
(needs a B200).

* GEMM route (the workspace sdpa_b200_bwd_workspace_bytes asks for): D, the
  score pass writing dS and P~ (dropout-scaled P), then dQ = scale dS K,
  dK = scale dS^T Q and dV = P~^T dO as GEMMs (5 launches).
* Recomputing route (a workspace of one float per query row, as the
  reference's op allocates): DQ, DK and DV passes (3 launches).

Tolerance (north star): fp32 max|new - ref| <= 1e-5 * max|ref|.
"""
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu  # noqa: E402

pytestmark = pytest.mark.gpu

fa = importlib.import_module("tf-custom-flash-attention_b200")


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def bwd(q, k, v, o, s, do, kw, minimal, ws_shift=0):
    """ws_shift: bytes by which the workspace start is moved off torch's
    256-byte alignment (TF's allocator guarantees only 64)."""
    L = fa._lib.lib()
    B, S_q, D_qk = q.shape
    S_kv, D_v = k.shape[1], v.shape[2]
    full = L.sdpa_b200_bwd_workspace_bytes(fa._lib.F32, B, S_q, S_kv, D_qk, D_v)
    n = B * S_q * 4 if minimal else full
    assert minimal or full > B * S_q * 4  # the GEMM route applies to these shapes
    ws = torch.empty((n + ws_shift + 3) // 4, dtype=torch.float32, device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    rc = L.sdpa_b200_bwd(fa._lib.F32, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), s.data_ptr(),
                         do.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S_q, S_kv, D_qk, D_v,
                         kw["scale"], kw["dropout"], int(kw["causal_mask"]), 5, 9, ws.data_ptr() + ws_shift, n,
                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0, fa._lib.strerror(rc)
    launches = fa.last_launch_count()
    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in (dq, dk, dv)], launches


@pytest.mark.parametrize("B,S_q,S_kv,D_qk,D_v,causal,p", [
    (2, 150, 150, 64, 32, True, 0.1),
    (1, 70, 300, 48, 20, False, 0.0),
    (2, 256, 640, 64, 128, False, 0.05),
    (2, 384, 384, 32, 64, True, 0.0),
    (3, 129, 33, 16, 100, False, 0.5),
])
def test_both_routes_match_oracle(B, S_q, S_kv, D_qk, D_v, causal, p):
    rng = np.random.default_rng(S_q + 3 * S_kv + D_v)
    q = (rng.standard_normal((B, S_q, D_qk)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, S_kv, D_qk)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, S_kv, D_v)) * 0.5).astype(np.float32)
    do = rng.standard_normal((B, S_q, D_v)).astype(np.float32)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 5, 9, **kw)
    t = [torch.from_numpy(x).cuda() for x in (q, k, v, o_ref, s_ref, do)]
    gemm, n_gemm = bwd(*t, kw, minimal=False)
    passes, n_passes = bwd(*t, kw, minimal=True)
    assert (n_gemm, n_passes) == (5, 3)
    for route, got in (("gemm", gemm), ("passes", passes)):
        for name, a, b in zip(("dq", "dk", "dv"), got, g_ref):
            assert rel(a, b) <= 1e-5, (route, name, rel(a, b))
    assert fa.device_status() == 0


@pytest.mark.parametrize("B,S_q,S_kv,D_qk,D_v,causal,p", [
    (2, 192, 192, 128, 64, True, 0.1),
    (1, 100, 300, 96, 20, False, 0.0),
    (1, 256, 1024, 128, 128, False, 0.05),
    (2, 150, 150, 100, 88, True, 0.1),
])
def test_gemm_route_serves_d_qk_128(B, S_q, S_kv, D_qk, D_v, causal, p):
    """D_qk = 128 runs on the tensor cores only on the GEMM route (the
    recomputing passes do not fit TMEM); with D_v over 64 as well the score
    pass keeps V lo in shared memory."""
    assert fa.kernel_path(torch.float32, D_qk, D_v, backward=True) == "tcgen05-3xtf32"
    rng = np.random.default_rng(D_qk + S_kv)
    q = (rng.standard_normal((B, S_q, D_qk)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, S_kv, D_qk)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, S_kv, D_v)) * 0.5).astype(np.float32)
    do = rng.standard_normal((B, S_q, D_v)).astype(np.float32)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 5, 9, **kw)
    t = [torch.from_numpy(x).cuda() for x in (q, k, v, o_ref, s_ref, do)]
    got, n = bwd(*t, kw, minimal=False)
    assert n == 5
    for name, a, b in zip(("dq", "dk", "dv"), got, g_ref):
        assert rel(a, b) <= 1e-5, (name, rel(a, b))
    assert fa.device_status() == 0


def test_gemm_route_with_a_64_byte_aligned_workspace():
    rng = np.random.default_rng(64)
    B, S_q, S_kv, D_qk, D_v = 2, 200, 264, 64, 64
    q = (rng.standard_normal((B, S_q, D_qk)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, S_kv, D_qk)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, S_kv, D_v)) * 0.5).astype(np.float32)
    do = rng.standard_normal((B, S_q, D_v)).astype(np.float32)
    kw = dict(scale=0.125, dropout=0.1, causal_mask=False)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 5, 9, **kw)
    t = [torch.from_numpy(x).cuda() for x in (q, k, v, o_ref, s_ref, do)]
    got, n = bwd(*t, kw, minimal=False, ws_shift=64)
    assert n == 5
    for name, a, b in zip(("dq", "dk", "dv"), got, g_ref):
        assert rel(a, b) <= 1e-5, (name, rel(a, b))


def test_workspace_query_sizes_the_gemm_route():
    """fp32 shapes ask for dS and P~ (of every row, or of the rows that fit
    under the cap); fp16 asks for one float per query row."""
    L = fa._lib.lib()
    B, S_q, S_kv = 2, 100, 70
    full = L.sdpa_b200_bwd_workspace_bytes(fa._lib.F32, B, S_q, S_kv, 64, 128)
    assert full >= B * S_q * 4 + 2 * B * S_q * 72 * 4  # dS, P~: rows of S_kv padded to 16 bytes
    assert L.sdpa_b200_bwd_workspace_bytes(fa._lib.F16, B, S_q, S_kv, 64, 128) == B * S_q * 4
    assert L.sdpa_b200_bwd_workspace_bytes(fa._lib.F32, B, S_q, S_kv, 128, 64) > B * S_q * 4  # D_qk = 128: GEMM route
    assert L.sdpa_b200_bwd_workspace_bytes(fa._lib.F32, B, S_q, S_kv, 128, 128) > B * S_q * 4
    big = L.sdpa_b200_bwd_workspace_bytes(fa._lib.F32, 64, 8192, 8192, 64, 64)  # 34 GB for all rows
    assert 64 * 8192 * 4 + (2 << 30) < big <= 64 * 8192 * 4 + 4096 + (4 << 30)  # rows that fit under 4 GiB


@pytest.mark.parametrize("B,S_q,S_kv,D_qk,D_v,causal,p", [
    (1, 256, 4096, 128, 128, False, 0.05),
    (2, 200, 200, 100, 72, True, 0.1),
])
def test_forward_with_both_dims_over_64(B, S_q, S_kv, D_qk, D_v, causal, p):
    """The fp32 forward with D_qk and D_v over 64 keeps Q lo in shared memory
    (TMEM holds Q hi, O, its running total and 32-key score tiles)."""
    assert fa.kernel_path(torch.float32, D_qk, D_v) == "tcgen05-3xtf32"
    rng = np.random.default_rng(D_v + S_kv)
    q = (rng.standard_normal((B, S_q, D_qk)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, S_kv, D_qk)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, S_kv, D_v)) * 0.5).astype(np.float32)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    o, s = fa.sdpa(*[torch.from_numpy(x).cuda() for x in (q, k, v)], 5, 9, **kw)
    assert fa.last_launch_count() == 1
    torch.cuda.synchronize()
    assert rel(o.cpu().numpy(), o_ref) <= 1e-5, rel(o.cpu().numpy(), o_ref)
    assert rel(s.cpu().numpy(), s_ref) <= 1e-5, rel(s.cpu().numpy(), s_ref)
    assert fa.device_status() == 0


@pytest.mark.parametrize("B,S_q,S_kv,D_qk,D_v,causal,p", [
    (128, 64, 384, 32, 32, False, 0.1),
    (96, 256, 256, 64, 48, True, 0.0),
])
def test_persistent_gemms_over_many_items(B, S_q, S_kv, D_qk, D_v, causal, p):
    """More work items than SMs: each persistent dK / dV GEMM CTA runs several
    items back to back (item boundaries inside one pipeline)."""
    rng = np.random.default_rng(B + S_kv)
    q = (rng.standard_normal((B, S_q, D_qk)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, S_kv, D_qk)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, S_kv, D_v)) * 0.5).astype(np.float32)
    do = rng.standard_normal((B, S_q, D_v)).astype(np.float32)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 5, 9, **kw)
    t = [torch.from_numpy(x).cuda() for x in (q, k, v, o_ref, s_ref, do)]
    got, n = bwd(*t, kw, minimal=False)
    assert n == 5
    for name, a, b in zip(("dq", "dk", "dv"), got, g_ref):
        assert rel(a, b) <= 1e-5, (name, rel(a, b))
    assert fa.device_status() == 0


def _chunk_ws_bytes(B, S_q, S_kv, rows):
    """Workspace for the delta rows of all B rows plus dS / P~ of `rows` rows."""
    r256 = lambda x: (x + 255) // 256 * 256  # noqa: E731
    ld = (S_kv + 3) // 4 * 4
    return r256(B * S_q * 4) + 2 * r256(rows * S_q * ld * 4) + 256


@pytest.mark.parametrize("B,S_q,S_kv,D_qk,D_v,causal,p,rows", [
    (5, 130, 130, 64, 128, True, 0.1, 2),
    (3, 96, 200, 128, 64, False, 0.2, 1),
])
def test_gemm_route_in_batch_chunks(B, S_q, S_kv, D_qk, D_v, causal, p, rows):
    """A workspace for fewer rows than the batch (as past the 4 GiB cap): the
    GEMM route runs in chunks of that many rows, each with its rows' offsets
    and dropout counters."""
    rng = np.random.default_rng(B * 7 + rows)
    q = (rng.standard_normal((B, S_q, D_qk)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, S_kv, D_qk)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, S_kv, D_v)) * 0.5).astype(np.float32)
    do = rng.standard_normal((B, S_q, D_v)).astype(np.float32)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 5, 9, **kw)
    tq, tk, tv, to, ts, tdo = (torch.from_numpy(x).cuda() for x in (q, k, v, o_ref, s_ref, do))
    L = fa._lib.lib()
    n = _chunk_ws_bytes(B, S_q, S_kv, rows)
    ws = torch.empty((n + 3) // 4, dtype=torch.float32, device="cuda")
    dq, dk, dv = torch.empty_like(tq), torch.empty_like(tk), torch.empty_like(tv)
    rc = L.sdpa_b200_bwd(fa._lib.F32, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), to.data_ptr(), ts.data_ptr(),
                         tdo.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S_q, S_kv, D_qk, D_v,
                         kw["scale"], p, int(causal), 5, 9, ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, fa._lib.strerror(rc)
    assert fa.last_launch_count() == 5 * ((B + rows - 1) // rows)
    torch.cuda.synchronize()
    for name, a, b in zip(("dq", "dk", "dv"), (dq, dk, dv), g_ref):
        assert rel(a.cpu().numpy(), b) <= 1e-5, (name, rel(a.cpu().numpy(), b))
    assert fa.device_status() == 0


def test_gemm_route_in_batch_chunks_bshd():
    """[B, S, H, D] layout: chunks hold whole outer batch rows (a multiple of H
    folded rows); a workspace for 3 folded rows with H = 2 runs chunks of 2."""
    B, H, S, D = 3, 2, 96, 64
    rng = np.random.default_rng(11)
    q, k, v, do = ((rng.standard_normal((B * H, S, D)) * 0.5).astype(np.float32) for _ in range(4))
    kw = dict(scale=D ** -0.5, dropout=0.1, causal_mask=True)
    o_ref, s_ref = cpu.sdpa(q, k, v, 5, 9, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 5, 9, **kw)

    def bshd(x):  # folded row b*H + h -> [B, S, H, D]
        return torch.from_numpy(x).cuda().reshape(B, H, S, x.shape[2]).permute(0, 2, 1, 3).contiguous()

    tq, tk, tv, to, tdo = (bshd(x) for x in (q, k, v, o_ref, do))
    ts = torch.from_numpy(s_ref).cuda().reshape(B, H, S).contiguous()
    L = fa._lib.lib()
    n = _chunk_ws_bytes(B * H, S, S, 3)
    ws = torch.empty((n + 3) // 4, dtype=torch.float32, device="cuda")
    dq, dk, dv = torch.empty_like(tq), torch.empty_like(tk), torch.empty_like(tv)
    rc = L.sdpa_b200_bwd_bshd(fa._lib.F32, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), to.data_ptr(), ts.data_ptr(),
                              None, tdo.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, S, S, D, D,
                              kw["scale"], 0.1, 1, 5, 9, ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, fa._lib.strerror(rc)
    assert fa.last_launch_count() == 5 * 3  # chunks of 2 folded rows
    torch.cuda.synchronize()
    for name, a, b in zip(("dq", "dk", "dv"), (dq, dk, dv), g_ref):
        got = a.permute(0, 2, 1, 3).reshape(B * H, S, D).cpu().numpy()
        assert rel(got, b) <= 1e-5, (name, rel(got, b))


def test_batch_chunks_equal_one_pass_bitwise_with_dstats():
    """Every kernel of the GEMM route works per batch row, so chunking the batch
    changes no bit of the result, also with a stats gradient (its rows offset
    per chunk like D and the stats)."""
    B, S_q, S_kv, D_qk, D_v = 5, 100, 140, 64, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, S_q, D_qk, generator=g, device="cuda") * 0.5
    k = torch.randn(B, S_kv, D_qk, generator=g, device="cuda") * 0.5
    v = torch.randn(B, S_kv, D_v, generator=g, device="cuda") * 0.5
    do = torch.randn(B, S_q, D_v, generator=g, device="cuda")
    dst = torch.randn(B, S_q, generator=g, device="cuda") * 0.1
    o, s = fa.sdpa(q, k, v, 5, 9, scale=0.125, dropout=0.1)
    L = fa._lib.lib()

    def run(n):
        ws = torch.empty((n + 3) // 4, dtype=torch.float32, device="cuda")
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        rc = L.sdpa_b200_bwd_dstats(fa._lib.F32, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), s.data_ptr(),
                                    dst.data_ptr(), do.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S_q,
                                    S_kv, D_qk, D_v, 0.125, 0.1, 0, 5, 9, ws.data_ptr(), n,
                                    torch.cuda.current_stream().cuda_stream)
        assert rc == 0, fa._lib.strerror(rc)
        return fa.last_launch_count(), (dq, dk, dv)

    n_full, full = run(L.sdpa_b200_bwd_workspace_bytes(fa._lib.F32, B, S_q, S_kv, D_qk, D_v))
    n_chunk, chunked = run(_chunk_ws_bytes(B, S_q, S_kv, 2))
    assert (n_full, n_chunk) == (5, 15)
    torch.cuda.synchronize()
    for a, b in zip(full, chunked):
        assert torch.equal(a, b)
