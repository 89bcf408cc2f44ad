"""CUDA kernels vs the oracle on the same seeded inputs (needs a B200).

Tolerances (north star): fp16  max|new - ref| <= 2e-3 * max|ref|  for o, stats, dq, dk, dv;
fp32 <= 1e-5 * max|ref|.  Dropout masks must be identical (exact).
"""
import glob
import importlib
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu, dense, ref  # noqa: E402

pytestmark = pytest.mark.gpu

fa = importlib.import_module("tf-custom-flash-attention_b200")

TOL = {np.float16: 2e-3, np.float32: 1e-5}


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if b.size == 0:
        return 0.0
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def make(dt, B, S_q, S_kv, D_qk, D_v, seed=0, std=1.0):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((B, S_q, D_qk)) * std).astype(dt)
    k = (rng.standard_normal((B, S_kv, D_qk)) * std).astype(dt)
    v = (rng.standard_normal((B, S_kv, D_v)) * std).astype(dt)
    do = rng.standard_normal((B, S_q, D_v)).astype(dt)
    return q, k, v, do


def cuda(*xs):
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in xs]


def host(*xs):
    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in xs]


FWD_CASES = [
    # dtype, B, S_q, S_kv, D_qk, D_v, causal, dropout
    (np.float16, 2, 256, 256, 128, 128, False, 0.0),
    (np.float16, 2, 256, 256, 128, 128, True, 0.0),
    (np.float16, 2, 384, 384, 64, 64, True, 0.0),
    (np.float16, 3, 200, 200, 128, 128, True, 0.1),
    (np.float16, 2, 130, 333, 64, 128, False, 0.05),
    (np.float16, 2, 77, 77, 40, 24, True, 0.3),
    (np.float16, 1, 1, 1, 8, 8, False, 0.0),
    (np.float16, 2, 129, 257, 128, 64, False, 0.0),
    (np.float16, 1, 300, 300, 100, 72, True, 0.0),
    (np.float16, 2, 90, 90, 5, 3, False, 0.2),          # not TMA-addressable: SIMT path
    (np.float32, 2, 64, 64, 32, 4, False, 0.2),
    (np.float32, 2, 40, 136, 64, 128, False, 0.05),
    (np.float32, 2, 50, 50, 5, 3, True, 0.25),
    (np.float32, 2, 150, 150, 64, 32, True, 0.1),      # 3xTF32, narrow values (D_v <= 32 kernels)
    (np.float32, 1, 70, 300, 48, 20, False, 0.0),
]


def ids(c):
    dt, B, S_q, S_kv, D_qk, D_v, causal, p = c
    return f"{np.dtype(dt).name}-B{B}-{S_q}x{S_kv}-d{D_qk}v{D_v}-{'c' if causal else 'n'}-p{p}"


@pytest.mark.parametrize("case", FWD_CASES, ids=[ids(c) for c in FWD_CASES])
def test_forward_matches_oracle(case):
    dt, B, S_q, S_kv, D_qk, D_v, causal, p = case
    q, k, v, _ = make(dt, B, S_q, S_kv, D_qk, D_v, seed=S_q + D_qk)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 42, 1000, **kw)
    o, s = fa.sdpa(*cuda(q, k, v), 42, 1000, **kw)
    o, s = host(o, s)
    assert rel(o, o_ref) <= TOL[dt], rel(o, o_ref)
    assert rel(s, s_ref) <= TOL[dt], rel(s, s_ref)


@pytest.mark.parametrize("case", FWD_CASES, ids=[ids(c) for c in FWD_CASES])
def test_backward_matches_oracle(case):
    dt, B, S_q, S_kv, D_qk, D_v, causal, p = case
    q, k, v, do = make(dt, B, S_q, S_kv, D_qk, D_v, seed=S_kv + D_v)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    o_ref, s_ref = cpu.sdpa(q, k, v, 7, 11, **kw)
    g_ref = cpu.sdpa_grad(q, k, v, o_ref, s_ref, do, 7, 11, **kw)
    g = fa.sdpa_grad(*cuda(q, k, v, o_ref, s_ref, do), 7, 11, **kw)
    for name, a, b in zip(("dq", "dk", "dv"), host(*g), g_ref):
        assert rel(a, b) <= TOL[dt], (name, rel(a, b))


GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "ref_*_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_matches_reference_golden(path):
    z = np.load(path)
    dt = z["q"].dtype.type
    kw = dict(scale=float(z["scale"]), dropout=float(z["dropout"]), causal_mask=bool(z["causal"]))
    seed, offset = int(z["seed"]), int(z["offset"])
    o, s = host(*fa.sdpa(*cuda(z["q"], z["k"], z["v"]), seed, offset, **kw))
    assert rel(o, z["o"]) <= TOL[dt]
    assert rel(s, z["stats"]) <= TOL[dt]
    g = host(*fa.sdpa_grad(*cuda(z["q"], z["k"], z["v"], z["o"], z["stats"], z["d_o"]), seed, offset, **kw))
    gpu_golden = os.path.basename(path).startswith("ref_gpu_")
    for name, a in zip(("dq", "dk", "dv"), g):
        # The reference CPU op accumulates dK/dV in T (sdpa/sdpa_cpu.cc:416-418):
        # for fp16 that golden is itself off by ~1e-2; its GPU op is not.
        tol = TOL[dt] if (gpu_golden or dt == np.float32 or name == "dq") else 2e-2
        assert rel(a, z[name]) <= tol, (name, rel(a, z[name]))


def test_dropout_mask_identical_to_reference_rng():
    for (seed, offset, B, S_q, S_kv, p) in [(42, 1000, 2, 64, 64, 0.2), (7, 0, 1, 33, 257, 0.1),
                                            ((1 << 64) - 3, (1 << 63) + 5, 3, 17, 33, 0.3),
                                            (1, 2, 1, 8, 8, 1e-7), (5, 6, 1, 16, 16, 0.999)]:
        m = fa.dropout_mask(seed, offset, B, S_q, S_kv, p).cpu().numpy()
        assert np.array_equal(m, cpu.dropout_mask(seed, offset, B, S_q, S_kv, p))


def test_dropout_mask_end_to_end_probe():
    """q = k = 0 makes P uniform (1/S_kv); V = identity columns expose the kernel's mask:
    O[i, c] = keep(i, j0 + c) / (1 - p) / S_kv for the window of keys j0..j0+D_v-1."""
    B, S, D, p = 2, 256, 128, 0.3
    seed, offset = 9, 123
    q = torch.zeros(B, S, D, dtype=torch.float16, device="cuda")
    k = torch.zeros(B, S, D, dtype=torch.float16, device="cuda")
    keep = dense.keep_mask(seed, offset, B, S, S, p)
    for j0 in (0, 128):
        v = torch.zeros(B, S, D, dtype=torch.float16, device="cuda")
        v[:, j0:j0 + D, :] = torch.eye(D, dtype=torch.float16, device="cuda")
        o, _ = fa.sdpa(q, k, v, seed, offset, scale=1.0, dropout=p)
        o = o.float().cpu().numpy() * S * (1 - p)
        assert np.array_equal(np.rint(o).astype(np.int64), keep[:, :, j0:j0 + D].astype(np.int64))


def test_sharded_offsets_reproduce_unsharded_run():
    dt, B, S, D = np.float16, 4, 128, 64
    q, k, v, _ = make(dt, B, S, S, D, D, seed=3)
    kw = dict(scale=0.125, dropout=0.2, causal_mask=True)
    full, _ = fa.sdpa(*cuda(q, k, v), 5, 77, **kw)
    parts = []
    for r in range(2):
        b0, b1 = fa.sharding.shard_rows(B, 2, r)
        off = fa.sharding.shard_offset(77, b0, S, S)
        parts.append(fa.sdpa(*cuda(q[b0:b1], k[b0:b1], v[b0:b1]), 5, off, **kw)[0])
    assert torch.equal(full, torch.cat(parts))


def test_validation_errors_match_reference():
    z = torch.zeros
    q = z(2, 8, 16, device="cuda")
    k = z(2, 8, 16, device="cuda")
    v = z(2, 8, 4, device="cuda")
    with pytest.raises(fa.InvalidArgumentError, match="^K batch size mismatch$"):
        fa.sdpa(q, k[:1], v, 1, 2)
    with pytest.raises(fa.InvalidArgumentError, match="^seq size Q != K while causal_mask = True$"):
        fa.sdpa(q, k[:, :4], v[:, :4], 1, 2, causal_mask=True)
    with pytest.raises(fa.InvalidArgumentError, match="feature size over 128"):
        fa.sdpa(z(1, 4, 130, device="cuda"), z(1, 4, 130, device="cuda"), z(1, 4, 4, device="cuda"), 1, 2)
    with pytest.raises(fa.InvalidArgumentError, match="^seed must be scalar$"):
        fa.sdpa(q, k, v, torch.tensor([1]), 2)
    with pytest.raises(fa.InvalidArgumentError, match="^dO seq size mismatch$"):
        fa.sdpa_grad(q, k, v, z(2, 8, 4, device="cuda"), z(2, 8, device="cuda"), z(2, 7, 4, device="cuda"), 1, 2)


def test_empty_and_degenerate_shapes():
    o, s = fa.sdpa(*[torch.zeros(0, 4, 8, dtype=torch.float16, device="cuda")] * 3, 1, 2)
    assert o.shape == (0, 4, 8) and s.shape == (0, 4)
    # S_kv = 0: no keys -> O = 0, stats = -1e9 + ln(1e-6) (sdpa/sdpa_fwd.cu.cc:160-163)
    q = torch.randn(1, 5, 8, device="cuda").half()
    kv = torch.zeros(1, 0, 8, dtype=torch.float16, device="cuda")
    o, s = fa.sdpa(q, kv, kv, 1, 2)
    torch.cuda.synchronize()
    assert torch.all(o == 0)
    assert torch.allclose(s, torch.full_like(s, np.float32(-1e9) + np.float32(np.log(np.float32(1e-6)))))


def test_device_wait_timeout_reports_status():
    L = fa._lib.lib()
    fa.device_status()  # clear
    assert L.sdpa_b200_test_wait_timeout(2_000_000, torch.cuda.current_stream().cuda_stream) == 0
    assert fa.device_status() & 1
    # the context stays usable
    x, = cuda(np.ones((1, 4, 8), np.float16))
    o, _ = fa.sdpa(x, x, x, 0, 0)
    torch.cuda.synchronize()
    assert fa.device_status() == 0


needs_ref_gpu = pytest.mark.skipif(not ref.available("GPU"), reason="oracle/_ref GPU build missing")


@needs_ref_gpu
@pytest.mark.parametrize("case", [
    (np.float16, 4, 512, 512, 128, 128, True, 0.1),
    (np.float16, 4, 1024, 1024, 64, 64, True, 0.0),
    (np.float16, 2, 256, 1024, 128, 64, False, 0.0),
    (np.float32, 2, 128, 1024, 64, 128, False, 0.05),
], ids=ids)
def test_matches_reference_gpu_op(case):
    """The north-star parity target: the reference's own GPU op on identical seeded inputs."""
    dt, B, S_q, S_kv, D_qk, D_v, causal, p = case
    q, k, v, do = make(dt, B, S_q, S_kv, D_qk, D_v, seed=11, std=1.0 if dt == np.float16 else 0.5)
    kw = dict(scale=D_qk ** -0.5, dropout=p, causal_mask=causal)
    tq, tk, tv, tdo = cuda(q, k, v, do)
    o_r, s_r = ref.ref_sdpa(tq, tk, tv, 7, 0, device="GPU", **kw)
    g_r = ref.ref_sdpa_grad(tq, tk, tv, o_r, s_r, tdo, 7, 0, device="GPU", **kw)
    o, s = fa.sdpa(tq, tk, tv, 7, 0, **kw)
    g = fa.sdpa_grad(tq, tk, tv, o_r, s_r, tdo, 7, 0, **kw)
    for a, b in zip(host(o, s, *g), host(o_r, s_r, *g_r)):
        assert rel(a, b) <= TOL[dt], rel(a, b)
