"""The oracle pinned against the reference: golden vectors + the reference's own build.

CPU only.  The C restatement (oracle/sdpa_oracle.c) must reproduce
  * the RNG known answers of test.py:33-46 (Python big-int LCG),
  * the golden outputs of the reference's own Sdpa / SdpaGrad ops,
  * the reference op run live (oracle/_ref), incl. its error strings,
  * float64 dense attention with the same dropout mask.
"""
import glob
import os

import numpy as np
import pytest

from oracle import cpu, dense, ref


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.abs(b).max() if b.size else 1.0
    return float(np.abs(a - b).max() / max(den, 1e-30)) if b.size else 0.0


def test_rng_known_answers(golden_dir):
    z = np.load(os.path.join(golden_dir, "rng_kat.npz"))
    for p, u in zip(z["points"], z["u"]):
        p = [int(x) for x in p]
        assert dense.get_random_float(*p) == u
        assert cpu.rng_uniform(*p) == u


def test_rng_vectorised_matches_bigint():
    seed, offset, B, S_q, S_kv = (1 << 64) - 7, 123, 2, 5, 9
    u = dense.uniform_tensor(seed, offset, B, S_q, S_kv)
    for b in range(B):
        for i in range(S_q):
            for j in range(S_kv):
                assert u[b, i, j] == dense.get_random_float(seed, offset, b, i, j, S_q, S_kv)


def test_dropout_mask_matches_dense():
    m = cpu.dropout_mask(42, 1000, 2, 30, 40, 0.2)
    keep = dense.keep_mask(42, 1000, 2, 30, 40, 0.2)
    assert np.array_equal(m == 0, keep == 1)
    assert 0.1 < m.mean() < 0.3
    assert cpu.dropout_mask(42, 1000, 1, 4, 4, 1e-7).sum() == 0  # enable rule: rate > 1e-6


GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "ref_cpu_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[8:-4] for p in GOLDEN])
def test_oracle_matches_reference_golden(path):
    z = np.load(path)
    kw = dict(scale=float(z["scale"]), dropout=float(z["dropout"]), causal_mask=bool(z["causal"]))
    seed, offset = int(z["seed"]), int(z["offset"])
    o, s = cpu.sdpa(z["q"], z["k"], z["v"], seed, offset, **kw)
    f16 = z["q"].dtype == np.float16
    tol = 2e-3 if f16 else 1e-5
    assert rel(o, z["o"]) <= tol
    assert rel(s, z["stats"]) <= (1e-3 if f16 else 1e-5)
    dq, dk, dv = cpu.sdpa_grad(z["q"], z["k"], z["v"], z["o"], z["stats"], z["d_o"], seed, offset, **kw)
    assert rel(dq, z["dq"]) <= tol
    # The reference's CPU backward accumulates dK/dV in T (sdpa/sdpa_cpu.cc:416-418,
    # :437-438), i.e. in half for fp16: allow for that rounding there.
    assert rel(dk, z["dk"]) <= (2e-2 if f16 else 1e-5)
    assert rel(dv, z["dv"]) <= (2e-2 if f16 else 1e-5)


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[8:-4] for p in GOLDEN])
def test_oracle_matches_dense_f64(path):
    z = np.load(path)
    kw = dict(scale=float(z["scale"]), dropout=float(z["dropout"]), causal_mask=bool(z["causal"]))
    seed, offset = int(z["seed"]), int(z["offset"])
    o, s = cpu.sdpa(z["q"], z["k"], z["v"], seed, offset, **kw)
    o64, s64, _, _ = dense.forward(z["q"], z["k"], z["v"], seed, offset, **kw)
    f16 = z["q"].dtype == np.float16
    assert rel(o, o64) <= (2e-3 if f16 else 1e-5)
    g = cpu.sdpa_grad(z["q"], z["k"], z["v"], o, s, z["d_o"], seed, offset, **kw)
    g64 = dense.backward(z["q"], z["k"], z["v"], z["d_o"], seed, offset, **kw)
    for a, b in zip(g, g64):
        # the oracle keeps the reference's p <= 1e-6 skip rule; dense does not
        assert rel(a, b) <= (4e-3 if f16 else 2e-5)


needs_ref = pytest.mark.skipif(not ref.available("CPU"), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("dt", [np.float32, np.float16])
@pytest.mark.parametrize("causal", [False, True])
def test_oracle_matches_reference_live(dt, causal):
    rng = np.random.default_rng(5)
    B, S_q, D_qk, D_v = 2, 45, 24, 16
    S_kv = S_q if causal else 61
    q = rng.standard_normal((B, S_q, D_qk)).astype(dt)
    k = rng.standard_normal((B, S_kv, D_qk)).astype(dt)
    v = rng.standard_normal((B, S_kv, D_v)).astype(dt)
    do = rng.standard_normal((B, S_q, D_v)).astype(dt)
    kw = dict(scale=0.3, dropout=0.15, causal_mask=causal)
    o1, s1 = cpu.sdpa(q, k, v, 9, 99, **kw)
    o2, s2 = ref.ref_sdpa(q, k, v, 9, 99, **kw)
    tol = 2e-3 if dt == np.float16 else 1e-5
    assert rel(o1, o2) <= tol and rel(s1, s2) <= tol
    g1 = cpu.sdpa_grad(q, k, v, o2, s2, do, 9, 99, **kw)
    g2 = ref.ref_sdpa_grad(q, k, v, o2, s2, do, 9, 99, **kw)
    assert rel(g1[0], g2[0]) <= tol
    for a, b in zip(g1[1:], g2[1:]):
        assert rel(a, b) <= (2e-2 if dt == np.float16 else 1e-5)


@needs_ref
def test_reference_error_strings():
    q = np.zeros((2, 8, 16), np.float32)
    k = np.zeros((2, 8, 16), np.float32)
    v = np.zeros((2, 8, 4), np.float32)
    cases = [
        ((q, k[:1], v), {}, "K batch size mismatch"),
        ((q, k[:, :, :8], v), {}, "K feature size mismatch"),
        ((q, k, v[:1]), {}, "V batch size mismatch"),
        ((q, k, v[:, :4]), {}, "V seq size mismatch"),
        ((q, k[:, :4], v[:, :4]), {"causal_mask": True}, "seq size Q != K while causal_mask = True"),
        ((np.zeros((2, 8, 130), np.float32), np.zeros((2, 8, 130), np.float32), v), {},
         "CUDA kernel does not support feature size over 128. Set smaller feature size or use more heads"),
    ]
    for args, kw, msg in cases:
        with pytest.raises(ref.RefOpError, match="^" + msg.replace("(", r"\(") + "$"):
            ref.ref_sdpa(*[np.ascontiguousarray(a) for a in args], 1, 2, **kw)
