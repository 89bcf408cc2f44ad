"""Times the reference's own GPU op (sdpa/sdpa_fwd.cu.cc, sdpa/sdpa_bwd.cu.cc built
unmodified for sm_100a by build_ref.sh) on the B200, as context for the
benchmark numbers.  Test infrastructure: nothing in the product imports it.

Only shapes the GPU test suite already ran the reference op at are timed
(see tests/test_gpu_parity.py and tests/test_gpu_configs.py); each line names
its shape.  TFLOP/s are algorithmic (fwd 2*S_q*S_kv*(D_qk+D_v), bwd
2*S_q*S_kv*(3*D_qk+2*D_v) per batch row, halved when causal), CUDA events,
one warm-up call.

    python oracle/time_ref_gpu.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import ref  # noqa: E402

SHAPES = [
    # name, dtype, B, S_q, S_kv, D_qk, D_v, causal, dropout, std
    ("cfg1 (exact shape)", np.float32, 20, 400, 400, 32, 4, False, 0.2, 1.0),
    ("cfg2 rows (B=4 of 64)", np.float16, 4, 1024, 1024, 64, 64, True, 0.0, 1.0),
    ("cfg4 D/causal/dropout at S=512 (B=4)", np.float16, 4, 512, 512, 128, 128, True, 0.1, 1.0),
    ("cfg5 rows (B=2 of 128)", np.float32, 2, 512, 4096, 64, 128, False, 0.05, 0.5),
]


def main():
    out = []
    for name, dt, B, S_q, S_kv, Dq, Dv, causal, p, std in SHAPES:
        rng = np.random.default_rng(0)
        q, k, v, do = (torch.from_numpy((rng.standard_normal(sh) * std).astype(dt)).cuda()
                       for sh in ((B, S_q, Dq), (B, S_kv, Dq), (B, S_kv, Dv), (B, S_q, Dv)))
        kw = dict(scale=Dq ** -0.5, dropout=p, causal_mask=causal)

        def step():
            o, s = ref.ref_sdpa(q, k, v, 1, 2, device="GPU", **kw)
            ref.ref_sdpa_grad(q, k, v, o, s, do, 1, 2, device="GPU", **kw)

        step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        f = 0.5 if causal else 1.0
        flops = 2.0 * S_q * S_kv * B * f * ((Dq + Dv) + (3 * Dq + 2 * Dv))
        out.append({"shape": name, "ms_fwd_bwd": ms, "tflops": flops / (ms * 1e-3) / 1e12})
        print(json.dumps(out[-1]), flush=True)


if __name__ == "__main__":
    main()
