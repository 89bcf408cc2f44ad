"""Benchmark: attention fwd+bwd TFLOP/s on B200 (BASELINE.json metric), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg4]

Workload (default, BASELINE.json configs[3], the long-context training case
the north-star targets are quoted on): fp16 q/k/v [32, 8192, 128] ~N(0,1),
causal, dropout 0.1, seed 7, offset 0, scale 1/sqrt(128); one step = forward
(Sdpa) + backward (SdpaGrad) with d_o ~N(0,1).  Synthetic seeded inputs.
Multi-GPU (--gpus N under torchrun): strong scaling.  The workload's global
batch is split into contiguous shards (sharding.shard_rows; cfg4: 32/16/8/4
rows per GPU at N = 1/2/4/8), each rank's dropout offset rebased
(sharding.shard_offset) so masks equal the unsharded run; no collective on the
data path; time = max over ranks.  Outside the timed region the first row of
every shard (o, stats, dq, dk, dv) is all-gathered over NCCL to rank 0, which
rebuilds each shard from its per-row seeds, reruns it at the global offset and
checks those rows bit for bit ("validated").
The weak-scaling figure (every rank the full per-GPU batch) is reported beside
it, as are each rank's pinned host<->device copy bandwidths measured alone and
with all ranks copying at once (what bounds the end-to-end number).

FLOPs per step (algorithmic, causal halves both): fwd 2*S^2*(Dqk+Dv)*B/2,
bwd 2*S^2*(3*Dqk+2*Dv)*B/2.

--impl reference times the reference's own CPU implementation
(sdpa/sdpa_cpu.cc built unmodified, oracle/_ref) on this host's cores, on a
bounded sample of the same workload (same D, dtype, causal, dropout; S and B
reduced, see `cpu_sample`), in the same unit.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "cfg4": dict(B=32, S=8192, D_qk=128, D_v=128, causal=True, dropout=0.1, seed=7, offset=0, dtype="f16"),
    "cfg3": dict(B=256, S=2048, D_qk=128, D_v=128, causal=False, dropout=0.0, seed=0, offset=0, dtype="f16"),
    "cfg2": dict(B=64, S=1024, D_qk=64, D_v=64, causal=True, dropout=0.0, seed=0, offset=0, dtype="f16"),
    # fp32 cases (BASELINE.json configs[0] and [4])
    "cfg1": dict(B=20, S=400, D_qk=32, D_v=4, causal=False, dropout=0.2, seed=42, offset=1000, dtype="f32"),
    "cfg5": dict(B=128, S=512, S_kv=4096, D_qk=64, D_v=128, causal=False, dropout=0.05, seed=0, offset=0,
                 dtype="f32", std=0.5),
}
# cuBLAS tf32 matmul, 8192^3, measured on this pool's B200s (profiles/tf32_matmul_peak.md)
TF32_MATMUL_TFLOPS = 738.7
METRIC = "fwd and fwd+bwd attention TFLOP/s per B200, % of dense fp16 tensor peak"


def seqs(w):
    """(S_q, S_kv) of a workload."""
    return w["S"], w.get("S_kv", w["S"])


def flops(w, B=None, S_q=None, S_kv=None):
    B = w["B"] if B is None else B
    sq, skv = seqs(w)
    S_q = sq if S_q is None else S_q
    S_kv = skv if S_kv is None else S_kv
    f = 0.5 if w["causal"] else 1.0
    fwd = 2.0 * S_q * S_kv * (w["D_qk"] + w["D_v"]) * B * f
    bwd = 2.0 * S_q * S_kv * (3 * w["D_qk"] + 2 * w["D_v"]) * B * f
    return fwd, bwd


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            m = json.load(fh)
        return float(m["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def min_bytes(w, B, S_q, S_kv, esize):
    """Bytes one fwd + bwd step must move at least: the forward reads Q, K, V and
    writes O and stats; the backward reads Q, K, V, O, dO and stats and writes
    dQ, dK, dV (a small shape's step is bound by latency, not by these)."""
    q, k, v, o = (B * S_q * w["D_qk"], B * S_kv * w["D_qk"], B * S_kv * w["D_v"], B * S_q * w["D_v"])
    stats = B * S_q * 4
    fwd = (q + k + v + o) * esize + stats
    bwd = (q + k + v + 2 * o) * esize + stats + (q + k + v) * esize
    return fwd + bwd


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init(n):
    import torch

    if n <= 1:
        return 0, 1, 0
    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return rank, world, local


def cpu_sample(w):
    """Bounded sample of the workload for the reference CPU op: same D, dtype, causal and
    dropout, S = 1024 and one batch row per host thread (its parallelFor is over B)."""
    from oracle import ref

    threads = ref.get_num_threads("CPU")
    sq, skv = seqs(w)
    return dict(B=threads, S_q=min(sq, 1024), S_kv=min(skv, 1024)), threads


def time_reference_cpu(w, steps=1):
    """TFLOP/s of the reference's own CPU Sdpa+SdpaGrad (sdpa/sdpa_cpu.cc) on this host."""
    import numpy as np

    from oracle import ref

    smp, threads = cpu_sample(w)
    B, S_q, S_kv = smp["B"], smp["S_q"], smp["S_kv"]
    rng = np.random.default_rng(0)
    dt = np.float16 if w["dtype"] == "f16" else np.float32
    std = w.get("std", 1.0)
    q, k, v, do = ((rng.standard_normal(shape) * std).astype(dt) for shape in
                   ((B, S_q, w["D_qk"]), (B, S_kv, w["D_qk"]), (B, S_kv, w["D_v"]), (B, S_q, w["D_v"])))
    kw = dict(scale=w["D_qk"] ** -0.5, dropout=w["dropout"], causal_mask=w["causal"])
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        o, s = ref.ref_sdpa(q, k, v, w["seed"], w["offset"], **kw)
        ref.ref_sdpa_grad(q, k, v, o, s, do, w["seed"], w["offset"], **kw)
        times.append(time.perf_counter() - t0)
    f, b = flops(w, B, S_q, S_kv)
    t = statistics.median(times)
    sample = (f"reference CPU op (sdpa/sdpa_cpu.cc, -O2) fwd+bwd on q[{B},{S_q},{w['D_qk']}] "
              f"kv[{B},{S_kv},{w['D_qk']}/{w['D_v']}] (sequences capped at 1024, one batch row per thread), {w['dtype']}, "
              f"causal={w['causal']}, dropout={w['dropout']}")
    return (f + b) / t / 1e12, threads, sample, t


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    warm = min(args.warmup, 1)  # each step is seconds of CPU work: one real warm-up step
    if warm:
        time_reference_cpu(w, steps=1)
    val, threads, sample, t = time_reference_cpu(w, steps=max(1, args.steps))
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": warm, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": {"workload": args.workload, **{k: w[k] for k in ("B", "S", "D_qk", "D_v", "causal", "dropout")},
                   "S_kv": seqs(w)[1]},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def make_rows(w, b0, b1, dev, dt):
    """Inputs q, k, v, d_o of global batch rows [b0, b1): each row from its own seeded
    generator, so any rank can rebuild any row."""
    import torch

    Dq, Dv = w["D_qk"], w["D_v"]
    S, S_kv = seqs(w)
    std = w.get("std", 1.0)
    out = [torch.empty((b1 - b0, n, d), dtype=dt, device=dev) for n, d in ((S, Dq), (S_kv, Dq), (S_kv, Dv), (S, Dv))]
    g = torch.Generator(device=dev)
    for b in range(b0, b1):
        g.manual_seed(1000003 * (b + 1))
        for t in out:
            t[b - b0].copy_(torch.randn(t.shape[1:], generator=g, device=dev, dtype=torch.float32) * std)
    out[3].div_(std)  # d_o ~ N(0, 1)
    return out


def host_copy_bandwidth(dev, world, rank, nbytes=1 << 28):
    """Pinned host <-> device copy GB/s of this rank: alone (ranks take turns) and
    with every rank copying at once."""
    import torch

    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def timed(src, dst):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dst.copy_(src, non_blocking=True)  # warm
        torch.cuda.synchronize()
        a.record()
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        return 3 * nbytes / (a.elapsed_time(b) * 1e-3) / 1e9

    res = {}
    for name, src, dst in (("h2d", h, d), ("d2h", d, h)):
        alone = None
        for r in range(world):
            if world > 1:
                torch.distributed.barrier()
            if r == rank:
                alone = timed(src, dst)
        if world > 1:
            torch.distributed.barrier()
        res[f"{name}_alone_gbs"] = alone
        res[f"{name}_concurrent_gbs"] = timed(src, dst)
    return res


def run_ours(args, w):
    import torch

    rank, world, local = dist_init(args.gpus)
    torch.cuda.set_device(local)
    fa = importlib.import_module("tf-custom-flash-attention_b200")
    dev = torch.device("cuda", local)
    B_glob, Dq, Dv = w["B"], w["D_qk"], w["D_v"]
    S, S_kv = seqs(w)
    dt = torch.float16 if w["dtype"] == "f16" else torch.float32
    b0, b1 = fa.sharding.shard_rows(B_glob, world, rank)  # strong scaling: this rank's global rows
    B = b1 - b0
    offset = fa.sharding.shard_offset(w["offset"], b0, S, S_kv)
    q, k, v, do = make_rows(w, b0, b1, dev, dt)
    kw = dict(scale=Dq ** -0.5, dropout=w["dropout"], causal_mask=w["causal"])
    stream = torch.cuda.current_stream()
    path = fa.kernel_path(dt, Dq, Dv, backward=True)
    # per-kernel timing of the backward on the launching stream, through the
    # library's diagnostic event hook: fp16 runs dQ then dK/dV; fp32 either the
    # GEMM route (D + the score pass writing dS and P~^T, then the dQ, dK and dV
    # GEMMs, when the workspace query asks for room for them) or the passes dQ, dK, dV
    tf32_gemm = (dt == torch.float32 and fa._lib.lib().sdpa_b200_bwd_workspace_bytes(
        fa._lib.F32, B, S, S_kv, Dq, Dv) > B * S * 4)
    knames = {"tcgen05": ("dq2_kernel", "dkdv_kernel"),
              "tcgen05-3xtf32": (("tf32 D + score pass", "tf32 dQ gemm", "tf32 dK gemm", "tf32 dV gemm") if tf32_gemm
                                 else ("tf32 dQ", "tf32 dK", "tf32 dV"))}.get(path)
    n_ev = 5 if knames and len(knames) == 4 else 4
    launches = [0]
    kev = []
    last = {}

    def step(q, k, v, do, off, record=True):
        o, s = fa.sdpa(q, k, v, w["seed"], off, **kw)
        n = fa.last_launch_count()
        e_mid = torch.cuda.Event(enable_timing=True)
        e_mid.record(stream)
        if knames and record:
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
            for e in evs:  # torch creates the CUDA event on its first record
                e.record(stream)
            arr = (ctypes.c_void_p * n_ev)(*[e.cuda_event for e in evs])
            fa._lib.lib().sdpa_b200_set_bwd_events(arr, n_ev)
            kev.append(evs)
        dq, dk, dv = fa.sdpa_grad(q, k, v, o, s, do, w["seed"], off, **kw)
        if knames and record:
            fa._lib.lib().sdpa_b200_set_bwd_events(None, 0)
        launches[0] += n + fa.last_launch_count()
        last.update(o=o, s=s, dq=dq, dk=dk, dv=dv)
        return e_mid

    in_bytes = sum(x.numel() * x.element_size() for x in (q, k, v, do))
    # inputs that fit in L2 (126 MB): a 256 MB write between timed steps evicts them
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if in_bytes <= 126e6 else None

    def timed_loop(q, k, v, do, off, steps, record=True, graph=None):
        """Sum over `steps` of the device time of one step (events around each step on
        the launching stream; the L2 flush, when used, runs between steps, untimed)."""
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        evs = []
        for _ in range(steps):
            if flush_buf is not None:
                flush_buf.zero_()
            start = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            if graph is not None:
                graph.replay()
                mid = start
            else:
                mid = step(q, k, v, do, off, record)
            end = torch.cuda.Event(enable_timing=True)
            end.record(stream)
            evs.append((start, mid, end))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(e) for a, _, e in evs), evs

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step(q, k, v, do, offset, record=False)
    clocks = ClockSampler(local)
    clocks.start()
    launches[0] = 0
    kev.clear()
    total_ms, evs = timed_loop(q, k, v, do, offset, args.steps)
    timed_launches = launches[0]
    fwd_ms = sum(a.elapsed_time(m) for a, m, _ in evs) / args.steps
    bwd_ms = sum(m.elapsed_time(e) for _, m, e in evs) / args.steps
    graph_ms = None
    if not args.no_graph:
        # The same step captured once in a CUDA graph and replayed: the timed
        # work is unchanged (every kernel of every step runs), the host-side
        # launch cost (Python, argument checks, TMA descriptor encoding) is
        # taken out, which is what bounds short steps.
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            o_, s_ = fa.sdpa(q, k, v, w["seed"], offset, **kw)
            fa.sdpa_grad(q, k, v, o_, s_, do, w["seed"], offset, **kw)
        for _ in range(2):
            g.replay()
        graph_ms, _ = timed_loop(q, k, v, do, offset, args.steps, graph=g)
        total_ms = graph_ms
        del g
    clk = clocks.stop()
    kernel_ms = None
    if knames and len(kev) == args.steps:
        kernel_ms = {name: sum(e[i].elapsed_time(e[i + 1]) for e in kev) / args.steps for i, name in enumerate(knames)}
    my_ms = total_ms / args.steps
    total_ms = max_over_ranks(total_ms)
    per_rank = [{"rank": rank, "rows": [b0, b1], "ms_per_step": my_ms, "sm_mhz": clk.get("sm_mhz"),
                 "reasons": clk.get("reasons")}]

    # ---- validation over NCCL (outside the timed region): the first row of every
    # shard, recomputed on rank 0 with the global offset, must match bit for bit
    names = ("o", "s", "dq", "dk", "dv")
    sample = [last[n][0].contiguous() for n in names]
    if world > 1:
        gathered = []
        for t in sample:
            bufs = [torch.empty_like(t) for _ in range(world)]
            torch.distributed.all_gather(bufs, t)
            gathered.append(bufs)
        shards = [fa.sharding.shard_rows(B_glob, world, r) for r in range(world)]
    else:
        gathered = [[t] for t in sample]
        shards = [(b0, b1)]
    starts = [a for a, _ in shards]
    validated, mismatched = None, []
    if rank == 0:
        validated = True
        for r, (gb, ge) in enumerate(shards):
            # the shard rebuilt from its seeds and run with the shard's own batch size
            # (the kernel choice depends on it), at the global offset of its first row
            rq, rk, rv, rdo = make_rows(w, gb, ge, dev, dt)
            off_r = fa.sharding.shard_offset(w["offset"], gb, S, S_kv)
            step(rq, rk, rv, rdo, off_r, record=False)
            for n, bufs in zip(names, gathered):
                if not torch.equal(last[n][0], bufs[r]):
                    validated = False
                    mismatched.append([gb, n])
        torch.cuda.synchronize()

    # ---- weak scaling beside it (every rank the full per-GPU batch), N > 1 only
    weak = None
    if world > 1:
        wq, wk, wv, wdo = make_rows(w, rank * B_glob, (rank + 1) * B_glob, dev, dt)
        woff = fa.sharding.shard_offset(w["offset"], rank * B_glob, S, S_kv)
        step(wq, wk, wv, wdo, woff, record=False)
        wsteps = max(1, min(args.steps, 5))
        wms, _ = timed_loop(wq, wk, wv, wdo, woff, wsteps, record=False)
        wms = max_over_ranks(wms) / wsteps
        ff, fb = flops(w)
        weak = {"per_gpu_batch": B_glob, "global_batch": B_glob * world, "ms_per_step": wms,
                "value": world * (ff + fb) / (wms * 1e-3) / 1e12, "unit": "TFLOP/s"}
        del wq, wk, wv, wdo

    # ---- host copy bandwidth (what bounds the end-to-end number)
    copy_bw = host_copy_bandwidth(dev, world, rank)
    per_rank[0].update({k2: round(v2, 2) for k2, v2 in copy_bw.items()})

    # ---- end to end through the public API: pinned host inputs in, results out, every step
    hq, hk, hv, hdo = (x.cpu().pin_memory() for x in (q, k, v, do))
    outs_h = None
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hdo))
    d2h = 0

    # about 16 MB of inputs per chunk (at most 16 chunks): a small step is not
    # cut into launches shorter than their overhead
    e2e_chunks = max(1, min(16, B, h2d // (16 << 20)))

    def e2e_step():
        # public host-buffer API: batch chunks pipelined over copy-in / compute / copy-out streams
        nonlocal outs_h, d2h
        outs_h = fa.pipeline.train_step_host(hq, hk, hv, hdo, w["seed"], offset, scale=kw["scale"],
                                             dropout=kw["dropout"], causal_mask=kw["causal_mask"],
                                             chunks=e2e_chunks, device=dev, out=outs_h)
        d2h = sum(x.numel() * x.element_size() for x in outs_h)

    e2e_steps = max(1, min(args.steps, 5))
    for _ in range(min(args.warmup, 2)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b_ = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b_.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b_) / e2e_steps)
    if world > 1:
        gathered_pr = [None] * world
        torch.distributed.all_gather_object(gathered_pr, per_rank[0])
        per_rank = gathered_pr
        torch.distributed.barrier()

    f_fwd, f_bwd = flops(w)  # the whole (global) workload: strong scaling
    ms = total_ms / args.steps
    value = (f_fwd + f_bwd) / (ms * 1e-3) / 1e12
    peak, peak_kind = peaks()
    if dt == torch.float32:  # 3xTF32: three tf32 MMAs per product, tf32 matmul measured on this pool
        peak, peak_kind = TF32_MATMUL_TFLOPS / 3.0, "measured tf32 matmul (cuBLAS 8192^3) / 3"
    mf_fwd, mf_bwd = flops(w, B=B)  # this rank's share
    fwd_tf = mf_fwd / (fwd_ms * 1e-3) / 1e12
    bwd_tf = mf_bwd / (bwd_ms * 1e-3) / 1e12
    # Dominant kernel and its algorithmic FLOPs per launch.  Of the backward's five
    # products (S, dP, dV, dK, dQ; 2*S_q*S_kv*D each, D = D_qk for S, dK, dQ and D_v
    # for dP, dV) fp16's dK/dV kernel carries S, dP, dV, dK and its dQ kernel dQ (its
    # S and dP are recomputation); fp32's dQ pass carries dQ, dK pass S, dP, dK, dV pass dV.
    fwd_name = {"tcgen05": "fwd_pair_kernel", "tcgen05-3xtf32": "tf32 forward"}.get(
        fa.kernel_path(dt, Dq, Dv), "simt forward")
    unit = mf_bwd / (3 * Dq + 2 * Dv)
    cands = [(fwd_name, fwd_ms, mf_fwd)]
    if kernel_ms and path == "tcgen05":
        cands += [("dkdv_kernel", kernel_ms["dkdv_kernel"], unit * (2 * Dq + 2 * Dv)),
                  ("dq2_kernel", kernel_ms["dq2_kernel"], unit * Dq)]
    elif kernel_ms:  # fp32 passes: the dK pass carries S, dP, dK; GEMM route: the score pass S, dP
        share = {"tf32 dQ": Dq, "tf32 dK": 2 * Dq + Dv, "tf32 dV": Dv,
                 "tf32 D + score pass": Dq + Dv, "tf32 dQ gemm": Dq, "tf32 dK gemm": Dq, "tf32 dV gemm": Dv}
        cands += [(n, kernel_ms[n], unit * share[n]) for n in knames]
    else:
        cands += [("bwd (all kernels)", bwd_ms, mf_bwd)]
    name, kms, kfl = max(cands, key=lambda c: c[1])
    achieved = kfl / (kms * 1e-3) / 1e12
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as fh:
            traffic = json.load(fh).get(f"{args.workload}_{name}")
    except Exception:
        pass
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        try:
            val, threads, sample_txt, _ = time_reference_cpu(w)
            cpu = {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": "reference", "sample": sample_txt}
        except Exception as e:  # the reference build is missing on this box
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    hbm = hbm_peak()
    mb = min_bytes(w, B, S, S_kv, 2 if dt == torch.float16 else 4)  # this rank's share
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16" if dt == torch.float16 else "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": args.workload, "global_batch": B_glob, "per_gpu_batch": B, "seq_len": S,
                   "seq_len_kv": S_kv, "D_qk": Dq, "D_v": Dv, "causal": w["causal"], "dropout": w["dropout"],
                   "parallelism": f"batch-sharded x{world} (strong scaling), no collective on the data path",
                   "cuda_graph": not args.no_graph,
                   "l2": f"inputs {in_bytes / 1e6:.0f} MB per rank per step "
                         + ("(larger than L2)" if flush_buf is None else
                            "(fit in L2: a 256 MB write flushes L2 between timed steps)")},
        "kernel_path": path,
        "fwd_tflops": fwd_tf, "bwd_tflops": bwd_tf, "pct_of_peak": 100.0 * value / world / peak,
        "roofline": {"bound": "tensor", "kernel": name, "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic, "ms_per_launch": kms,
                     "flops_per_launch": kfl, "kernel_ms": kernel_ms},
        "memory": {"min_bytes_per_step": mb, "achieved_gbs": mb / (ms * 1e-3) / 1e9, "peak_gbs": hbm[0],
                   "peak_kind": hbm[1], "frac": mb / (ms * 1e-3) / 1e9 / hbm[0]},
        "e2e": {"value": (f_fwd + f_bwd) / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "chunks": e2e_chunks,
                "bound": "pinned host<->device copies (see per_rank copy GB/s)"},
        "validated": validated, "validation": {"rows_checked": starts, "mismatches": mismatched,
                                               "method": "NCCL all_gather of each shard's first row; rank 0 "
                                                         "rebuilds that shard from its seeds, reruns it with the "
                                                         "global offset and compares bit for bit"},
        "weak_scaling": weak,
        "gpu_launches": timed_launches,  # per step x steps (the graph replays the same launches)
        "per_rank": per_rank,
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    if world > 1:
        line["limiter"] = (f"{B} batch rows per GPU: forward {B * ((S + 255) // 256)} CTAs, backward "
                           f"{B * ((S + 127) // 128)} CTAs per kernel on 148 SMs"
                           + (", causal tiles of unequal length" if w["causal"] else ""))
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg4", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time the eager launches instead of a CUDA graph replay")
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (small profiling runs)")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.workload])
    if args.batch > 0:
        w["B"] = args.batch
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
