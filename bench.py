"""Benchmark: attention fwd+bwd TFLOP/s on B200 (BASELINE.json metric), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg4]

Workload (default, BASELINE.json configs[3], the long-context training case
the north-star targets are quoted on): fp16 q/k/v [32, 8192, 128] ~N(0,1),
causal, dropout 0.1, seed 7, offset 0, scale 1/sqrt(128); one step = forward
(Sdpa) + backward (SdpaGrad) with d_o ~N(0,1).  Synthetic seeded inputs.
Multi-GPU: weak scaling, every rank owns its own 32 batch rows (global rows
rank*32 ..), dropout offset rebased so masks equal an unsharded run; no
collective on the data path; time = max over ranks.

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
    for _ in range(args.warmup if args.warmup < 1 else 1):
        pass
    val, threads, sample, t = time_reference_cpu(w, steps=max(1, args.steps))
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": {"workload": args.workload, **{k: w[k] for k in ("B", "S", "D_qk", "D_v", "causal", "dropout")},
                   "S_kv": seqs(w)[1]},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, w):
    import torch

    rank, world, local = dist_init(args.gpus)
    torch.cuda.set_device(local)
    fa = importlib.import_module("tf-custom-flash-attention_b200")
    dev = torch.device("cuda", local)
    B, Dq, Dv = w["B"], w["D_qk"], w["D_v"]
    S, S_kv = seqs(w)
    dt = torch.float16 if w["dtype"] == "f16" else torch.float32
    b0 = rank * B  # weak scaling: this rank's global batch rows
    offset = fa.sharding.shard_offset(w["offset"], b0, S, S_kv)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    std = w.get("std", 1.0)
    q, k, v, do = ((torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std).to(dt)
                   for shape in ((B, S, Dq), (B, S_kv, Dq), (B, S_kv, Dv), (B, S, Dv)))
    kw = dict(scale=Dq ** -0.5, dropout=w["dropout"], causal_mask=w["causal"])
    stream = torch.cuda.current_stream()

    launches = [0]
    # per-kernel timing of the backward (rowsum | dK/dV | dQ) on the launching
    # stream, through the library's diagnostic event hook (tensor-core path only)
    per_kernel = fa.kernel_path(dt, Dq, Dv, backward=True) == "tcgen05"
    kev = []

    def step():
        o, s = fa.sdpa(q, k, v, w["seed"], offset, **kw)
        n = fa.last_launch_count()
        e_mid = torch.cuda.Event(enable_timing=True)
        e_mid.record(stream)
        if per_kernel:
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            for e in evs:  # torch creates the CUDA event on its first record
                e.record(stream)
            arr = (ctypes.c_void_p * 4)(*[e.cuda_event for e in evs])
            fa._lib.lib().sdpa_b200_set_bwd_events(arr, 4)
            kev.append(evs)
        dq, dk, dv = fa.sdpa_grad(q, k, v, o, s, do, w["seed"], offset, **kw)
        if per_kernel:
            fa._lib.lib().sdpa_b200_set_bwd_events(None, 0)
        launches[0] += n + fa.last_launch_count()
        return e_mid

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    launches[0] = 0
    kev.clear()
    evs = []
    e0 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    prev = e0
    for _ in range(args.steps):
        mid = step()
        end = torch.cuda.Event(enable_timing=True)
        end.record(stream)
        evs.append((prev, mid, end))
        prev = end
    torch.cuda.synchronize()
    total_ms = e0.elapsed_time(prev)
    fwd_ms = sum(a.elapsed_time(m) for a, m, _ in evs) / args.steps
    bwd_ms = sum(m.elapsed_time(e) for _, m, e in evs) / args.steps
    kernel_ms = None
    if per_kernel and len(kev) == args.steps:
        kernel_ms = {name: sum(e[i].elapsed_time(e[i + 1]) for e in kev) / args.steps
                     for i, name in enumerate(("dq", "dkdv"))}
    clk = clocks.stop()
    per_rank = [{"rank": rank, "ms_per_step": total_ms / args.steps, "sm_mhz": clk.get("sm_mhz"),
                 "reasons": clk.get("reasons")}]
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
        gathered = [None] * world
        torch.distributed.all_gather_object(gathered, per_rank[0])
        per_rank = gathered
        torch.distributed.barrier()

    # ---- end to end through the public API: pinned host inputs in, results out, every step
    hq, hk, hv, hdo = (x.cpu().pin_memory() for x in (q, k, v, do))
    outs_h = None
    e2e_ms = None
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hdo))
    d2h = 0

    def e2e_step():
        # public host-buffer API: batch chunks pipelined over copy-in / compute / copy-out streams
        nonlocal outs_h, d2h
        outs_h = fa.pipeline.train_step_host(hq, hk, hv, hdo, w["seed"], offset, scale=kw["scale"],
                                             dropout=kw["dropout"], causal_mask=kw["causal_mask"], chunks=8,
                                             device=dev, out=outs_h)
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
    e2e_ms = a.elapsed_time(b_) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())

    f_fwd, f_bwd = flops(w)
    ms = total_ms / args.steps
    value = world * (f_fwd + f_bwd) / (ms * 1e-3) / 1e12
    peak, peak_kind = peaks()
    fwd_tf = f_fwd / (fwd_ms * 1e-3) / 1e12
    bwd_tf = f_bwd / (bwd_ms * 1e-3) / 1e12
    # Dominant kernel.  Algorithmic FLOPs per launch: fwd = the forward; of the
    # backward's 5 MMA-units (S, dP, dV, dK, dQ), dK/dV carries 4 and dQ 1 (its
    # S and dP are recomputation, not algorithmic work).
    cands = [("fwd_pair_kernel", fwd_ms, f_fwd)]
    if kernel_ms:
        cands += [("dkdv_kernel", kernel_ms["dkdv"], 0.8 * f_bwd), ("dq2_kernel", kernel_ms["dq"], 0.2 * f_bwd)]
    else:
        cands += [("bwd (all kernels)", bwd_ms, f_bwd)]
    name, kms, kfl = max(cands, key=lambda c: c[1])
    dominant = (name, kfl / (kms * 1e-3) / 1e12, kms, kfl)
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
            val, threads, sample, _ = time_reference_cpu(w)
            cpu = {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": "reference", "sample": sample}
        except Exception as e:  # the reference build is missing on this box
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16" if dt == torch.float16 else "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": args.workload, "global_batch": B * world, "per_gpu_batch": B, "seq_len": S,
                   "seq_len_kv": S_kv,
                   "D_qk": Dq, "D_v": Dv, "causal": w["causal"], "dropout": w["dropout"],
                   "parallelism": f"batch-sharded x{world}, no collective",
                   "l2": (f"inputs {sum(x.numel() * x.element_size() for x in (q, k, v, do)) / 1e6:.0f} MB per step "
                          + ("(larger than L2)" if sum(x.numel() * x.element_size() for x in (q, k, v, do)) > 126e6
                             else "(fit in L2: small config)"))},
        "fwd_tflops": fwd_tf, "bwd_tflops": bwd_tf, "pct_of_peak": 100.0 * value / world / peak,
        "roofline": {"bound": "tensor", "kernel": dominant[0], "achieved": dominant[1], "peak": peak,
                     "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": dominant[1] / peak, "traffic": traffic,
                     "ms_per_launch": dominant[2], "flops_per_launch": dominant[3],
                     "kernel_ms": kernel_ms, "traffic_source": "profiles/traffic_cfg4.md (ncu, scaled)"},
        "e2e": {"value": world * (f_fwd + f_bwd) / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": launches[0],
        "per_rank": per_rank,
        "clocks": clk,
        "cpu_baseline": cpu,
    }
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
