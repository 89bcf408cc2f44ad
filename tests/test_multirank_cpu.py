"""Multi-rank host logic on CPU: two gloo ranks shard a batch the way bench.py
and the multi-GPU runs do (contiguous rows, dropout offset rebased), compute
their shard with the oracle, all-gather, and must reproduce the unsharded
result bit for bit.  A rank that fails is reported to the other through the
process group (it learns of it on the host, no device involved)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, k, v, out_dir, fail_rank):
    import importlib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import cpu

    fa = importlib.import_module("tf-custom-flash-attention_b200")
    B, S, _ = q.shape
    b0, b1 = fa.sharding.shard_rows(B, world, rank)
    off = fa.sharding.shard_offset(1000, b0, S, S)
    ok = torch.tensor([0 if rank == fail_rank else 1])
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)  # every rank learns of a failed peer before computing
    if ok.item() == 1:
        o, s = cpu.sdpa(q[b0:b1], k[b0:b1], v[b0:b1], 42, off, scale=0.25, dropout=0.3, causal_mask=True)
        parts = [None] * world
        dist.all_gather_object(parts, (b0, o, s))
        if rank == 0:
            np.savez(os.path.join(out_dir, "gathered.npz"), o=np.concatenate([p[1] for p in sorted(parts)]),
                     s=np.concatenate([p[2] for p in sorted(parts, key=lambda x: x[0])]))
    elif rank == 0:
        open(os.path.join(out_dir, "peer_failed"), "w").close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_two_rank_shards_reproduce_unsharded(tmp_path, fail_rank):
    from oracle import cpu

    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((5, 40, 16)).astype(np.float32) for _ in range(3))
    mp.spawn(_worker, args=(2, _free_port(), q, k, v, str(tmp_path), fail_rank), nprocs=2, join=True)
    if fail_rank >= 0:
        assert (tmp_path / "peer_failed").exists()
        return
    z = np.load(tmp_path / "gathered.npz")
    o, s = cpu.sdpa(q, k, v, 42, 1000, scale=0.25, dropout=0.3, causal_mask=True)
    assert np.array_equal(z["o"], o) and np.array_equal(z["s"], s)
