"""Multi-GPU partitioning: plan properties, and a world_size-2 gloo run on CPU
that shards a varlen prefill by (sequence, head group), computes each shard
with the CPU oracle, gathers, and compares with the unsharded result."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastaf_kernel_b200 import sharding, workloads as W


@pytest.mark.parametrize("lengths,world", [
    ([100, 5, 77, 3000, 64], 2), ([1, 1, 1], 8), ([500], 4), ([300, 200], 8),
    (W.loguniform_lengths(4, n=256), 8), ([0, 10, 0], 2)])
def test_plan_covers_every_chain_once(lengths, world):
    Hq, Hv = 16, 32
    plans = sharding.plan_prefill(lengths, world, Hq, Hv)
    seen = {}
    for pl in plans:
        for it in pl.items:
            for h in it.v_heads(Hv // Hq):
                assert (it.seq, h) not in seen
                seen[(it.seq, h)] = pl.rank
    assert set(seen) == {(s, h) for s in range(len(lengths)) for h in range(Hv)}


def test_plan_balances_loguniform_lengths():
    lengths = W.loguniform_lengths(4, n=256)
    plans = sharding.plan_prefill(lengths, 8, 16, 32)
    loads = [pl.load for pl in plans]
    assert max(loads) / (sum(loads) / len(loads)) < 1.05


def test_head_split_only_when_fewer_sequences_than_ranks():
    assert sharding.head_groups(16, 8, 16) == 1
    assert sharding.head_groups(4, 8, 16) == 2
    assert sharding.head_groups(1, 8, 16) == 8
    assert sharding.head_groups(3, 8, 4) == 4
    plans = sharding.plan_prefill([1000, 900], 8, 16, 32)
    assert all(len(pl.items) == 1 for pl in plans)
    assert {it.hq1 - it.hq0 for pl in plans for it in pl.items} == {4}


def test_decode_plan_equal_counts():
    plans = sharding.plan_decode(512, 8, 16, 32)
    assert sorted(len(pl.items) for pl in plans) == [64] * 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lengths, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import c_oracle
        Hq, Hv = 4, 8
        x = W.prefill_inputs(lengths, seed=9, Hq=Hq, Hv=Hv, state_mask=[True, False, True, True])
        plans = sharding.plan_prefill(lengths, world, Hq, Hv)
        T, N = x["q"].shape[0], len(lengths)
        out = torch.zeros((T, Hv, 128), dtype=torch.bfloat16)
        ns = torch.zeros((N, Hv, 128, 128))
        results = []
        for sub, items, idx in sharding.shard_prefill_inputs(x, plans[rank], Hq, Hv):
            r = c_oracle.prefill(sub["q"], sub["k"], sub["v"], sub["state"], sub["A_log"],
                                 sub["a"], sub["dt_bias"], sub["b"], sub["cu_seqlens"],
                                 sub["scale"], num_threads=1)
            results.append((r, items, idx))
        sharding.scatter_prefill_outputs(out, ns, results, Hq, Hv)
        # results are disjoint across ranks: a sum gathers them (checking only)
        out_f = out.float()
        dist.all_reduce(out_f)
        dist.all_reduce(ns)
        if rank == 0:
            ro, rs = c_oracle.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"],
                                      x["dt_bias"], x["b"], x["cu_seqlens"], x["scale"],
                                      num_threads=1)
            q.put((torch.equal(out_f.to(torch.bfloat16), ro), torch.equal(ns, rs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("lengths", [[40, 3, 70, 9], [130, 1, 2, 64]])
def test_gloo_world2_sharded_prefill_equals_unsharded(lengths):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    out_ok, state_ok = q.get(timeout=5)
    assert out_ok and state_ok
