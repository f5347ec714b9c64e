#!/usr/bin/env python
"""Benchmark of the Gated DeltaNet hot paths on B200 (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one varlen prefill of 16 sequences x 8192 tokens (131072 tokens,
Hq=Hk=16, Hv=32, D=128, bf16 q/k/v, nonzero fp32 initial state, per-token decay
in [0.5, 0.999]) through the reference-facing ``kernel`` entry point.
``value`` is prefill tokens/s over all ranks with inputs resident in HBM;
the ``decode`` object reports the batched decode step (B=512, in-place state,
fresh q/k/v/a/b per step) in seq/s and state GB/s against the HBM roofline.

Multi-GPU (torchrun, one process per GPU), no data-path collective (sequences and
heads are independent; the only collectives are the timing barrier and max):
  * the headline step is weak-scaled: a global batch of 16 x N sequences of 8192
    tokens, placed by sharding.plan_prefill (16 per rank);
  * the ``mixed`` object is the strong-scaled mixed workload: 256 sequences with
    log-uniform lengths in [128, 32768] (1.55 M tokens) placed by plan_prefill
    (longest first on the least-loaded rank, load = tokens x v-heads), prefilled,
    then 1024 decode steps on the states each rank keeps resident; it reports the
    whole job's prefill tokens/s and decode sequence-steps/s and the load imbalance.
Timing is device time (CUDA events), max over ranks.

``--small-configs`` times only the two small configurations (a B = 4 decode step and a
4-sequence varlen prefill) through this library, the reference's Triton kernels and its
CPU torch code, as eager calls and as CUDA-graph replays (one GPU, one JSON object).

``--impl reference`` times the reference's own CPU implementation of the path
(the fp32 torch recurrence of solution/gdn_baseline_torch.py, restated in
oracle/gdn_ref.py) on the host cores, rank 0 only, on a bounded sample.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "prefill tokens/s; decode state GB/s (% of HBM peak)"
UNIT = "tokens/s"
N_SEQS, SEQ_LEN = 16, 8192
DECODE_B, DECODE_STEPS = 512, 100
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def profiled_traffic(name):
    """DRAM bytes per unit of work from a committed ncu summary (profiles/<name>.md,
    line 'dram_bytes_per_unit: <float>'), or None."""
    path = os.path.join(REPO, "profiles", name + ".md")
    try:
        with open(path) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_unit:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload_name():
    return f"gdn_prefill_{N_SEQS}x{SEQ_LEN}_hq16_hv32_d128"


def base_config(n_gpus):
    return {"workload": workload_name(), "n_seqs": N_SEQS, "seq_len": SEQ_LEN,
            "global_batch_seqs": N_SEQS * n_gpus,
            "tokens_per_gpu_step": N_SEQS * SEQ_LEN, "num_qk_heads": 16, "num_v_heads": 32,
            "head_size": 128, "initial_state": "fp32 N(0,0.02^2)", "decay_range": [0.5, 0.999],
            "decode_workload": f"gdn_decode_b{DECODE_B}_inplace_{DECODE_STEPS}steps",
            "l2": "inputs larger than L2 (2.2 GB per prefill step, 1 GiB decode state)",
            "parallelism": (f"sharded{n_gpus}: a global batch of {N_SEQS * n_gpus} x {SEQ_LEN} sequences "
                            f"placed by plan_prefill, {N_SEQS} per rank (weak scaling, no data-path "
                            "collective)")}


def cpu_prefill_sample(impl, budget_s):
    """Time a CPU implementation on a prefix of the 16 x 8192 workload (all 32
    heads, nonzero state), growing the sample until it takes ~budget_s."""
    from fastaf_kernel_b200 import workloads as W
    x = W.prefill_long(seed=3)
    n = 256
    total = N_SEQS * SEQ_LEN
    while True:
        lens = []
        left = n
        while left > 0:
            lens.append(min(SEQ_LEN, left))
            left -= lens[-1]
        cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(lens), 0)
        idx = torch.cat([torch.arange(s * SEQ_LEN, s * SEQ_LEN + L) for s, L in enumerate(lens)])
        sl = lambda t: t.index_select(0, idx)
        args = (sl(x["q"]), sl(x["k"]), sl(x["v"]), x["state"][:len(lens)], x["A_log"],
                sl(x["a"]), x["dt_bias"], sl(x["b"]), cu, x["scale"])
        t0 = time.perf_counter()
        impl(*args)
        dt = time.perf_counter() - t0
        if dt >= budget_s or n >= total:
            return n / dt, n, len(lens), dt
        n = min(total, max(n * 2, int(n * budget_s / max(dt, 1e-3) * 1.1)))


def reference_arm(args):
    """The reference's CPU implementation, timed on the host cores (rank 0)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import gdn_ref
    from fastaf_kernel_b200 import workloads as W
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample_tokens = 256
    x = W.prefill_inputs([SEQ_LEN], seed=3, decay_range=(0.5, 0.999))
    cu = torch.tensor([0, sample_tokens], dtype=torch.int32)
    sl = lambda t: t[:sample_tokens]
    run = lambda: gdn_ref.prefill(sl(x["q"]), sl(x["k"]), sl(x["v"]), x["state"], x["A_log"],
                                  sl(x["a"]), x["dt_bias"], sl(x["b"]), cu, x["scale"])
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = time.perf_counter() - t0
    value = sample_tokens * args.steps / dt
    # decode: one step of 8 sequences of the batched decode workload
    d = W.decode_inputs(8, seed=2)
    t1 = time.perf_counter()
    gdn_ref.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                   d["b"], d["scale"])
    ddt = time.perf_counter() - t1
    dec_gbs = 8 * W.bytes_per_decode_seq() / ddt / 1e9
    sample = (f"first {sample_tokens} tokens of one {SEQ_LEN}-token sequence, 32 v-heads, "
              f"per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": dict(base_config(world), cpu_sample=sample),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "impl": "oracle/gdn_ref.py (torch fp32 recurrence of "
                                 "solution/gdn_baseline_torch.py)", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "decode": {"value": dec_gbs, "unit": "GB/s", "seq_per_s": 8 / ddt,
                   "sample": "one decode step of 8 sequences"},
    }
    print(json.dumps(line), flush=True)
    return 0


MIXED_SEED, MIXED_SEQS, MIXED_STEPS = 4, 256, 1024
CP_TOKENS, CP_SEGMENTS_PER_RANK = 262144, 4


def run_context_parallel(args, rank, world, dev, barrier, gather):
    """One 262,144-token sequence (Hq 16, Hv 32, nonzero state, decay in [0.999, 0.99999])
    prefilled by context_parallel.prefill_context_parallel over all ranks (each rank a
    contiguous slice cut into 4 segments; one all-gather of the (M, C) state maps and one
    broadcast of the final state over NCCL), beside the same sequence as one ordinary
    prefill call on rank 0's GPU; returns the ``context_parallel`` object (rank 0)."""
    import torch.distributed as dist
    import fastaf_kernel_b200 as fk
    from fastaf_kernel_b200 import context_parallel as cp, workloads as W
    x = W.prefill_inputs([CP_TOKENS], seed=5, device=dev, decay_range=(0.999, 0.99999))
    per = (CP_TOKENS // world) // 64 * 64
    lo, hi = rank * per, (CP_TOKENS if rank == world - 1 else (rank + 1) * per)
    sl = lambda t: t[lo:hi]
    stream = torch.cuda.current_stream()

    def parallel():
        return cp.prefill_context_parallel(sl(x["q"]), sl(x["k"]), sl(x["v"]), x["state"], x["A_log"],
                                           sl(x["a"]), x["dt_bias"], sl(x["b"]), x["scale"],
                                           segments_per_rank=CP_SEGMENTS_PER_RANK)
    for _ in range(args.warmup):
        parallel()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(args.steps, 5))
    e0.record(stream)
    for _ in range(steps):
        _, fin = parallel()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    cp_ms = e0.elapsed_time(e1) / steps
    one_ms, rel = 0.0, 0.0
    if rank == 0:
        cu = torch.tensor([0, CP_TOKENS], dtype=torch.int32, device=dev)

        def one_pass():
            return fk.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                             cu, x["scale"])
        for _ in range(args.warmup):
            _, s1 = one_pass()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            _, s1 = one_pass()
        e1.record(stream)
        torch.cuda.synchronize()
        one_ms = e0.elapsed_time(e1) / steps
        rel = float(((fin - s1).abs().max() / s1.abs().max()).item())
    rows = gather([cp_ms, one_ms, rel])
    del x
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    par = max(r[0] for r in rows)
    return {"workload": f"gdn_context_parallel_1x{CP_TOKENS}_hq16_hv32_d128", "scaling": "strong",
            "segments_per_rank": CP_SEGMENTS_PER_RANK, "ranks": world, "ms": par,
            "tokens_per_s": CP_TOKENS / (par / 1e3), "one_gpu_one_pass_ms": rows[0][1],
            "speedup_vs_one_gpu_one_pass": rows[0][1] / par,
            "final_state_max_rel_vs_one_pass": rows[0][2],
            "exchange": "one NCCL all-gather of 3 x Hv x 128 x 128 float64 per rank, one broadcast of the "
                        "final state",
            "timing": f"mean of {steps} calls after {args.warmup} warm-up calls, max over ranks"}


def reference_gpu_leg(args, x, out, ns, d0, dsteps, dout, our_prefill, our_dec_gbs, stream):
    """The reference's own Triton GPU kernels (solution/triton/kernel.py:138-409, compiled
    ahead of time for sm_100 into oracle/_ref/ by oracle/ref_triton.py) on the same inputs
    as the timed prefill and decode steps, autotuned on this GPU as the reference's autotuner
    would; a measured baseline beside cpu_baseline, not the product path."""
    from oracle import ref_triton
    if not ref_triton.available():
        return {"unavailable": "oracle/_ref/ holds no compiled reference kernels (build() compiles them "
                               "where the reference checkout is present)"}
    from fastaf_kernel_b200 import workloads as W
    ref = ref_triton.RefTriton()
    T = x["q"].shape[0]

    def prefill():
        ref.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                    x["cu_seqlens"], x["scale"], out, ns)
    prefill()                        # autotunes: the fastest configuration of the list
    for _ in range(args.warmup - 1):
        prefill()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 5))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        prefill()
    e1.record(stream)
    torch.cuda.synchronize()
    pre_ms = e0.elapsed_time(e1) / steps
    B = d0["q"].shape[0]
    new_state = torch.empty_like(d0["state"])
    dec_out = dout.view(B, dout.shape[2], dout.shape[3])

    def decode(s):
        st = dsteps[s % len(dsteps)]
        ref.decode(st["q"], st["k"], st["v"], d0["state"], d0["A_log"], st["a"], d0["dt_bias"], st["b"],
                   d0["scale"], dec_out, new_state)
    decode(0)
    for s in range(1, args.warmup):
        decode(s)
    torch.cuda.synchronize()
    dsteps_n = len(dsteps)
    e0.record(stream)
    for s in range(dsteps_n):
        decode(s)
    e1.record(stream)
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1) / dsteps_n
    dec_gbs = B * W.bytes_per_decode_seq() / (dec_ms / 1e3) / 1e9
    del new_state
    torch.cuda.empty_cache()
    tps = T / (pre_ms / 1e3)
    return {"kind": "the reference's Triton kernels (_gdn_prefill_kernel_v2, _gdn_decode_kernel_v3 of "
                    "solution/triton/kernel.py), compiled for sm_100 from the reference sources, autotuned "
                    "over their own configuration lists on this GPU",
            "prefill": {"value": tps, "unit": UNIT, "ms_per_step": pre_ms, "steps": steps,
                        "config": ref.config("prefill"), "configs_timed": ref.tried["prefill"],
                        "ours_over_reference": our_prefill / tps},
            "decode": {"value": dec_gbs, "unit": "GB/s", "ms_per_step": dec_ms, "steps": dsteps_n,
                       "seq_per_s": B / (dec_ms / 1e3), "config": ref.config("decode"),
                       "configs_timed": ref.tried["decode"], "ours_over_reference": our_dec_gbs / dec_gbs,
                       "note": "out of place (the reference allocates a new state each step)"}}


def run_mixed(args, rank, world, dev, barrier, gather, peaks):
    """The mixed prefill + decode workload, strong-scaled over the ranks (see the module
    docstring); returns the ``mixed`` object (rank 0) or None."""
    import fastaf_kernel_b200 as fk
    from fastaf_kernel_b200 import sharding, workloads as W
    lengths = W.mixed_lengths(MIXED_SEED, MIXED_SEQS)
    plans = sharding.plan_prefill(lengths, world, 16, 32)
    mine = plans[rank].items
    spans = {(it.hq0, it.hq1) for it in mine}
    # 256 sequences on at most 8 ranks: whole sequences, every rank all heads
    assert len(spans) <= 1, "the mixed bench expects whole-sequence items"
    hq0, hq1 = spans.pop() if spans else (0, 16)
    seqs = [it.seq for it in mine]
    x = W.mixed_shard(lengths, seqs, MIXED_SEED, device=dev, hq0=hq0, hq1=hq1)
    n, T = len(seqs), int(x["cu_seqlens"][-1].item()) if seqs else 0
    Hq_r, Hv_r = hq1 - hq0, 2 * (hq1 - hq0)
    stream = torch.cuda.current_stream()
    pre_ms = dec_ms = 0.0
    if n:
        out = torch.empty((T, Hv_r, 128), dtype=torch.bfloat16, device=dev)
        ns = torch.empty((n, Hv_r, 128, 128), dtype=torch.float32, device=dev)

        def prefill():
            fk.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                      x["cu_seqlens"], x["scale"], output=out, new_state=ns)
    for _ in range(args.warmup):
        if n:
            prefill()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if n:
            prefill()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    pre_ms = e0.elapsed_time(e1) / args.steps
    if n:
        fk.device_status()
    # 1024 decode steps on this rank's resident states (in place), fresh q/k/v/a/b per
    # step, captured once as a CUDA graph (no host launch cost inside the timed replay)
    graph = None
    if n:
        state = ns
        steps_in = [W.decode_step_inputs(n, seed=50_000 + 7919 * rank + s, Hq=Hq_r, Hv=Hv_r, device=dev)
                    for s in range(MIXED_STEPS)]
        dout = torch.empty((n, 1, Hv_r, 128), dtype=torch.bfloat16, device=dev)

        def decode(s):
            st = steps_in[s]
            fk.kernel_decode(st["q"], st["k"], st["v"], state, x["A_log"], st["a"], x["dt_bias"], st["b"],
                             x["scale"], output=dout, new_state=state)
        for s in range(args.warmup):
            decode(s)
        torch.cuda.synchronize()
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cs):
            for s in range(MIXED_STEPS):
                decode(s)
        graph.replay()          # warm
        torch.cuda.synchronize()
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    if graph is not None:
        graph.replay()
    d1.record(stream)
    torch.cuda.synchronize()
    barrier()
    dec_ms = d0.elapsed_time(d1)
    del graph
    rows = gather([float(n), float(T), float(plans[rank].load), pre_ms, dec_ms])
    if rank != 0:
        return None
    pre = max(r[3] for r in rows)
    dec = max(r[4] for r in rows)
    total_tokens = sum(lengths)
    mean = lambda v: sum(v) / len(v)
    dec_bytes = MIXED_SEQS * W.bytes_per_decode_seq()
    return {
        "workload": f"gdn_mixed_{MIXED_SEQS}_loguniform_128_32768_then_{MIXED_STEPS}_decode_hq16_hv32_d128",
        "scaling": "strong", "n_seqs": MIXED_SEQS, "prefill_tokens": total_tokens,
        "parallelism": (f"sharded{world}: (sequence, v-head-group) items placed by plan_prefill "
                        "(longest first, least-loaded rank, load = tokens x v-heads); states stay on "
                        "their rank between prefill and decode; no data-path collective"),
        "prefill_tokens_per_s": total_tokens / (pre / 1e3), "prefill_ms": pre,
        "decode_seq_steps_per_s": MIXED_SEQS * MIXED_STEPS / (dec / 1e3), "decode_ms": dec,
        "decode_gbs": dec_bytes * MIXED_STEPS / (dec / 1e3) / 1e9,
        "decode_hbm_frac_per_gpu": dec_bytes * MIXED_STEPS / (dec / 1e3) / 1e9 / world / peaks["hbm_gbs"],
        "job_ms": pre + dec,
        "imbalance": {"planned_load_max_over_mean": max(r[2] for r in rows) / mean([r[2] for r in rows]),
                      "prefill_ms_max_over_mean": pre / mean([r[3] for r in rows]),
                      "decode_ms_max_over_mean": dec / mean([r[4] for r in rows])},
        "per_rank": [{"rank": i, "seqs": int(r[0]), "tokens": int(r[1]), "prefill_ms": r[3], "decode_ms": r[4]}
                     for i, r in enumerate(rows)],
        "timing": f"prefill: mean of {args.steps} calls after {args.warmup} warm-up calls; decode: one replay "
                  f"of a CUDA graph of {MIXED_STEPS} steps after a warm replay; max over ranks",
    }


def _time_calls(fn, calls=200, graph_calls=20, replays=10):
    """(ms per eager call, device ms per call from replays of a CUDA graph of `graph_calls`
    calls): the first includes the host cost of each call, the second only the device's."""
    for _ in range(20):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(calls):
        fn()
    e1.record()
    torch.cuda.synchronize()
    eager = e0.elapsed_time(e1) / calls
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(graph_calls):
                fn()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(replays):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    dev_ms = e0.elapsed_time(e1) / (replays * graph_calls)
    del graph
    return eager, dev_ms


def run_small_configs(args):
    """The two small configurations, one GPU: one B = 4 decode step (Hq 16, Hv 32, with
    state) and a varlen prefill of 4 sequences with lengths U[64, 512] (seed 1: 1,311
    tokens; sequences 1 and 3 with state).  Each through this library, through the
    reference's own Triton kernels compiled for sm_100 (oracle/ref_triton.py, when built)
    and through the reference's CPU torch implementation (oracle/gdn_ref.py) on all host
    threads.  Prints one JSON object."""
    import fastaf_kernel_b200 as fk
    from fastaf_kernel_b200 import workloads as W
    from oracle import gdn_ref, ref_triton
    torch.set_num_threads(os.cpu_count() or 1)
    dev = torch.device("cuda", 0)
    ref = ref_triton.RefTriton() if ref_triton.available() else None
    res = {"configs": "small", "cpu_threads": torch.get_num_threads(),
           "timing": "eager: CUDA events around 200 calls; graph: replays of a CUDA graph of 20 calls"}
    # decode, B = 4
    d = W.decode_inputs(4, seed=0)
    g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
    out = torch.empty((4, 1, 32, 128), dtype=torch.bfloat16, device=dev)
    ns = torch.empty_like(g["state"])
    nbytes = 4 * W.bytes_per_decode_seq()
    ours = _time_calls(lambda: fk.kernel_decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                                g["dt_bias"], g["b"], g["scale"], output=out, new_state=ns))
    dec = {"workload": "gdn_decode_b4_hq16_hv32_d128", "bytes_per_step": nbytes,
           "ours_ms": {"eager": ours[0], "graph": ours[1]}, "ours_gbs": nbytes / (ours[1] / 1e3) / 1e9}
    if ref is not None:
        o2 = out.view(4, 32, 128)
        rt = _time_calls(lambda: ref.decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                            g["dt_bias"], g["b"], g["scale"], o2, ns))
        dec["ref_triton_ms"] = {"eager": rt[0], "graph": rt[1]}
    t0 = time.perf_counter()
    for _ in range(5):
        gdn_ref.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], d["scale"])
    dec["cpu_torch_ms"] = (time.perf_counter() - t0) / 5 * 1e3
    res["decode_b4"] = dec
    # varlen prefill, 4 sequences U[64, 512]
    x = W.prefill_varlen(seed=1)
    T = x["q"].shape[0]
    g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}
    out = torch.empty((T, 32, 128), dtype=torch.bfloat16, device=dev)
    ns = torch.empty((4, 32, 128, 128), device=dev)
    ours = _time_calls(lambda: fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"],
                                         g["b"], g["cu_seqlens"], g["scale"], output=out, new_state=ns))
    pre = {"workload": f"gdn_prefill_varlen_4seqs_{T}tok_hq16_hv32_d128", "tokens": T,
           "method": fk.prefill_method(T, num_seqs=4), "ours_ms": {"eager": ours[0], "graph": ours[1]},
           "ours_tokens_per_s": T / (ours[1] / 1e3)}
    if ref is not None:
        rt = _time_calls(lambda: ref.prefill(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                             g["dt_bias"], g["b"], g["cu_seqlens"], g["scale"], out, ns),
                         calls=50)
        pre["ref_triton_ms"] = {"eager": rt[0], "graph": rt[1]}
    t0 = time.perf_counter()
    gdn_ref.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                    x["cu_seqlens"], x["scale"])
    pre["cpu_torch_ms"] = (time.perf_counter() - t0) * 1e3
    res["prefill_varlen"] = pre
    print(json.dumps(res))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--method", choices=["auto", "tcgen05", "chunked", "recurrent"], default="auto")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-mixed", action="store_true", help="skip the mixed prefill + decode workload")
    ap.add_argument("--no-cp", action="store_true", help="skip the context-parallel prefill (N > 1)")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip timing the reference's own Triton kernels on this GPU")
    ap.add_argument("--small-configs", action="store_true",
                    help="time only the B = 4 decode step and the 4-sequence varlen prefill (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return reference_arm(args)
    if args.small_configs:
        return run_small_configs(args)

    import torch.distributed as dist
    import fastaf_kernel_b200 as fk
    from fastaf_kernel_b200 import _lib, workloads as W
    from fastaf_kernel_b200.clocks import ClockSampler

    rank, world, local = dist_env()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            print("--gpus > 1 needs torchrun (one process per GPU)", file=sys.stderr)
            return 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()   # fail loudly if the CUDA library is missing
    peaks = load_peaks()

    def barrier():
        if world > 1:
            dist.barrier()

    def gather(row):
        """Per-rank rows of floats, on every rank (a sum of one-hot rows: no object pickling)."""
        t = torch.zeros((world, len(row)), dtype=torch.float64, device=dev)
        t[rank] = torch.tensor(row, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t)
        return t.cpu().tolist()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- prefill: inputs resident in HBM ----------------
    # this rank's 16 sequences of the global batch (plan_prefill gives each rank 16)
    from fastaf_kernel_b200 import sharding
    plan = sharding.plan_prefill([SEQ_LEN] * (N_SEQS * world), world, 16, 32)
    assert all(len(pl.items) == N_SEQS and all(it.hq1 - it.hq0 == 16 for it in pl.items) for pl in plan)
    x = W.prefill_long(seed=3 + rank, device=dev)
    T = N_SEQS * SEQ_LEN
    kernel_name = fk.prefill_method(T, args.method, N_SEQS)
    # the tcgen05 path is two launches per step (chunk prep, then the chains), four when
    # the library splits off the last partial wave of chains onto its second stream, one
    # more when it ranks the sequences longest first (the library's own rule,
    # gdn_prefill_tc_launches: five for 16 x 8192 on 148 SMs)
    launches_per_step = 1
    if kernel_name == "tcgen05":
        from fastaf_kernel_b200 import _lib
        launches_per_step = _lib.load().gdn_prefill_tc_launches(
            N_SEQS, 16, 32, torch.cuda.get_device_properties(dev).multi_processor_count)
    out = torch.empty((T, 32, 128), dtype=torch.bfloat16, device=dev)
    ns = torch.empty((N_SEQS, 32, 128, 128), dtype=torch.float32, device=dev)

    def prefill_step():
        fk.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                  x["b"], x["cu_seqlens"], x["scale"], output=out, new_state=ns,
                  method=args.method)

    for _ in range(args.warmup):
        prefill_step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(local, period_ms=50).__enter__()
    evs[0].record(stream)
    for i in range(args.steps):
        prefill_step()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    barrier()
    launch_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    total_ms = max_over_ranks(evs[0].elapsed_time(evs[-1]))
    ms_per_step = total_ms / args.steps
    value = world * T * args.steps / (total_ms / 1e3)
    flops = T * W.prefill_flops_per_token()
    avg_launch_s = sum(launch_ms) / len(launch_ms) / 1e3
    achieved_tflops = flops / avg_launch_s / 1e12
    pbytes = W.prefill_bytes(T, N_SEQS, N_SEQS)
    roofline = {"bound": "tensor", "achieved": achieved_tflops, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved_tflops / peaks["bf16_tflops"],
                "traffic": (lambda b: None if b is None else b * T)(
                    profiled_traffic("ncu_prefill_" + kernel_name + "_16x4096")),
                "peak_source": peaks["source"],
                "kernel": "gdn prefill (" + kernel_name + ")",
                "flops_per_launch": flops, "algorithmic_bytes_per_launch": pbytes,
                "hbm_gbs_achieved": pbytes / avg_launch_s / 1e9,
                "hbm_frac": pbytes / avg_launch_s / 1e9 / peaks["hbm_gbs"]}

    # ---------------- decode: B=512, in place, fresh inputs per step ----------------
    d0 = W.decode_inputs(DECODE_B, seed=2 + 1000 * rank, device=dev)
    dstate = d0["state"]
    dsteps = [W.decode_step_inputs(DECODE_B, seed=10_000 + s + 1000 * rank, device=dev)
              for s in range(DECODE_STEPS)]
    dout = torch.empty((DECODE_B, 1, 32, 128), dtype=torch.bfloat16, device=dev)

    def decode_step(s):
        st = dsteps[s % DECODE_STEPS]
        fk.kernel_decode(st["q"], st["k"], st["v"], dstate, d0["A_log"], st["a"],
                         d0["dt_bias"], st["b"], d0["scale"], output=dout, new_state=dstate)

    for s in range(args.warmup):
        decode_step(s)
    torch.cuda.synchronize()
    barrier()
    dev0 = torch.cuda.Event(enable_timing=True)
    dev1 = torch.cuda.Event(enable_timing=True)
    dev0.record(stream)
    for s in range(DECODE_STEPS):
        decode_step(s)
    dev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    dec_ms = max_over_ranks(dev0.elapsed_time(dev1))
    dec_step_s = dec_ms / 1e3 / DECODE_STEPS
    dec_bytes = DECODE_B * W.bytes_per_decode_seq()
    dec_gbs = dec_bytes / dec_step_s / 1e9
    decode = {"value": world * dec_gbs, "unit": "GB/s", "per_gpu_gbs": dec_gbs,
              "seq_per_s": world * DECODE_B / dec_step_s, "ms_per_step": dec_step_s * 1e3,
              "steps": DECODE_STEPS,
              "roofline": {"bound": "hbm", "achieved": dec_gbs, "peak": peaks["hbm_gbs"],
                           "unit": "GB/s", "frac": dec_gbs / peaks["hbm_gbs"],
                           "traffic": (lambda b: None if b is None else b * DECODE_B)(
                               profiled_traffic("ncu_decode_b512")),
                           "peak_source": peaks["source"],
                           "bytes_per_launch": dec_bytes}}

    # ---------------- the reference's own Triton kernels on this GPU (rank 0, N = 1) ----------------
    ref_gpu = None
    if rank == 0 and world == 1 and not args.no_ref_gpu:
        ref_gpu = reference_gpu_leg(args, x, out, ns, d0, dsteps, dout, value, dec_gbs, stream)

    # ---------------- end to end through the public API, host buffers ----------------
    e2e = None
    if not args.no_e2e:
        hx = {k: (v.cpu().pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in x.items()}
        h2d = sum(v.numel() * v.element_size() for v in hx.values() if isinstance(v, torch.Tensor))
        d2h = out.numel() * out.element_size() + ns.numel() * ns.element_size()
        # Two buffer sets and three streams, so step i+1's host->device copies and step
        # i-1's device->host copies overlap step i's compute (every step still copies
        # all of its inputs in and its output and new state out).
        sets = []
        for _ in range(2):
            sets.append({
                "x": {k: (torch.empty_like(v, device=dev) if isinstance(v, torch.Tensor) else v)
                      for k, v in hx.items()},
                "out": torch.empty_like(out), "ns": torch.empty_like(ns),
                "hout": torch.empty(out.shape, dtype=out.dtype, pin_memory=True),
                "hns": torch.empty(ns.shape, dtype=ns.dtype, pin_memory=True),
                "h2d": torch.cuda.Event(), "comp": torch.cuda.Event(), "d2h": torch.cuda.Event()})
        s_h2d, s_cmp, s_d2h = (torch.cuda.Stream(dev) for _ in range(3))

        def e2e_step(i):
            S = sets[i % 2]
            with torch.cuda.stream(s_h2d):
                s_h2d.wait_event(S["comp"])        # step i-2's compute has read this set
                for k2, v2 in hx.items():
                    if isinstance(v2, torch.Tensor):
                        S["x"][k2].copy_(v2, non_blocking=True)
                S["h2d"].record(s_h2d)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(S["h2d"])
                s_cmp.wait_event(S["d2h"])         # step i-2's results have left this set
                d = S["x"]
                fk.kernel(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                          d["cu_seqlens"], d["scale"], output=S["out"], new_state=S["ns"],
                          method=args.method)
                S["comp"].record(s_cmp)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(S["comp"])
                S["hout"].copy_(S["out"], non_blocking=True)
                S["hns"].copy_(S["ns"], non_blocking=True)
                S["d2h"].record(s_d2h)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        # up to 12 steps (each ~45 ms, bound by the 2.2 GB host->device copy), so the one
        # trailing device->host copy of the drain weighs less on the throughput
        n_e2e = max(2, min(args.steps, 12))
        e0.record(s_h2d)
        for i in range(n_e2e):
            e2e_step(i)
        e1.record(s_d2h)
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": world * T * n_e2e / (e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": n_e2e,
               "path": "pinned host -> device copies, fastaf_kernel_b200.kernel (default arguments), device -> "
                       "pinned host copies of output and new_state; two buffer sets on three "
                       "streams, so one step's copies overlap the neighbouring steps' compute"}

    clk.__exit__(None, None, None)

    # ---------------- mixed prefill + decode workload, strong-scaled ----------------
    mixed = None
    if not args.no_mixed:
        del x, out, ns, dsteps, d0, dstate, dout
        if e2e is not None:
            del sets, hx
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        mixed = run_mixed(args, rank, world, dev, barrier, gather, peaks)

    # ---------------- one long sequence over all ranks (N > 1) ----------------
    cpar = None
    if world > 1 and not args.no_cp:
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        cpar = run_context_parallel(args, rank, world, dev, barrier, gather)

    # ---------------- CPU baseline (rank 0, one GPU only) ----------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import c_oracle
        threads = os.cpu_count() or 1
        tps, n_tok, n_seq, dt = cpu_prefill_sample(
            lambda *a: c_oracle.prefill(*a, num_threads=threads), args.cpu_budget)
        cpu = {"value": tps, "unit": UNIT, "cores": threads, "kind": "port",
               "impl": "oracle/gdn_oracle.c (fp32 recurrence, OpenMP over (sequence, v-head))",
               "sample": f"first {n_tok} tokens ({n_seq} sequences) of the {N_SEQS}x{SEQ_LEN} "
                         f"workload, 32 v-heads, nonzero state ({dt:.1f} s)"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded; shapes and distributions of "
                                         "the benchmark configurations)",
                "config": base_config(world), "roofline": roofline, "cpu_baseline": cpu,
                "e2e": e2e, "gpu_launches": args.steps * launches_per_step, "clocks": clk.summary(),
                "decode": decode, "mixed": mixed, "context_parallel": cpar, "reference_gpu": ref_gpu,
                "launch_ms": launch_ms}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
