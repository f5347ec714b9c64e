"""Seeded synthetic Gated DeltaNet workloads (the benchmark and test inputs).

No contest dataset is available offline, so inputs are drawn with the shapes
and value distributions of the five benchmark configurations:

  decode_b4        B=4 decode step, Hq=Hk=16, Hv=32, D=128
  prefill_varlen   4 sequences, lengths U[64, 512], half with a zero state
  decode_b512      B=512 decode, 100 steps, fresh q/k/v/a/b per step, in-place state
  prefill_long     16 x 8192 tokens, nonzero state, per-token decay in [0.5, 0.999]
  mixed            256 sequences, log-uniform lengths in [128, 32768], then 1024 decode
                   steps on the resident states (mixed_lengths, mixed_shard: any shard of it)

Distributions: q, k ~ N(0,1) L2-normalised per head, then bf16; v ~ N(0,1) bf16;
a, b ~ N(0,1) bf16; A_log = log U(1,16) fp32; dt_bias ~ U(-1,1) fp32;
state ~ N(0, 0.02^2) fp32 (k-last [.., V, K]); scale = 1/sqrt(128).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

D = 128
HQ = 16
HV = 32
STATE_STD = 0.02


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _normal(shape, g, device, std=1.0):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def _unit_bf16(shape, g, device):
    x = _normal(shape, g, device)
    return torch.nn.functional.normalize(x, dim=-1).to(torch.bfloat16)


def head_params(seed: int, Hv: int = HV, device="cpu"):
    """A_log = log U(1,16), dt_bias ~ U(-1,1), both fp32 [Hv]."""
    g = _gen(seed, device)
    A_log = torch.log(torch.rand(Hv, generator=g, device=device) * 15.0 + 1.0)
    dt_bias = torch.rand(Hv, generator=g, device=device) * 2.0 - 1.0
    return A_log, dt_bias


def decode_inputs(B: int, seed: int, Hq: int = HQ, Hv: int = HV, device="cpu",
                  with_state: bool = True, params=None) -> Dict[str, torch.Tensor]:
    """One decode step: q,k [B,1,Hq,D], v [B,1,Hv,D], a,b [B,1,Hv], state [B,Hv,D,D]."""
    g = _gen(seed, device)
    A_log, dt_bias = params if params is not None else head_params(seed + 1_000_003, Hv, device)
    out = {
        "q": _unit_bf16((B, 1, Hq, D), g, device),
        "k": _unit_bf16((B, 1, Hq, D), g, device),
        "v": _normal((B, 1, Hv, D), g, device).to(torch.bfloat16),
        "a": _normal((B, 1, Hv), g, device).to(torch.bfloat16),
        "b": _normal((B, 1, Hv), g, device).to(torch.bfloat16),
        "A_log": A_log,
        "dt_bias": dt_bias,
        "state": _normal((B, Hv, D, D), g, device, STATE_STD) if with_state else None,
        "scale": 1.0 / math.sqrt(D),
    }
    return out


def decode_step_inputs(B: int, seed: int, Hq: int = HQ, Hv: int = HV, device="cpu"):
    """Fresh per-step q/k/v/a/b (no state) for multi-step decode loops."""
    g = _gen(seed, device)
    return {
        "q": _unit_bf16((B, 1, Hq, D), g, device),
        "k": _unit_bf16((B, 1, Hq, D), g, device),
        "v": _normal((B, 1, Hv, D), g, device).to(torch.bfloat16),
        "a": _normal((B, 1, Hv), g, device).to(torch.bfloat16),
        "b": _normal((B, 1, Hv), g, device).to(torch.bfloat16),
    }


def prefill_inputs(lengths: List[int], seed: int, Hq: int = HQ, Hv: int = HV, device="cpu",
                   state_mask: Optional[List[bool]] = None,
                   decay_range: Optional[tuple] = None) -> Dict[str, torch.Tensor]:
    """Packed varlen prefill inputs for the given sequence lengths.

    state_mask[i] False gives sequence i a zero initial state; None of the mask
    entries True means ``state`` is None.  decay_range=(lo, hi) draws the
    per-token decay alpha ~ U(lo, hi) and inverts the gate for ``a`` (then
    rounds ``a`` to bf16), so alpha spans that range."""
    g = _gen(seed, device)
    T = int(sum(lengths))
    N = len(lengths)
    A_log, dt_bias = head_params(seed + 1_000_003, Hv, device)
    cu = torch.zeros(N + 1, dtype=torch.int32)
    if N:
        cu[1:] = torch.cumsum(torch.tensor(lengths, dtype=torch.int64), 0).to(torch.int32)
    q = _unit_bf16((T, Hq, D), g, device)
    k = _unit_bf16((T, Hq, D), g, device)
    v = _normal((T, Hv, D), g, device).to(torch.bfloat16)
    if decay_range is not None:
        lo, hi = decay_range
        alpha = torch.rand((T, Hv), generator=g, device=device) * (hi - lo) + lo
        sp = -torch.log(alpha) / torch.exp(A_log)            # softplus(a + dt_bias)
        x = sp + torch.log(-torch.expm1(-sp))                # softplus^{-1}(sp), stable
        a = (x - dt_bias).to(torch.bfloat16)
    else:
        a = _normal((T, Hv), g, device).to(torch.bfloat16)
    b = _normal((T, Hv), g, device).to(torch.bfloat16)
    if state_mask is None:
        state_mask = [True] * N
    state = None
    if any(state_mask):
        state = _normal((N, Hv, D, D), g, device, STATE_STD)
        for i, m in enumerate(state_mask):
            if not m:
                state[i].zero_()
    return {"q": q, "k": k, "v": v, "state": state, "A_log": A_log, "a": a,
            "dt_bias": dt_bias, "b": b, "cu_seqlens": cu.to(device), "scale": 1.0 / math.sqrt(D)}


def varlen_lengths(seed: int, n: int = 4, lo: int = 64, hi: int = 512) -> List[int]:
    g = _gen(seed, "cpu")
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=g)]


def loguniform_lengths(seed: int, n: int = 256, lo: int = 128, hi: int = 32768) -> List[int]:
    g = _gen(seed, "cpu")
    u = torch.rand(n, generator=g, dtype=torch.float64)
    return [int(round(math.exp(math.log(lo) + float(x) * (math.log(hi) - math.log(lo))))) for x in u]


def mixed_lengths(seed: int = 4, n: int = 256) -> List[int]:
    """Sequence lengths of the mixed prefill + decode workload: 256 log-uniform in
    [128, 32768] (1.55 M tokens at seed 4)."""
    return loguniform_lengths(seed, n=n)


def mixed_shard(lengths: List[int], seqs: List[int], seed: int, device="cpu", hq0: int = 0,
                hq1: int = HQ, Hq: int = HQ, Hv: int = HV) -> Dict[str, torch.Tensor]:
    """Packed prefill inputs of sequences `seqs` (in that order) of the mixed workload,
    restricted to q/k heads [hq0, hq1) and their v-heads.  Sequence i is drawn from its
    own seed (seed * 1_000_003 + i) and the head parameters from `seed`, so a sequence's
    inputs are the same whichever rank holds it: every sharding of the batch computes
    the same workload.  Every sequence has a nonzero N(0, 0.02^2) initial state."""
    ratio = Hv // Hq
    h0, h1 = hq0 * ratio, hq1 * ratio
    A_log, dt_bias = head_params(seed + 1_000_003, Hv, device)
    parts = {k: [] for k in ("q", "k", "v", "a", "b", "state")}
    for i in seqs:
        L = int(lengths[i])
        g = _gen(seed * 1_000_003 + i, device)
        parts["q"].append(_unit_bf16((L, Hq, D), g, device)[:, hq0:hq1])
        parts["k"].append(_unit_bf16((L, Hq, D), g, device)[:, hq0:hq1])
        parts["v"].append(_normal((L, Hv, D), g, device).to(torch.bfloat16)[:, h0:h1])
        parts["a"].append(_normal((L, Hv), g, device).to(torch.bfloat16)[:, h0:h1])
        parts["b"].append(_normal((L, Hv), g, device).to(torch.bfloat16)[:, h0:h1])
        parts["state"].append(_normal((1, Hv, D, D), g, device, STATE_STD)[:, h0:h1])
    n = len(seqs)
    cu = torch.zeros(n + 1, dtype=torch.int32)
    if n:
        cu[1:] = torch.cumsum(torch.tensor([int(lengths[i]) for i in seqs], dtype=torch.int64), 0).to(torch.int32)
    out = {k: (torch.cat(v).contiguous() if v else None) for k, v in parts.items()}
    out.update({"A_log": A_log[h0:h1].contiguous(), "dt_bias": dt_bias[h0:h1].contiguous(),
                "cu_seqlens": cu.to(device), "scale": 1.0 / math.sqrt(D)})
    return out


def prefill_varlen(seed: int = 1, device="cpu", Hq: int = HQ, Hv: int = HV):
    """4 sequences with lengths U[64,512]; sequences 1 and 3 carry an initial state."""
    lengths = varlen_lengths(seed)
    return prefill_inputs(lengths, seed, Hq, Hv, device, state_mask=[False, True, False, True])


def prefill_long(seed: int = 3, device="cpu", n_seqs: int = 16, seq_len: int = 8192,
                 Hq: int = HQ, Hv: int = HV):
    """16 x 8192 tokens, nonzero initial state, per-token decay in [0.5, 0.999]."""
    return prefill_inputs([seq_len] * n_seqs, seed, Hq, Hv, device, decay_range=(0.5, 0.999))


def bytes_per_decode_seq(Hq: int = HQ, Hv: int = HV) -> int:
    """Algorithmic HBM bytes of one (sequence, step): state read+write, q/k/v/o, a/b."""
    return Hv * D * D * 4 * 2 + 2 * Hq * D * 2 + Hv * D * 2 * 2 + 2 * Hv * 2


def prefill_flops_per_token(Hq: int = HQ, Hv: int = HV, C: int = 64) -> int:
    """Canonical FLOPs/token of the chunked (C=64) algorithm:
    Hv*(6*C*D + 6*D^2 + C^2/3) + Hk*(4*C*D)."""
    return Hv * (6 * C * D + 6 * D * D + (C * C) // 3) + Hq * (4 * C * D)


def prefill_bytes(T: int, n_seqs_with_state: int, n_seqs: int, Hq: int = HQ, Hv: int = HV) -> int:
    """Algorithmic HBM bytes of a prefill: q,k,v,o bf16 + a,b bf16 per token, the
    final state written per sequence, the initial state read where present."""
    per_tok = 2 * Hq * D * 2 + 2 * Hv * D * 2 + 2 * Hv * 2
    st = Hv * D * D * 4
    return T * per_tok + n_seqs * st + n_seqs_with_state * st
