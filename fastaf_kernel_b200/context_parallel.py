"""Context-parallel prefill of one long sequence: the sequence is cut into segments
that are computed at the same time -- on one GPU, or spread over the GPUs of a
process group -- and joined by a scan over the segments' state maps.

For one v-head the recurrence is affine in the state (k-last S[v][k],
solution/gdn_baseline_torch.py:79-84):

    S_t = S_{t-1} A_t + B_t,   A_t = alpha_t (I - beta_t k_t k_t^T),  B_t = beta_t v_t k_t^T

so a segment maps its initial state S to  S M + C  with

    M = prod_t A_t  -- the segment's final state from initial state I with v = 0,
    C               -- the segment's final state from initial state 0.

Both are ordinary prefill calls over the segments.  The scan

    S_start(0) = state,   S_start(p + 1) = S_start(p) M_p + C_p

runs in float64 on the device, and a last prefill of every segment from its
S_start gives the outputs and the final state.  That is three passes over the
tokens instead of one, traded for parallelism: a single sequence otherwise keeps
only one chain per v-head (32 of the GPU's 148 SMs at Hv = 32) busy for its whole
length.  Across GPUs each rank takes a contiguous slice of the sequence, reduces
its segments to one map (M, C), and the ranks exchange those maps -- 2 x Hv x
128 x 128 float64 per rank -- in one all-gather; that is the only data the
recurrence sends between GPUs.

The per-segment work is whatever ``prefill_fn`` does (by default this library's
CUDA prefill, ``fastaf_kernel_b200.kernel``); the functions here only cut, scan
and join.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch

Prefill = Callable[..., Tuple[torch.Tensor, torch.Tensor]]


def _default_prefill(method: str) -> Prefill:
    from . import api

    def run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale):
        return api.kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, method=method)
    return run


def segment_bounds(T: int, segments: int, align: int = 64) -> List[int]:
    """Cut points 0 = s_0 < s_1 < ... < s_P = T of P nearly equal segments, the inner
    cuts on multiples of ``align`` tokens (whole chunks).  Fewer segments are returned
    when T is too short for P aligned ones."""
    if T < 0 or segments < 1 or align < 1:
        raise ValueError("need T >= 0, segments >= 1, align >= 1")
    bounds = [0]
    for p in range(1, segments):
        cut = (T * p // segments) // align * align
        if bounds[-1] < cut < T:
            bounds.append(cut)
    bounds.append(T)
    return bounds


def segment_maps(q, k, v, A_log, a, dt_bias, b, bounds: Sequence[int], scale,
                 prefill_fn: Prefill) -> Tuple[torch.Tensor, torch.Tensor]:
    """(M, C) [P, Hv, D, D] float32 of the segments [bounds[p], bounds[p+1]) of one
    sequence: two prefill calls (initial state 0 with the real v; initial state I with
    v = 0), each over all P segments at once."""
    P = len(bounds) - 1
    Hv, D = v.shape[1], v.shape[2]
    dev = q.device
    cu = torch.tensor(bounds, dtype=torch.int32, device=dev)
    _, C = prefill_fn(q, k, v, None, A_log, a, dt_bias, b, cu, scale)
    eye = torch.eye(D, dtype=torch.float32, device=dev).expand(P, Hv, D, D).contiguous()
    _, M = prefill_fn(q, k, torch.zeros_like(v), eye, A_log, a, dt_bias, b, cu, scale)
    return M, C


def compose(M: torch.Tensor, C: torch.Tensor, state0: Optional[torch.Tensor]):
    """Scan of the maps (float64): returns (starts [P, Hv, D, D], end [Hv, D, D]) with
    starts[0] = state0 (zero if None) and starts[p + 1] = starts[p] M_p + C_p."""
    P, Hv, D = M.shape[0], M.shape[1], M.shape[2]
    S = (torch.zeros((Hv, D, D), dtype=torch.float64, device=M.device) if state0 is None
         else state0.reshape(Hv, D, D).to(torch.float64))
    starts = []
    for p in range(P):
        starts.append(S)
        S = torch.matmul(S, M[p].to(torch.float64)) + C[p].to(torch.float64)
    return torch.stack(starts), S


def compose_maps(M: torch.Tensor, C: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """The single map (M_0 M_1 ... M_{P-1}, C') of P consecutive segments, float64."""
    Hv, D = M.shape[1], M.shape[2]
    Mt = torch.eye(D, dtype=torch.float64, device=M.device).expand(Hv, D, D).clone()
    Ct = torch.zeros((Hv, D, D), dtype=torch.float64, device=M.device)
    for p in range(M.shape[0]):
        Mp = M[p].to(torch.float64)
        Mt = torch.matmul(Mt, Mp)
        Ct = torch.matmul(Ct, Mp) + C[p].to(torch.float64)
    return Mt, Ct


def _check_single(q, v, state):
    if q.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be [T, H, D] (one sequence)")
    if state is not None and state.shape[0] != 1:
        raise ValueError("state must be [1, Hv, D, D] (one sequence) or None")


def prefill_segmented(q, k, v, state, A_log, a, dt_bias, b, scale, *, segments: int,
                      method: str = "auto", prefill_fn: Optional[Prefill] = None):
    """Prefill of ONE sequence (q, k [T, Hq, D], v [T, Hv, D], a, b [T, Hv], state
    [1, Hv, D, D] or None) as ``segments`` segments computed in parallel on this
    device.  Returns (output [T, Hv, D] bf16, new_state [1, Hv, D, D] fp32) -- the
    same as one prefill call with cu_seqlens = [0, T], up to rounding."""
    _check_single(q, v, state)
    fn = prefill_fn or _default_prefill(method)
    T = q.shape[0]
    bounds = segment_bounds(T, segments)
    if len(bounds) == 2:
        return fn(q, k, v, state, A_log, a, dt_bias, b,
                  torch.tensor([0, T], dtype=torch.int32, device=q.device), scale)
    M, C = segment_maps(q, k, v, A_log, a, dt_bias, b, bounds, scale, fn)
    starts, _ = compose(M, C, state)
    cu = torch.tensor(bounds, dtype=torch.int32, device=q.device)
    out, ns = fn(q, k, v, starts.to(torch.float32).contiguous(), A_log, a, dt_bias, b, cu, scale)
    return out, ns[-1:].contiguous()


def prefill_context_parallel(q, k, v, state, A_log, a, dt_bias, b, scale, *, group=None,
                             segments_per_rank: int = 1, method: str = "auto",
                             prefill_fn: Optional[Prefill] = None):
    """Prefill of ONE sequence spread over the ranks of ``group`` (torch.distributed;
    NCCL on GPUs).  Rank r passes its contiguous slice of the tokens -- slices in rank
    order make up the sequence -- and the sequence's initial ``state`` [1, Hv, D, D]
    (read on rank 0 only; None for zero).  Each rank cuts its slice into
    ``segments_per_rank`` segments.  Returns (output of this rank's slice, final state
    of the whole sequence [1, Hv, D, D] fp32 -- the same on every rank).

    Communication: one all-gather of every rank's (M, C) map and of rank 0's initial
    state (float64), then one broadcast of the final state from the last rank."""
    import torch.distributed as dist

    _check_single(q, v, state)
    fn = prefill_fn or _default_prefill(method)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T = q.shape[0]
    Hv, D = v.shape[1], v.shape[2]
    dev = q.device
    bounds = segment_bounds(T, segments_per_rank)
    if T > 0:
        M, C = segment_maps(q, k, v, A_log, a, dt_bias, b, bounds, scale, fn)
        Mr, Cr = compose_maps(M, C)
    else:
        Mr = torch.eye(D, dtype=torch.float64, device=dev).expand(Hv, D, D).clone()
        Cr = torch.zeros((Hv, D, D), dtype=torch.float64, device=dev)
    s0 = (torch.zeros((Hv, D, D), dtype=torch.float64, device=dev)
          if (rank != 0 or state is None) else state.reshape(Hv, D, D).to(torch.float64))
    mine = torch.stack([Mr, Cr, s0]).contiguous()
    gathered = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine, group=group)
    S = gathered[0][2]
    for r in range(rank):
        S = torch.matmul(S, gathered[r][0]) + gathered[r][1]
    if T > 0:
        starts, _ = compose(M, C, S)
        cu = torch.tensor(bounds, dtype=torch.int32, device=dev)
        out, ns = fn(q, k, v, starts.to(torch.float32).contiguous(), A_log, a, dt_bias, b, cu, scale)
        final = ns[-1].to(torch.float64)
    else:
        out = torch.empty((0, Hv, D), dtype=torch.bfloat16, device=dev)
        final = S
    if rank == world - 1:
        fin = final.contiguous()
    else:
        fin = torch.empty((Hv, D, D), dtype=torch.float64, device=dev)
    dist.broadcast(fin, src=dist.get_global_rank(group, world - 1) if group is not None else world - 1,
                   group=group)
    return out, fin.to(torch.float32).reshape(1, Hv, D, D)
