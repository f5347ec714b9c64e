"""Partitioning of the Gated DeltaNet path across GPUs: one process per GPU.

The recurrence has no reduction across sequences or v-heads
(solution/gdn_baseline_torch.py:56-89 runs every (sequence, head) chain
independently), so the box is used as independent shards with no data-path
collective: every rank gets whole (sequence, v-head-group) chains, keeps their
states in its own HBM between prefill and decode, and nothing crosses NVLink
except an optional gather of results for checking.

Work items are (sequence, head group).  Head groups are GVA-aligned: a group
holds whole q/k heads and the Hv/Hq v-heads that read them, so a rank receives
only the q/k heads it needs.  Heads are split only when there are fewer
sequences than ranks.  Items are placed longest-first on the least-loaded rank
(LPT), with load = tokens x v-heads, and each rank's items stay longest first.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch


@dataclass(frozen=True)
class WorkItem:
    seq: int          # sequence index in the packed batch
    hq0: int          # q/k heads [hq0, hq1)
    hq1: int
    tokens: int

    def v_heads(self, ratio: int) -> range:
        return range(self.hq0 * ratio, self.hq1 * ratio)


@dataclass
class RankPlan:
    rank: int
    items: List[WorkItem] = field(default_factory=list)
    load: int = 0


def head_groups(num_seqs: int, world: int, Hq: int) -> int:
    """Number of q/k-head groups per sequence: the smallest divisor g of Hq with
    num_seqs * g >= world (1 when there are at least as many sequences as ranks)."""
    if num_seqs <= 0:
        return 1
    for g in range(1, Hq + 1):
        if Hq % g == 0 and num_seqs * g >= world:
            return g
    return Hq


def plan_prefill(lengths: Sequence[int], world: int, Hq: int, Hv: int) -> List[RankPlan]:
    """LPT placement of (sequence, head-group) items on `world` ranks."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if Hv % Hq:
        raise ValueError("Hv must be a multiple of Hq")
    ratio = Hv // Hq
    g = head_groups(len(lengths), world, Hq)
    per = Hq // g
    items = [WorkItem(s, j * per, (j + 1) * per, int(L))
             for s, L in enumerate(lengths) for j in range(g)]
    items.sort(key=lambda it: (-(it.tokens * (it.hq1 - it.hq0)), it.seq, it.hq0))
    plans = [RankPlan(r) for r in range(world)]
    heap = [(0, r) for r in range(world)]
    for it in items:
        load, r = heapq.heappop(heap)
        plans[r].items.append(it)
        plans[r].load = load + it.tokens * (it.hq1 - it.hq0) * ratio
        heapq.heappush(heap, (plans[r].load, r))
    # Each rank's batch runs longest first: its chains are scheduled in batch order on the
    # GPU's SMs, and a long sequence late in the batch would start its chains last and keep
    # a few SMs busy after all others are done (list scheduling of the 256 log-uniform
    # sequences on 8 ranks x 148 SMs: the slowest rank's chain phase 963 chunk-times in
    # sequence order, 660 longest first, against a 658 lower bound).
    for pl in plans:
        pl.items.sort(key=lambda it: (-it.tokens, it.seq, it.hq0))
    return plans


def plan_decode(batch: int, world: int, Hq: int, Hv: int) -> List[RankPlan]:
    """Decode: every sequence costs the same, so this is plan_prefill with unit lengths."""
    return plan_prefill([1] * batch, world, Hq, Hv)


def _head_uniform(items: List[WorkItem]) -> Optional[range]:
    spans = {(it.hq0, it.hq1) for it in items}
    return range(*spans.pop()) if len(spans) == 1 else None


def shard_prefill_inputs(x: Dict[str, torch.Tensor], plan: RankPlan, Hq: int, Hv: int):
    """Slice packed varlen inputs down to one rank's items.

    Returns a list of (inputs, items) groups, one per distinct head span, each
    a self-contained packed batch for ``kernel(...)``."""
    ratio = Hv // Hq
    cu = x["cu_seqlens"].to("cpu", torch.int64)
    by_span: Dict[tuple, List[WorkItem]] = {}
    for it in plan.items:
        by_span.setdefault((it.hq0, it.hq1), []).append(it)
    out = []
    for (hq0, hq1), items in sorted(by_span.items()):
        seqs = [it.seq for it in items]
        idx = torch.cat([torch.arange(int(cu[s]), int(cu[s + 1])) for s in seqs]) if seqs else \
            torch.zeros(0, dtype=torch.int64)
        dev = x["q"].device
        idx_d = idx.to(dev)
        h0, h1 = hq0 * ratio, hq1 * ratio
        lens = [int(cu[s + 1] - cu[s]) for s in seqs]
        new_cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
        if seqs:
            new_cu[1:] = torch.cumsum(torch.tensor(lens), 0).to(torch.int32)
        sub = {
            "q": x["q"].index_select(0, idx_d)[:, hq0:hq1].contiguous(),
            "k": x["k"].index_select(0, idx_d)[:, hq0:hq1].contiguous(),
            "v": x["v"].index_select(0, idx_d)[:, h0:h1].contiguous(),
            "a": x["a"].index_select(0, idx_d)[:, h0:h1].contiguous(),
            "b": x["b"].index_select(0, idx_d)[:, h0:h1].contiguous(),
            "A_log": x["A_log"][h0:h1].contiguous(),
            "dt_bias": x["dt_bias"][h0:h1].contiguous(),
            "state": None if x.get("state") is None else
            x["state"][torch.tensor(seqs, dtype=torch.int64, device=x["state"].device)][:, h0:h1].contiguous(),
            "cu_seqlens": new_cu.to(x["cu_seqlens"].device),
            "scale": x.get("scale", 0.0),
        }
        out.append((sub, items, idx))
    return out


def scatter_prefill_outputs(output: torch.Tensor, new_state: torch.Tensor, group_results,
                            Hq: int, Hv: int) -> None:
    """Write per-group (sub_output, sub_new_state) back into full-size buffers."""
    ratio = Hv // Hq
    for (sub_out, sub_state), items, idx in group_results:
        hq0, hq1 = items[0].hq0, items[0].hq1
        h0, h1 = hq0 * ratio, hq1 * ratio
        output[idx.to(output.device), h0:h1] = sub_out.to(output.device)
        for j, it in enumerate(items):
            new_state[it.seq, h0:h1] = sub_state[j].to(new_state.device)
