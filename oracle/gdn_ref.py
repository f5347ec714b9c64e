"""CPU oracle for the Gated DeltaNet prefill/decode path (test infrastructure only).

This module is the CHECKER, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``fastaf_kernel_b200``) never routes through it.

It restates, in plain fp32 PyTorch on the CPU, the reference's torch
implementation of the gated delta rule:

  * ``solution/gdn_baseline_torch.py:12-91``  (``run``; Hq=Hk=16, Hv=32)
  * ``local_test/origina_gdn_prefill.py:20-98`` (same math for Hq=Hk=4, Hv=8,
    TF32 disabled in its matmul, ``:6-16``)

with the head-count asserts (``gdn_baseline_torch.py:33-36``) lifted so the
same code serves every GVA shape.  The per-token update keeps the reference's
operation order:

  g    = exp(-exp(A_log) * softplus(a + dt_bias))      (``:42-43``)
  beta = sigmoid(b)                                      (``:44``)
  S'   = g * S                                           (``:79``)
  u    = k @ S'                                          (``:80``)
  v'   = beta * v + (1 - beta) * u                       (``:81``)
  S    = S' - k^T u + k^T v'                             (``:82-84``)
  o    = scale * q @ S                                   (``:86-87``)

with S held in [H, K, V] inside the loop and returned k-last [H, V, K]
(``:65``, ``:89``).  A sequence of length 0 leaves its new_state at zero
(``:61-62``), and ``scale`` of None/0 means 1/sqrt(D) (``:38-39``).

Parity of this restatement is pinned against outputs of the reference's own
``run`` committed under ``tests/golden/`` (see ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

__all__ = ["gates", "prefill", "decode"]


def gates(A_log: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor,
          b: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-token decay g and write strength beta, in fp32.

    Follows ``solution/gdn_baseline_torch.py:42-44``: torch's ``F.softplus``
    (beta=1, threshold=20) and ``torch.sigmoid``.
    """
    x = a.float() + dt_bias.float()
    g = torch.exp(-torch.exp(A_log.float()) * F.softplus(x))
    beta = torch.sigmoid(b.float())
    return g, beta


def _matmul_fp32(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    # fp32 matmul on the CPU; the reference disables TF32 for the same reason
    # (local_test/origina_gdn_prefill.py:6-16).  CPU matmul never uses TF32.
    return x.float() @ y.float()


@torch.no_grad()
def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
            state: Optional[torch.Tensor], A_log: torch.Tensor, a: torch.Tensor,
            dt_bias: torch.Tensor, b: torch.Tensor, cu_seqlens: torch.Tensor,
            scale: Optional[float]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Varlen prefill oracle.

    Shapes (packed varlen, as ``solution/triton/kernel.py:416-431``):
      q, k  [T, Hq, D] (Hk == Hq), v [T, Hv, D], a, b [T, Hv],
      A_log, dt_bias [Hv], state [N, Hv, D(V), D(K)] fp32 or None,
      cu_seqlens [N+1].
    Returns (output [T, Hv, D] bf16, new_state [N, Hv, D, D] fp32).
    """
    q = q.cpu(); k = k.cpu(); v = v.cpu(); a = a.cpu(); b = b.cpu()
    A_log = A_log.cpu(); dt_bias = dt_bias.cpu(); cu_seqlens = cu_seqlens.cpu()
    if state is not None:
        state = state.cpu()
    T, Hq, D = q.shape
    Hk = k.shape[1]
    Hv = v.shape[1]
    if Hv % Hq or Hv % Hk:
        raise ValueError(f"Hv={Hv} must be a multiple of Hq={Hq} and Hk={Hk}")
    H = max(Hq, Hv)
    N = cu_seqlens.numel() - 1
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)

    g, beta = gates(A_log, a, dt_bias, b)                       # [T, Hv]
    q_exp = q.repeat_interleave(Hv // Hq, dim=1)                # :46
    k_exp = k.repeat_interleave(Hv // Hk, dim=1)                # :47

    output = torch.zeros((T, H, D), dtype=torch.bfloat16)
    new_state = torch.zeros((N, H, D, D), dtype=torch.float32)
    for n in range(N):
        s0 = int(cu_seqlens[n].item())
        s1 = int(cu_seqlens[n + 1].item())
        if s1 - s0 <= 0:
            continue                                            # :61-62
        if state is not None:
            S = state[n].clone().float().transpose(-1, -2)      # [H,K,V]
        else:
            S = torch.zeros((H, D, D), dtype=torch.float32)
        for t in range(s0, s1):
            q_t = q_exp[t].unsqueeze(1).float()                 # [H,1,K]
            k_t = k_exp[t].unsqueeze(1).float()
            v_t = v[t].unsqueeze(1).float()                     # [H,1,V]
            g_t = g[t].view(H, 1, 1)
            b_t = beta[t].view(H, 1, 1)
            S_dec = g_t * S
            u = _matmul_fp32(k_t, S_dec)                        # [H,1,V]
            v_new = b_t * v_t + (1 - b_t) * u
            k_col = k_t.transpose(-1, -2)                       # [H,K,1]
            S = S_dec - k_col @ u + k_col @ v_new
            output[t] = (scale * _matmul_fp32(q_t, S)).squeeze(1).to(torch.bfloat16)
        new_state[n] = S.transpose(-1, -2)                      # [H,V,K]
    return output, new_state


@torch.no_grad()
def decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
           state: Optional[torch.Tensor], A_log: torch.Tensor, a: torch.Tensor,
           dt_bias: torch.Tensor, b: torch.Tensor,
           scale: Optional[float]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Single-token decode oracle: the prefill recurrence with T=1 per sequence.

    Shapes follow ``solution/triton/kernel.py:492-506``: q, k [B,1,Hq,D],
    v [B,1,Hv,D], a, b [B,1,Hv], state [B,Hv,D,D] or None.
    Returns (output [B,1,Hv,D] bf16, new_state [B,Hv,D,D] fp32).
    """
    B = q.shape[0]
    Hq, D = q.shape[2], q.shape[3]
    Hv = v.shape[2]
    cu = torch.arange(B + 1, dtype=torch.int32)
    out, ns = prefill(q.reshape(B, Hq, D), k.reshape(B, k.shape[2], D),
                      v.reshape(B, Hv, D), state, A_log, a.reshape(B, Hv),
                      dt_bias, b.reshape(B, Hv), cu, scale)
    return out.unsqueeze(1), ns
