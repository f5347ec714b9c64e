"""Golden-fixture cases: input specs and their deterministic input generator.

Inputs are regenerated from a numpy PCG64 seed (a SHA-256 of the generated
bytes is stored with each fixture, so a drift in the generator fails loudly);
outputs were produced by the reference's own torch implementation
(``solution/gdn_baseline_torch.py:run`` for Hq=Hk=16/Hv=32 and
``local_test/origina_gdn_prefill.py:run`` for Hq=Hk=4/Hv=8) by
``make_golden.py`` and are stored in ``<name>.npz``:
  out        bf16 output as uint16 (full)
  state_idx  flat indices of the sampled new_state elements
  state_val  new_state at those indices (fp32; every element for small cases)
  state_sum  float64 sums of new_state per (sequence, head)
  input_sha  SHA-256 of the regenerated inputs
"""

from __future__ import annotations

import hashlib
import os
from typing import Dict, List

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
D = 128

# name -> spec.  kind: 'prefill' | 'decode'.  dist: 'reftest' draws every input
# from randn like local_test/test_cuda_kernel_direct.py:106-113; 'config' uses
# the benchmark distributions (unit-norm q/k, A_log = log U(1,16), ...).
CASES: Dict[str, dict] = {
    # The reference test's own fixture shape: T=17, cu_seqlens=[0,8,17],
    # Hq=Hk=4, Hv=8 (local_test/test_cuda_kernel_direct.py:91-116).
    "prefill_qk4_v8_t17": dict(kind="prefill", Hq=4, Hv=8, lengths=[8, 9], state=True,
                               dist="reftest", scale=1.0 / np.sqrt(128), seed=17,
                               sample_stride=1),
    # Varlen with an empty and a length-1 sequence, benchmark head counts.
    "prefill_qk16_v32_ragged": dict(kind="prefill", Hq=16, Hv=32, lengths=[5, 0, 23, 1],
                                    state=True, dist="config", scale=0.0, seed=101,
                                    sample_stride=61),
    # Chunk-boundary lengths (64 and 65 tokens) from a zero state.
    "prefill_qk16_v32_chunk_edges": dict(kind="prefill", Hq=16, Hv=32, lengths=[64, 65],
                                         state=False, dist="config", scale=0.0, seed=202,
                                         sample_stride=61),
    # Long-memory decay (alpha in [0.99, 0.9999]) over 200 tokens.
    "prefill_qk4_v8_long_memory": dict(kind="prefill", Hq=4, Hv=8, lengths=[200, 57],
                                       state=True, dist="config", decay=(0.99, 0.9999),
                                       scale=0.0, seed=303, sample_stride=7),
    # The decode benchmark's CPU-runnable case (B=4, Hq=Hk=16, Hv=32).
    "decode_qk16_v32_b4": dict(kind="decode", Hq=16, Hv=32, B=4, state=True, dist="config",
                               scale=1.0 / np.sqrt(128), seed=0, sample_stride=61),
}


def _bf16(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16)


def _unit(x: np.ndarray) -> np.ndarray:
    return x / np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-12)


def make_inputs(name: str) -> dict:
    """Regenerate the CPU inputs of a fixture case (torch tensors)."""
    c = CASES[name]
    rng = np.random.Generator(np.random.PCG64(c["seed"]))
    Hq, Hv = c["Hq"], c["Hv"]
    if c["kind"] == "prefill":
        lengths: List[int] = c["lengths"]
        T, N = int(sum(lengths)), len(lengths)
        lead = (T,)
    else:
        T = N = c["B"]
        lead = (N, 1)
    sn = rng.standard_normal
    if c["dist"] == "reftest":
        q = sn(lead + (Hq, D), dtype=np.float32)
        k = sn(lead + (Hq, D), dtype=np.float32)
        v = sn(lead + (Hv, D), dtype=np.float32)
        state = sn((N, Hv, D, D), dtype=np.float32)
        A_log = sn((Hv,), dtype=np.float32)
        a = sn(lead + (Hv,), dtype=np.float32)
        dt_bias = sn((Hv,), dtype=np.float32)
        b = sn(lead + (Hv,), dtype=np.float32)
    else:
        q = _unit(sn(lead + (Hq, D), dtype=np.float32))
        k = _unit(sn(lead + (Hq, D), dtype=np.float32))
        v = sn(lead + (Hv, D), dtype=np.float32)
        state = (0.02 * sn((N, Hv, D, D), dtype=np.float32)).astype(np.float32)
        A_log = np.log(rng.uniform(1.0, 16.0, (Hv,))).astype(np.float32)
        dt_bias = rng.uniform(-1.0, 1.0, (Hv,)).astype(np.float32)
        if "decay" in c:
            lo, hi = c["decay"]
            alpha = rng.uniform(lo, hi, lead + (Hv,))
            sp = -np.log(alpha) / np.exp(A_log.astype(np.float64))
            a = (sp + np.log(-np.expm1(-sp)) - dt_bias).astype(np.float32)
        else:
            a = sn(lead + (Hv,), dtype=np.float32)
        b = sn(lead + (Hv,), dtype=np.float32)
    inp = {
        "q": _bf16(q), "k": _bf16(k), "v": _bf16(v),
        "state": torch.from_numpy(state) if c["state"] else None,
        "A_log": torch.from_numpy(A_log), "a": _bf16(a), "dt_bias": torch.from_numpy(dt_bias),
        "b": _bf16(b), "scale": float(c["scale"]),
    }
    if c["kind"] == "prefill":
        cu = np.zeros(N + 1, dtype=np.int32)
        cu[1:] = np.cumsum(lengths)
        inp["cu_seqlens"] = torch.from_numpy(cu)
    return inp


def input_sha(inp: dict) -> str:
    h = hashlib.sha256()
    for key in sorted(inp):
        t = inp[key]
        if isinstance(t, torch.Tensor):
            h.update(key.encode())
            h.update(t.contiguous().view(torch.uint8).numpy().tobytes()
                     if t.dtype != torch.bfloat16
                     else t.contiguous().view(torch.int16).numpy().tobytes())
        elif t is not None:
            h.update(f"{key}={t!r}".encode())
    return h.hexdigest()


def sample_indices(numel: int, stride: int) -> np.ndarray:
    return np.arange(0, numel, stride, dtype=np.int64)


def load(name: str) -> dict:
    with np.load(os.path.join(HERE, name + ".npz")) as z:
        return {k: z[k] for k in z.files}
