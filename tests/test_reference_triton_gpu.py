"""The reference's own Triton GPU kernels (solution/triton/kernel.py:138-409), compiled for
sm_100 into oracle/_ref/ by oracle/ref_triton.py, on the GPU: they agree with the oracle
and with this library's kernels on the same inputs.  This pins the baseline bench.py's
`reference_gpu` leg times (the compiled launch path and its argument conventions), not the
product.  Skipped when the compiled kernels are absent (they are built where the reference
checkout is present)."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import workloads as W
from oracle import c_oracle, ref_triton
from tolerances import assert_parity

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_triton.available(), reason="oracle/_ref holds no compiled reference kernels")]
DEV = torch.device("cuda", 0)


def _gpu(x):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


def test_reference_triton_prefill_matches_oracle_and_ours():
    x = W.prefill_inputs([300, 129, 64], seed=71, decay_range=(0.5, 0.999))   # Hq 16, Hv 32, with state
    g = _gpu(x)
    T, N = g["q"].shape[0], 3
    out = torch.empty((T, 32, 128), dtype=torch.bfloat16, device=DEV)
    ns = torch.empty((N, 32, 128, 128), device=DEV)
    ref = ref_triton.RefTriton()
    ref.prefill(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"], g["cu_seqlens"],
                g["scale"], out, ns)
    torch.cuda.synchronize()
    assert ref.config("prefill") is not None
    ro, rs = c_oracle.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                              x["cu_seqlens"], x["scale"])
    assert_parity(out.cpu(), ro, ns.cpu(), rs)
    o2, s2 = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                       g["cu_seqlens"], g["scale"])
    fk.device_status()
    assert_parity(o2.cpu(), out.cpu(), s2.cpu(), ns.cpu())


def test_reference_triton_decode_matches_oracle_and_ours():
    d = W.decode_inputs(8, seed=72)
    g = _gpu(d)
    out = torch.empty((8, 32, 128), dtype=torch.bfloat16, device=DEV)
    ns = torch.empty_like(g["state"])
    ref = ref_triton.RefTriton()
    ref.decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"], g["scale"], out, ns)
    torch.cuda.synchronize()
    ro, rs = c_oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                             d["scale"])
    assert_parity(out.view(8, 1, 32, 128).cpu(), ro, ns.cpu(), rs)
    o2, s2 = fk.kernel_decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                              g["scale"])
    torch.cuda.synchronize()
    assert_parity(o2.cpu(), out.view(8, 1, 32, 128).cpu(), s2.cpu(), ns.cpu())
