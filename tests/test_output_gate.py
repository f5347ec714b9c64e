"""Gated RMSNorm of the recurrence output (``output_gate=``, ``norm_weight=``):
o <- o / sqrt(mean(o^2) + eps) * w * silu(z) per 128-element head vector.  The
reference returns the ungated o; Gated DeltaNet layers apply this step before the
output projection.  Checked against a plain PyTorch fp32 restatement."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _reference(o, z, w, eps):
    x = o.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float() * torch.nn.functional.silu(z.float())
    return y.to(torch.bfloat16)


def _assert_close(got, ref):
    # bf16 outputs: one bf16 rounding step apart at most
    diff = (got.float() - ref.float()).abs()
    tol = 1e-2 * ref.float().abs() + 1e-3
    assert bool((diff <= tol).all()), f"max excess {(diff - tol).max().item():.3e}"


@pytest.mark.parametrize("shape,wdtype", [((7, 32, 128), torch.float32), ((1000, 8, 128), torch.bfloat16),
                                          ((3, 1, 128), torch.float32)])
def test_output_gate_matches_torch(shape, wdtype):
    g = torch.Generator(device=DEV).manual_seed(5)
    o = (torch.randn(shape, generator=g, device=DEV) * 0.3).to(torch.bfloat16)
    z = torch.randn(shape, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.rand(128, generator=g, device=DEV) + 0.5).to(wdtype)
    ref = _reference(o, z, w, 1e-6)
    got = fk.output_gate(o.clone(), z, w, 1e-6)
    torch.cuda.synchronize()
    _assert_close(got, ref)


@pytest.mark.parametrize("method", ["tcgen05", "chunked", "recurrent"])
def test_prefill_with_output_gate(method):
    x = W.prefill_inputs([300, 77, 64], seed=71, Hq=4, Hv=8, device=DEV)
    T = x["q"].shape[0]
    g = torch.Generator(device=DEV).manual_seed(6)
    z = torch.randn((T, 8, 128), generator=g, device=DEV).to(torch.bfloat16)
    w = torch.rand(128, generator=g, device=DEV) + 0.5
    args = (x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"], x["cu_seqlens"], x["scale"])
    o_plain, s_plain = fk.kernel(*args, method=method)
    o_gated, s_gated = fk.kernel(*args, method=method, output_gate=z, norm_weight=w, norm_eps=1e-5)
    fk.device_status()
    assert torch.equal(s_gated, s_plain)
    _assert_close(o_gated, _reference(o_plain, z, w, 1e-5))


@pytest.mark.parametrize("lengths,Hq,Hv,wdtype", [
    ([700, 129, 64, 1], 4, 8, torch.float32),          # partial chunks, a one-token sequence
    ([300, 128, 257, 64, 200], 16, 32, torch.bfloat16),  # 160 chains: the wave split
    ([256, 0, 191, 64, 300], 16, 32, torch.float32),     # an empty sequence among them
    ([1500, 4096, 999, 2048], 16, 32, torch.bfloat16),   # many chunks per chain through the store warps
])
def test_gated_prefill_is_bit_identical_to_two_calls(lengths, Hq, Hv, wdtype):
    """kernel(..., output_gate=) (gdn_prefill_gated; on tcgen05 the gating is applied in the
    chains' output store) equals prefill, then output_gate, bit for bit; the state too."""
    x = W.prefill_inputs(lengths, seed=73, Hq=Hq, Hv=Hv, device=DEV)
    T = x["q"].shape[0]
    g = torch.Generator(device=DEV).manual_seed(8)
    z = torch.randn((T, Hv, 128), generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.rand(128, generator=g, device=DEV) + 0.5).to(wdtype)
    args = (x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"], x["cu_seqlens"], x["scale"])
    o_fused, s_fused = fk.kernel(*args, method="tcgen05", output_gate=z, norm_weight=w, norm_eps=1e-5)
    o_plain, s_plain = fk.kernel(*args, method="tcgen05")
    fk.output_gate(o_plain, z, w, 1e-5)
    fk.device_status()
    assert torch.equal(o_fused, o_plain)
    assert torch.equal(s_fused, s_plain)


@pytest.mark.parametrize("B,Hq,Hv,l2norm", [(16, 4, 8, False), (3, 16, 32, True), (512, 16, 32, False)])
def test_decode_with_output_gate(B, Hq, Hv, l2norm):
    """kernel_decode(..., output_gate=) (gdn_decode_gated: the gating in the decode kernel's
    store) equals decode, then output_gate, bit for bit; in place, the state too."""
    d = W.decode_inputs(B, seed=72, Hq=Hq, Hv=Hv, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(7)
    z = torch.randn((B, 1, Hv, 128), generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.rand(128, generator=g, device=DEV) + 0.5).to(torch.bfloat16)
    st_plain, st_gated = d["state"].clone(), d["state"].clone()
    args = lambda st: (d["q"], d["k"], d["v"], st, d["A_log"], d["a"], d["dt_bias"], d["b"], d["scale"])
    o_plain, _ = fk.kernel_decode(*args(st_plain), new_state=st_plain, use_qk_l2norm=l2norm)
    o_gated, _ = fk.kernel_decode(*args(st_gated), new_state=st_gated, use_qk_l2norm=l2norm,
                                  output_gate=z, norm_weight=w, norm_eps=1e-5)
    o_two = o_plain.clone()
    fk.output_gate(o_two, z, w, 1e-5)
    fk.device_status()
    assert torch.equal(st_gated, st_plain)
    assert torch.equal(o_gated, o_two)
    _assert_close(o_gated, _reference(o_plain, z, w, 1e-5))


def test_output_gate_rejects_bad_arguments():
    o = torch.zeros((4, 2, 128), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        fk.output_gate(o, torch.zeros((4, 2, 64), dtype=torch.bfloat16, device=DEV), torch.ones(128, device=DEV))
    with pytest.raises(ValueError):
        fk.output_gate(o, torch.zeros_like(o), torch.ones(64, device=DEV))
