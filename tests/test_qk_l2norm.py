"""Optional q/k L2 normalisation (``use_qk_l2norm``): every 128-element q and k head
vector becomes bf16(x / sqrt(sum x^2 + 1e-6)) before the recurrence.  The reference
has no such step (its inputs arrive normalised), so the oracle carries it as an
option; these tests check the oracle's option on the CPU and the kernels' against it
on the GPU."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import workloads as W
from oracle import c_oracle
from tolerances import assert_parity

DEV = torch.device("cuda", 0)


def _raw(x, scale_q=3.0, scale_k=0.25):
    """The same inputs with q and k no longer unit-norm."""
    y = dict(x)
    y["q"] = (x["q"].float() * scale_q).to(torch.bfloat16)
    y["k"] = (x["k"].float() * scale_k).to(torch.bfloat16)
    return y


def _oracle_prefill(x, l2):
    return c_oracle.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                            x["cu_seqlens"], x["scale"], qk_l2norm=l2)


def _oracle_decode(d, l2):
    return c_oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                           d["scale"], qk_l2norm=l2)


# ---------------------------------------------------------------- oracle (CPU)

def test_oracle_l2norm_undoes_input_scaling():
    """Normalising makes the result independent of the q/k magnitudes."""
    x = W.prefill_inputs([40, 25], seed=31, Hq=2, Hv=4)
    o1, s1 = _oracle_prefill(x, True)
    o2, s2 = _oracle_prefill(_raw(x), True)
    assert_parity(o2, o1, s2, s1)


def test_oracle_l2norm_is_near_identity_on_unit_inputs():
    """The workload's q and k are already unit-norm (then bf16), so normalising them
    again changes the result only at bf16 rounding level."""
    x = W.prefill_inputs([50, 31], seed=32, Hq=2, Hv=4)
    o1, s1 = _oracle_prefill(x, False)
    o2, s2 = _oracle_prefill(x, True)
    assert_parity(o2, o1, s2, s1)


def test_oracle_l2norm_changes_unnormalised_inputs():
    """Sanity: on inputs that are not unit-norm the option is not a no-op."""
    x = _raw(W.prefill_inputs([40], seed=33, Hq=1, Hv=2))
    o1, s1 = _oracle_prefill(x, False)
    o2, s2 = _oracle_prefill(x, True)
    assert (o1.float() - o2.float()).abs().max() > 1e-2


# ---------------------------------------------------------------- kernels (GPU)

def _gpu(d):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hv", [(4, 16, 32), (64, 4, 8), (3, 1, 2)])
def test_decode_l2norm_matches_oracle(B, Hq, Hv):
    d = _raw(W.decode_inputs(B, seed=40 + B, Hq=Hq, Hv=Hv))
    g = _gpu(d)
    o, s = fk.kernel_decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                            g["scale"], use_qk_l2norm=True)
    fk.device_status()
    ro, rs = _oracle_decode(d, True)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.gpu
@pytest.mark.parametrize("method", ["tcgen05", "chunked", "recurrent"])
def test_prefill_l2norm_matches_oracle(method):
    x = _raw(W.prefill_inputs([300, 7, 129, 64], seed=44, Hq=4, Hv=8))
    g = _gpu(x)
    o, s = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                     g["cu_seqlens"], g["scale"], method=method, use_qk_l2norm=True)
    fk.device_status()
    ro, rs = _oracle_prefill(x, True)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.gpu
def test_l2norm_prefill_then_decode_continues():
    """Normalised prefill of T tokens + one normalised decode step = normalised prefill
    of T + 1 tokens (the two kernels normalise with the same arithmetic)."""
    T = 200
    x = _raw(W.prefill_inputs([T + 1], seed=45, Hq=4, Hv=8))
    g = _gpu(x)
    o_full, s_full = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                               g["cu_seqlens"], g["scale"], method="tcgen05", use_qk_l2norm=True)
    cu = torch.tensor([0, T], dtype=torch.int32, device=DEV)
    sl = lambda t: t[:T]
    o_p, s_p = fk.kernel(sl(g["q"]), sl(g["k"]), sl(g["v"]), g["state"], g["A_log"], sl(g["a"]), g["dt_bias"],
                         sl(g["b"]), cu, g["scale"], method="tcgen05", use_qk_l2norm=True)
    tail = lambda t: t[T:].unsqueeze(0)
    o_d, s_d = fk.kernel_decode(tail(g["q"]), tail(g["k"]), tail(g["v"]), s_p, g["A_log"], tail(g["a"]),
                                g["dt_bias"], tail(g["b"]), g["scale"], use_qk_l2norm=True)
    fk.device_status()
    assert_parity(o_d.view(1, 8, 128).cpu(), o_full[T:].cpu(), s_d.cpu(), s_full.cpu())
