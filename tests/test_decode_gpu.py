"""Decode kernel parity on the GPU against the CPU oracle (through the C ABI)."""
import numpy as np
import pytest
import torch

import fastaf_kernel_b200 as fk
import fixtures
from fastaf_kernel_b200 import workloads as W
from oracle import c_oracle
from tolerances import assert_parity

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _gpu(d):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def _decode(d, **kw):
    g = _gpu(d)
    o, s = fk.kernel_decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                            g["dt_bias"], g["b"], g["scale"], **kw)
    torch.cuda.synchronize()
    return o, s


def _oracle(d):
    return c_oracle.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"],
                           d["dt_bias"], d["b"], d["scale"])


@pytest.mark.parametrize("B,Hq,Hv", [(4, 16, 32), (1, 4, 8), (3, 4, 8), (7, 16, 32),
                                      (2, 8, 32), (64, 16, 32)])
def test_decode_matches_oracle(B, Hq, Hv):
    d = W.decode_inputs(B, seed=B * 31 + Hv, Hq=Hq, Hv=Hv)
    o, s = _decode(d)
    ro, rs = _oracle(d)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_decode_golden_fixture():
    name = "decode_qk16_v32_b4"
    g = fixtures.load(name)
    o, s = _decode(fixtures.make_inputs(name))
    ref_o = torch.from_numpy(g["out"].view(np.int16).copy()).view(torch.bfloat16).reshape(
        tuple(g["out_shape"]))
    got = s.cpu().reshape(-1).numpy()[g["state_idx"]].astype(np.float64)
    ref = g["state_val"].astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()
    assert ((o.cpu().float() - ref_o.float()).abs() <= 2e-2 + 2e-2 * ref_o.float().abs()).all()


def test_decode_zero_state():
    d = W.decode_inputs(5, seed=9, with_state=False)
    o, s = _decode(d)
    ro, rs = _oracle(d)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_decode_inplace_equals_out_of_place():
    d = W.decode_inputs(16, seed=4)
    o1, s1 = _decode(d)
    g = _gpu(d)
    st = g["state"].clone()
    o2, s2 = fk.kernel_decode(g["q"], g["k"], g["v"], st, g["A_log"], g["a"], g["dt_bias"],
                              g["b"], g["scale"], new_state=st)
    torch.cuda.synchronize()
    assert s2.data_ptr() == st.data_ptr()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_decode_f32_gates_and_bf16_params():
    d = W.decode_inputs(6, seed=5, Hq=4, Hv=8)
    d["a"] = d["a"].float() + 0.25
    d["b"] = d["b"].float() - 0.5
    d["A_log"] = d["A_log"].to(torch.bfloat16)
    d["dt_bias"] = d["dt_bias"].to(torch.bfloat16)
    o, s = _decode(d)
    ro, rs = _oracle(d)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_decode_extreme_gates():
    # softplus threshold (x > 20), saturated sigmoid, alpha -> 0 and alpha -> 1.
    d = W.decode_inputs(4, seed=6, Hq=4, Hv=8)
    d["a"] = torch.tensor([30.0, -30.0, 0.0, 19.9, -19.9, 5.0, -5.0, 25.0]).repeat(4).view(4, 1, 8)
    d["b"] = torch.tensor([40.0, -40.0, 0.0, 3.0, -3.0, 10.0, -10.0, 1.0]).repeat(4).view(4, 1, 8)
    d["A_log"] = torch.tensor([-8.0, 3.0, 0.0, 1.0, -2.0, 2.7, 0.5, -5.0])
    o, s = _decode(d)
    ro, rs = _oracle(d)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_decode_batched_full_size_sample():
    """The B=512 in-place step: checks 8 sampled sequences against the oracle and
    that the untouched-by-sampling rest equals an out-of-place run bit for bit."""
    d = W.decode_inputs(512, seed=2)
    g = _gpu(d)
    o1, s1 = fk.kernel_decode(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                              g["dt_bias"], g["b"], g["scale"])
    st = g["state"].clone()
    o2, s2 = fk.kernel_decode(g["q"], g["k"], g["v"], st, g["A_log"], g["a"], g["dt_bias"],
                              g["b"], g["scale"], new_state=st)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, st)
    idx = torch.tensor([0, 1, 77, 128, 255, 300, 411, 511])
    sub = {k: (v[idx] if isinstance(v, torch.Tensor) and v.shape[0] == 512 else v)
           for k, v in d.items()}
    ro, rs = _oracle(sub)
    assert_parity(o1.cpu()[idx], ro, s1.cpu()[idx], rs)


def test_decode_steps_equal_prefill():
    """T decode steps from a state equal one T-token prefill (size-independent)."""
    T, Hq, Hv = 12, 4, 8
    x = W.prefill_inputs([T], seed=21, Hq=Hq, Hv=Hv)
    g = _gpu(x)
    po, ps = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"],
                       g["b"], g["cu_seqlens"], g["scale"], method="recurrent")
    st = g["state"].clone()
    outs = []
    for t in range(T):
        o, st = fk.kernel_decode(g["q"][t:t + 1].unsqueeze(0), g["k"][t:t + 1].unsqueeze(0),
                                 g["v"][t:t + 1].unsqueeze(0), st, g["A_log"],
                                 g["a"][t:t + 1].unsqueeze(0), g["dt_bias"],
                                 g["b"][t:t + 1].unsqueeze(0), g["scale"], new_state=st)
        outs.append(o.view(1, Hv, 128))
    torch.cuda.synchronize()
    assert_parity(torch.cat(outs).cpu(), po.cpu(), st.cpu(), ps.cpu(), state_tol=1e-5,
                  atol=1e-2, rtol=1e-2)


def test_decode_step_matches_kernel_decode():
    """A prepared decode step over fixed buffers (refilled in place every token, state
    updated in place) gives bit for bit what kernel_decode gives, and creating it launches
    nothing."""
    B, Hq, Hv = 8, 16, 32
    x = W.decode_inputs(B, seed=71, Hq=Hq, Hv=Hv, device=DEV)
    bufs = {k2: x[k2].clone() for k2 in ("q", "k", "v", "a", "b")}
    state = x["state"].clone()
    ref_state = x["state"].clone()
    out = torch.empty((B, 1, Hv, 128), dtype=torch.bfloat16, device=DEV)
    step = fk.decode_step(bufs["q"], bufs["k"], bufs["v"], state, x["A_log"], bufs["a"], x["dt_bias"],
                          bufs["b"], x["scale"], out, state)
    torch.cuda.synchronize()
    assert torch.equal(state, x["state"]), "creating the step must not run it"
    for s in range(3):
        d = W.decode_step_inputs(B, seed=100 + s, Hq=Hq, Hv=Hv, device=DEV)
        for k2 in bufs:
            bufs[k2].copy_(d[k2])
        step()
        ro, _ = fk.kernel_decode(d["q"], d["k"], d["v"], ref_state, x["A_log"], d["a"], x["dt_bias"], d["b"],
                                 x["scale"], new_state=ref_state)
        fk.device_status()
        assert torch.equal(out, ro) and torch.equal(state, ref_state)


def test_decode_step_needs_direct_buffers():
    """Buffers that kernel_decode would copy (a strided q, a and b of different dtypes)
    cannot back a prepared step."""
    x = W.decode_inputs(2, seed=72, device=DEV)
    out = torch.empty((2, 1, 32, 128), dtype=torch.bfloat16, device=DEV)
    q_strided = torch.empty((2, 1, 16, 256), dtype=torch.bfloat16, device=DEV)[..., :128]
    q_strided.copy_(x["q"])
    with pytest.raises(ValueError, match="decode_step"):
        fk.decode_step(q_strided, x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"],
                       x["scale"], out, x["state"])
    with pytest.raises(ValueError, match="decode_step"):
        fk.decode_step(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"].float(), x["dt_bias"], x["b"],
                       x["scale"], out, x["state"])
