"""The mixed prefill + decode workload at full size: 256 sequences with log-uniform
lengths in [128, 32768] (1.55 M packed tokens, nonzero initial state), prefilled,
then 1024 decode steps on all 256 states (Hq=16, Hv=32, D=128).

Size-independent checks on the GPU:
  * decode continues prefill: prefill of each sequence's first L_i tokens followed by
    1024 single-token decode steps gives the outputs and the final state of one prefill
    over all L_i + 1024 tokens;
  * the tcgen05 prefill equals the token-serial CUDA-core prefill over every token;
and, pinned to the oracle, four whole sequences (the shortest, the longest and two
others) against the CPU oracle.

Peak device memory is about 95 GB (inputs 28 GB, the tcgen05 workspace 37 GB, two
output buffers); comparisons run on the device in slices, so host memory stays small."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import workloads as W
from oracle import c_oracle
from tolerances import ATOL, RTOL, STATE_MAX_REL, assert_parity

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
N_SEQS, STEPS = 256, 1024


def _out_excess(got, ref, rows=1 << 16):
    """max(|got - ref| - (ATOL + RTOL |ref|)) over all elements, in row slices."""
    worst = -1.0
    for i in range(0, got.shape[0], rows):
        g, r = got[i:i + rows].float(), ref[i:i + rows].float()
        assert torch.isfinite(g).all(), "non-finite output"
        worst = max(worst, ((g - r).abs() - (ATOL + RTOL * r.abs())).max().item())
    return worst


def _state_rel(got, ref):
    assert torch.isfinite(got).all(), "non-finite state"
    return ((got - ref).abs().max() / ref.abs().max()).item()


def _prefill(x, cu, state, method):
    o, s = fk.kernel(x["q"], x["k"], x["v"], state, x["A_log"], x["a"], x["dt_bias"], x["b"], cu,
                     x["scale"], method=method)
    fk.device_status()
    return o, s


@pytest.fixture
def release_memory():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_prefill_then_1024_decode_steps_256_loguniform_sequences(release_memory):
    lengths = W.loguniform_lengths(4, n=N_SEQS)
    ext = [n + STEPS for n in lengths]
    x = W.prefill_inputs(ext, seed=4, device=DEV)
    Hv = x["v"].shape[1]
    cu = x["cu_seqlens"].long()
    starts = cu[:-1]
    L = torch.tensor(lengths, dtype=torch.int64, device=DEV)

    # Split every sequence into its first L_i tokens and its 1024 continuation tokens
    # (2N packed sequences over the same token buffers; the continuations start from
    # zero state and are not used).
    cu2 = torch.stack([starts, starts + L], 1).reshape(-1)
    cu2 = torch.cat([cu2, cu[-1:]]).to(torch.int32)
    state2 = torch.zeros((2 * N_SEQS,) + tuple(x["state"].shape[1:]), device=DEV)
    state2[0::2] = x["state"]
    o2, s2 = _prefill(x, cu2, state2, "tcgen05")
    o_r, s_r = _prefill(x, cu2, state2, "recurrent")
    ex = _out_excess(o2, o_r)
    assert ex <= 0, f"tcgen05 vs recurrent prefill output exceeds tolerance by {ex:.3e}"
    rel = _state_rel(s2, s_r)
    assert rel <= STATE_MAX_REL, f"tcgen05 vs recurrent prefill state max rel {rel:.3e}"
    state = s2[0::2].contiguous()
    del o2, o_r, s_r, state2

    # One prefill over all L_i + 1024 tokens.
    o_ext, s_ext = _prefill(x, x["cu_seqlens"], x["state"], "tcgen05")

    # 1024 decode steps on all 256 states, in place.
    dout = torch.empty((N_SEQS, 1, Hv, 128), dtype=torch.bfloat16, device=DEV)
    worst = -1.0
    for s in range(STEPS):
        tok = starts + L + s
        fk.kernel_decode(x["q"][tok].unsqueeze(1), x["k"][tok].unsqueeze(1), x["v"][tok].unsqueeze(1),
                         state, x["A_log"], x["a"][tok].unsqueeze(1), x["dt_bias"],
                         x["b"][tok].unsqueeze(1), x["scale"], output=dout, new_state=state)
        if s % 64 == 63 or s == STEPS - 1:
            fk.device_status()
        worst = max(worst, _out_excess(dout.view(N_SEQS, Hv, 128), o_ext[tok]))
    assert worst <= 0, f"decode outputs exceed the prefill's by {worst:.3e}"
    rel = _state_rel(state, s_ext)
    assert rel <= STATE_MAX_REL, f"decoded state vs prefilled state max rel {rel:.3e}"

    # Four whole sequences against the oracle.
    pick = sorted({min(range(N_SEQS), key=lambda i: lengths[i]),
                   max(range(N_SEQS), key=lambda i: lengths[i]), 0, N_SEQS // 2})
    for i in pick:
        a, b = int(cu[i]), int(cu[i + 1])
        sub = {k: (x[k][a:b].cpu() if k in ("q", "k", "v", "a", "b") else x[k]) for k in x}
        sub["A_log"], sub["dt_bias"] = x["A_log"].cpu(), x["dt_bias"].cpu()
        ro, rs = c_oracle.prefill(sub["q"], sub["k"], sub["v"], x["state"][i:i + 1].cpu(), sub["A_log"],
                                  sub["a"], sub["dt_bias"], sub["b"],
                                  torch.tensor([0, b - a], dtype=torch.int32), x["scale"])
        assert_parity(o_ext[a:b].cpu(), ro, s_ext[i:i + 1].cpu(), rs)
