"""Gate inputs a and b taken straight from a wider projection output (the step before the
path: a Gated DeltaNet layer's projection GEMM emits a and b side by side in one [T, ...]
tensor).  The kernels read them through their row stride -- no copy -- and the results
equal those of packed a and b bit for bit."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import _lib
from fastaf_kernel_b200 import workloads as W

DEV = torch.device("cuda", 0)


def test_strided_entry_points_reject_short_strides():
    """Host-only: a row stride below num_v_heads is refused before any launch."""
    lib = _lib.load()
    rc = lib.gdn_prefill_strided(16, 16, 16, None, 16, 16, 16, 16, 16, 1, 4, 16, 32, 128, 0.0, 1, 0, 16, 4096,
                                 31, 0, 0, 0, None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT and "row strides" in lib.gdn_last_error().decode()
    rc = lib.gdn_decode_strided(16, 16, 16, 16, 16, 16, 16, 16, 1, 16, 32, 128, 0.0, 1, 0, 16, 16, 0, 20, 0, None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT


def _projection(T, Hv, extra, dtype, seed):
    """[T, Hv + Hv + extra] rows: b, a, then other projection columns; a and b are views."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    proj = torch.randn((T, 2 * Hv + extra), generator=g, device=DEV).to(dtype)
    return proj[:, Hv:2 * Hv], proj[:, :Hv]


def _allocations(fn):
    """Tensors torch allocated while fn ran (a copy of a or b would be one)."""
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats(DEV)["allocation.all.allocated"]
    fn()
    torch.cuda.synchronize()
    return torch.cuda.memory_stats(DEV)["allocation.all.allocated"] - before


@pytest.mark.gpu
@pytest.mark.parametrize("method", ["tcgen05", "chunked", "recurrent"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_prefill_gates_from_projection_view(method, dtype):
    x = W.prefill_inputs([300, 129, 64], seed=81, Hq=4, Hv=8, device=DEV)
    T, Hv = x["q"].shape[0], 8
    a, b = _projection(T, Hv, 40, dtype, 82)
    assert not a.is_contiguous() and a.stride(0) == 2 * Hv + 40
    out = torch.empty((T, Hv, 128), dtype=torch.bfloat16, device=DEV)
    ns = torch.empty((3, Hv, 128, 128), device=DEV)
    run = lambda: fk.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], a, x["dt_bias"], b, x["cu_seqlens"],
                            x["scale"], method=method, output=out, new_state=ns)
    run()
    o_ref, s_ref = fk.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], a.contiguous(), x["dt_bias"],
                             b.contiguous(), x["cu_seqlens"], x["scale"], method=method)
    fk.device_status()
    assert torch.equal(out, o_ref) and torch.equal(ns, s_ref)
    assert _allocations(run) == 0, "a or b was copied"


@pytest.mark.gpu
def test_decode_gates_from_projection_view_and_decode_step():
    B, Hq, Hv = 6, 16, 32
    d = W.decode_inputs(B, seed=83, Hq=Hq, Hv=Hv, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(84)
    proj = torch.randn((B, 1, 2 * Hv + 8), generator=g, device=DEV).to(torch.bfloat16)
    a, b = proj[:, :, Hv:2 * Hv], proj[:, :, :Hv]
    st1, st2, st3 = d["state"].clone(), d["state"].clone(), d["state"].clone()
    o1, _ = fk.kernel_decode(d["q"], d["k"], d["v"], st1, d["A_log"], a, d["dt_bias"], b, d["scale"], new_state=st1)
    o2, _ = fk.kernel_decode(d["q"], d["k"], d["v"], st2, d["A_log"], a.contiguous(), d["dt_bias"], b.contiguous(),
                             d["scale"], new_state=st2)
    out = torch.empty_like(o1)
    step = fk.decode_step(d["q"], d["k"], d["v"], st3, d["A_log"], a, d["dt_bias"], b, d["scale"], out, st3)
    step()
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(st1, st2)
    assert torch.equal(out, o1) and torch.equal(st3, st1)
