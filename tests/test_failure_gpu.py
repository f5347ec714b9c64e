"""Failure detection without a GPU fault: bounded device waits that run out, and a
malformed cu_seqlens that the kernels detect themselves.

Every failure here is made on purpose by the host: a wait limit far below a chunk's
latency (so the tcgen05 chains' waits run out), an mbarrier that nothing arrives on
(in the self-test library), a decreasing cu_seqlens.  None of them faults, traps or
hangs the GPU: each wait gives up after its limit, the CTA waits for its own copies
and MMAs in flight, frees its tensor memory and exits, and the host reads the status
word.  The reference has only a synchronize-and-print check
(local_test/test_cuda_kernel_direct.py:21-27)."""
import ctypes

import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import _lib
from fastaf_kernel_b200 import workloads as W
from fastaf_kernel_b200.build import SELFTEST_LIB_PATH
from oracle import c_oracle
from tolerances import assert_parity

DEV = torch.device("cuda", 0)


def test_wait_limit_setter_returns_previous_setting():
    """Host-only: gdn_set_wait_limit_ns returns the previous limit (0 = the 2 s default)."""
    lib = _lib.load()
    prev = lib.gdn_set_wait_limit_ns(12345)
    try:
        assert lib.gdn_set_wait_limit_ns(777) == 12345
        assert lib.gdn_set_wait_limit_ns(0) == 777
    finally:
        lib.gdn_set_wait_limit_ns(prev)


def test_host_cu_seqlens_is_checked_on_the_host():
    """A CPU cu_seqlens is checked on the host before anything reaches the device."""
    from fastaf_kernel_b200.api import _check_cu_seqlens_host
    with pytest.raises(ValueError, match="non-decreasing"):
        _check_cu_seqlens_host(torch.tensor([0, 5, 3, 8]), 8)
    with pytest.raises(ValueError, match="start at 0"):
        _check_cu_seqlens_host(torch.tensor([1, 5, 8]), 8)
    with pytest.raises(ValueError, match="end at T"):
        _check_cu_seqlens_host(torch.tensor([0, 5, 7]), 8)
    _check_cu_seqlens_host(torch.tensor([0, 5, 5, 8]), 8)


def _gpu(x):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}


def _run(g, method, cu=None):
    return fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                     g["cu_seqlens"] if cu is None else cu, g["scale"], method=method)


def _oracle(x):
    return c_oracle.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                            x["b"], x["cu_seqlens"], x["scale"])


@pytest.mark.gpu
def test_mbarrier_wait_nobody_arrives_gives_up():
    """One warp waits on an mbarrier nothing arrives on, with a 1 ms limit: the wait
    reports failure after about 1 ms and the kernel runs to its end."""
    lib = ctypes.CDLL(SELFTEST_LIB_PATH)
    lib.gdn_selftest_wait_timeout.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    lib.gdn_selftest_wait_timeout.restype = ctypes.c_int
    out = torch.zeros(3, dtype=torch.int64, device=DEV)
    rc = lib.gdn_selftest_wait_timeout(1_000_000, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    completed, elapsed_ns, finished = out.tolist()
    assert completed == 0, "the wait reported a completion nobody signalled"
    assert finished == 1
    assert 1_000_000 <= elapsed_ns < 50_000_000, elapsed_ns


@pytest.mark.gpu
@pytest.mark.parametrize("gated", [False, True])
def test_chain_waits_run_out_then_next_call_is_correct(gated):
    """With a 1 us limit the tcgen05 chains' waits run out: the call returns, the status
    word says GDN_ERR_DEVICE_TIMEOUT (and is cleared by reading it), and the next call
    with the default limit -- which allocates the same tensor memory -- matches the oracle.
    Gated: the output-store warps also have gate-row copies in flight when they give up."""
    lib = _lib.load()
    x = W.prefill_inputs([700, 300, 513], seed=91, Hq=16, Hv=32)
    g = _gpu(x)
    kw = {}
    if gated:
        gen = torch.Generator(device=DEV).manual_seed(92)
        kw = dict(output_gate=torch.randn((g["q"].shape[0], 32, 128), generator=gen, device=DEV).to(torch.bfloat16),
                  norm_weight=torch.rand(128, generator=gen, device=DEV) + 0.5)
    run = lambda: fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                            g["cu_seqlens"], g["scale"], method="tcgen05", **kw)
    prev = lib.gdn_set_wait_limit_ns(1000)
    try:
        run()
        with pytest.raises(_lib.GdnError) as ei:
            fk.device_status()
        assert ei.value.status == _lib.GDN_ERR_DEVICE_TIMEOUT
    finally:
        lib.gdn_set_wait_limit_ns(prev)
    fk.device_status()    # cleared
    o, s = run()
    fk.device_status()
    if gated:
        o_plain, s_plain = _run(g, "tcgen05")
        assert torch.equal(s, s_plain)
        fk.output_gate(o_plain, kw["output_gate"], kw["norm_weight"], 1e-6)
        assert torch.equal(o, o_plain)
    else:
        ro, rs = _oracle(x)
        assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.gpu
@pytest.mark.parametrize("method", ["tcgen05", "chunked", "recurrent"])
@pytest.mark.parametrize("bad", [[0, 300, 200, 600], [0, 250, 700, 600], [5, 300, 450, 600],
                                 [0, -4, 300, 600], [0, 300, 450, 590]])
def test_device_resident_cu_seqlens_is_checked_on_the_device(method, bad):
    """A malformed device-resident cu_seqlens does not make the call synchronize or
    raise; the kernels clamp it (every access stays in bounds) and record it, and
    device_status() raises ValueError once, then the next good call is clean."""
    x = W.prefill_inputs([300, 150, 150], seed=92, Hq=4, Hv=8)
    g = _gpu(x)
    cu_bad = torch.tensor(bad, dtype=torch.int32, device=DEV)
    _run(g, method, cu=cu_bad)
    with pytest.raises(ValueError, match="cu_seqlens"):
        fk.device_status()
    fk.device_status()    # cleared
    o, s = _run(g, method)
    fk.device_status()
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.gpu
@pytest.mark.parametrize("bad_at,value", [(3, 10**6), (5, -7), (7, 100)])
def test_device_cu_seqlens_check_with_the_sequence_ranking(bad_at, value):
    """Enough chains (10 sequences x 32 v-heads = 320 > 148 SMs) that the pooled tcgen05
    call ranks its sequences on the device before the chains: with one malformed entry
    (past T, negative, or below its predecessor) the ranking still gives a permutation of
    the clamped lengths, every access stays in bounds, the error is recorded, and the next
    good call matches the oracle."""
    lengths = [300, 64, 1, 257, 128, 65, 500, 0, 192, 129]
    x = W.prefill_inputs(lengths, seed=93, Hq=16, Hv=32)
    g = _gpu(x)
    cu = [0]
    for L in lengths:
        cu.append(cu[-1] + L)
    cu[bad_at] = value
    _run(g, "tcgen05", cu=torch.tensor(cu, dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError, match="cu_seqlens"):
        fk.device_status()
    fk.device_status()    # cleared
    o, s = _run(g, "tcgen05")
    fk.device_status()
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)
