"""Context-parallel prefill of one long sequence (segments joined by a scan of their
affine state maps).

CPU: the cutting and the scan with the CPU oracle as the per-segment prefill -- one
process, and a world_size-2 gloo run where each rank holds half of the sequence.
GPU: the same with this library's CUDA prefill, against one prefill call over the
whole sequence."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fastaf_kernel_b200 import context_parallel as cp
from fastaf_kernel_b200 import workloads as W
from tolerances import STATE_MAX_REL, assert_parity

# Slow decay, so the state carried across segment boundaries matters (with the
# default gates it is forgotten within a few tokens).
SLOW = (0.95, 0.9999)


def _oracle_fn(q, k, v, state, A_log, a, dt_bias, b, cu, scale):
    from oracle import c_oracle
    return c_oracle.prefill(q, k, v, state, A_log, a, dt_bias, b, cu, scale, num_threads=2)


def _whole(x, fn):
    T = x["q"].shape[0]
    cu = torch.tensor([0, T], dtype=torch.int32, device=x["q"].device)
    return fn(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"], x["b"], cu, x["scale"])


@pytest.mark.parametrize("T,P", [(1000, 4), (700, 3), (64, 4), (130, 2), (5000, 1)])
def test_segment_bounds(T, P):
    b = cp.segment_bounds(T, P)
    assert b[0] == 0 and b[-1] == T
    assert all(x < y for x, y in zip(b, b[1:])) or T == 0
    assert all(c % 64 == 0 for c in b[1:-1])
    assert len(b) - 1 <= P


@pytest.mark.parametrize("T,P,with_state", [(700, 4, True), (450, 3, False)])
def test_segmented_prefill_equals_one_pass_oracle(T, P, with_state):
    """(Also checks the carried state matters: dropping it changes the result.)"""
    x = W.prefill_inputs([T], seed=61, Hq=2, Hv=4, state_mask=[with_state], decay_range=SLOW)
    ro, rs = _whole(x, _oracle_fn)
    o, s = cp.prefill_segmented(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                                x["b"], x["scale"], segments=P, prefill_fn=_oracle_fn)
    assert_parity(o, ro, s, rs)
    bounds = cp.segment_bounds(T, P)
    cu = torch.tensor(bounds, dtype=torch.int32)
    lo, ls = _oracle_fn(x["q"], x["k"], x["v"], None, x["A_log"], x["a"], x["dt_bias"], x["b"], cu, x["scale"])
    # the last segment alone (no carried state) is off by more than the state tolerance
    assert (ls[-1] - rs[0]).abs().max() > 2 * STATE_MAX_REL * rs.abs().max()


def test_scan_maps_compose():
    """compose_maps of consecutive maps equals applying them one by one."""
    g = torch.Generator().manual_seed(3)
    M = torch.randn((3, 2, 8, 8), generator=g) * 0.3
    C = torch.randn((3, 2, 8, 8), generator=g)
    S0 = torch.randn((2, 8, 8), generator=g, dtype=torch.float64)
    _, end = cp.compose(M, C, S0)
    Mt, Ct = cp.compose_maps(M, C)
    assert torch.allclose(torch.matmul(S0, Mt) + Ct, end, rtol=1e-12, atol=1e-12)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, cuts, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = W.prefill_inputs([T], seed=62, Hq=2, Hv=4, decay_range=SLOW)
        a0, a1 = cuts[rank], cuts[rank + 1]
        sl = lambda t: t[a0:a1]
        o, s = cp.prefill_context_parallel(sl(x["q"]), sl(x["k"]), sl(x["v"]), x["state"], x["A_log"],
                                           sl(x["a"]), x["dt_bias"], sl(x["b"]), x["scale"],
                                           segments_per_rank=2, prefill_fn=_oracle_fn)
        parts = [torch.empty(0)] * world
        dist.all_gather_object(parts, o)
        if rank == 0:
            ro, rs = _whole(x, _oracle_fn)
            out = torch.cat(parts)
            try:
                assert_parity(out, ro, s, rs)
                q.put("ok")
            except AssertionError as e:
                q.put(str(e))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cuts", [[0, 300, 640], [0, 0, 256]])
def test_gloo_world2_context_parallel_equals_one_pass(cuts):
    T = cuts[-1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, T, cuts, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == "ok"


@pytest.mark.gpu
@pytest.mark.parametrize("method,P", [("tcgen05", 8), ("chunked", 4)])
def test_segmented_prefill_gpu_equals_one_pass(method, P):
    import fastaf_kernel_b200 as fk
    dev = torch.device("cuda", 0)
    x = W.prefill_inputs([20000], seed=63, device=dev, decay_range=(0.99, 0.9999))
    fn = lambda *args: fk.kernel(*args, method=method)
    ro, rs = _whole(x, fn)
    o, s = cp.prefill_segmented(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                                x["b"], x["scale"], segments=P, method=method)
    fk.device_status()
    assert_parity(o.cpu(), ro.cpu(), s.cpu(), rs.cpu())


@pytest.mark.gpu
def test_segmented_prefill_gpu_against_oracle():
    """8 segments of 4096 tokens of one sequence (Hq 16, Hv 32, nonzero initial state,
    slow decay so the carried state matters) through the tcgen05 kernel, against the C
    oracle over the whole 32768-token sequence, at the same tolerances as every prefill."""
    import fastaf_kernel_b200 as fk
    from oracle import c_oracle
    dev = torch.device("cuda", 0)
    x = W.prefill_inputs([8 * 4096], seed=64, decay_range=(0.99, 0.9999))
    assert x["state"] is not None and float(x["state"].abs().max()) > 0
    ro, rs = _whole(x, c_oracle.prefill)
    g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}
    o, s = cp.prefill_segmented(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"],
                                g["b"], g["scale"], segments=8, method="tcgen05")
    fk.device_status()
    assert_parity(o.cpu(), ro, s.cpu(), rs)
