"""Host-side behaviour of the reference-facing API that needs no GPU."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import api as kmod
from fastaf_kernel_b200 import workloads


def test_no_cpu_path_prefill():
    x = workloads.prefill_inputs([3, 2], seed=0, Hq=4, Hv=8)
    with pytest.raises(ValueError, match="CUDA"):
        fk.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                  x["b"], x["cu_seqlens"], x["scale"])


def test_no_cpu_path_decode():
    x = workloads.decode_inputs(2, seed=0, Hq=4, Hv=8)
    with pytest.raises(ValueError, match="CUDA"):
        fk.kernel_decode(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"],
                         x["dt_bias"], x["b"], x["scale"])


def test_no_cpu_path_decode_step():
    x = workloads.decode_inputs(2, seed=0, Hq=4, Hv=8)
    out = torch.empty((2, 1, 8, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fk.decode_step(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                       x["b"], x["scale"], out, x["state"])


def test_scale_default_matches_reference():
    # solution/triton/kernel.py:438-439
    assert kmod._scale(0.0, 128) == pytest.approx(128 ** -0.5)
    assert kmod._scale(None, 128) == pytest.approx(128 ** -0.5)
    assert kmod._scale(0.5, 128) == 0.5


@pytest.mark.parametrize("cu,T,ok", [
    ([0, 3, 5], 5, True), ([0, 0, 5], 5, True), ([0], 0, True),
    ([1, 5], 5, False), ([0, 4], 5, False), ([0, 4, 3, 5], 5, False),
])
def test_cu_seqlens_validation(cu, T, ok):
    t = torch.tensor(cu, dtype=torch.int64)
    if ok:
        kmod._check_cu_seqlens_host(t, T)
    else:
        with pytest.raises(ValueError):
            kmod._check_cu_seqlens_host(t, T)


def test_workload_constants():
    assert workloads.bytes_per_decode_seq() == 4_219_008
    assert workloads.prefill_flops_per_token() == 5_286_560


def test_long_prefill_decay_range():
    x = workloads.prefill_inputs([300, 200], seed=3, Hq=4, Hv=8, decay_range=(0.5, 0.999))
    g = torch.exp(-torch.exp(x["A_log"]) * torch.nn.functional.softplus(
        x["a"].float() + x["dt_bias"]))
    assert 0.45 < g.min().item() and g.max().item() < 0.9995
