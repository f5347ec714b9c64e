"""gdn_prefill_noalloc: the tcgen05 prefill with its workspace in the library's fixed
64 MiB device array (no allocation in the call).  Collected last on purpose, so it also
runs after every other test has used the library in the same process."""
import pytest
import torch

import fastaf_kernel_b200 as fk
from fastaf_kernel_b200 import _lib
from fastaf_kernel_b200 import workloads as W

DEV = torch.device("cuda", 0)
CAPACITY = 64 << 20          # bytes of the fixed workspace
SLOT_BYTES = 41984           # one (chunk, v-head) slot: 4 bf16 T tiles, bf16 P [64][64], 4 gate vectors


def _noalloc(g, out, ns):
    lib = _lib.load()
    T, Hq = g["q"].shape[0], g["q"].shape[1]
    Hv = g["v"].shape[1]
    N = g["cu_seqlens"].numel() - 1
    ptr = lambda t: None if t is None else t.data_ptr()
    return lib.gdn_prefill_noalloc(
        ptr(g["q"]), ptr(g["k"]), ptr(g["v"]), ptr(g["state"]), ptr(g["A_log"]), ptr(g["a"]),
        ptr(g["dt_bias"]), ptr(g["b"]), ptr(g["cu_seqlens"]), N, T, Hq, Hv, 128, float(g["scale"]),
        _lib.GDN_DTYPE_BF16 if g["a"].dtype == torch.bfloat16 else _lib.GDN_DTYPE_F32,
        _lib.GDN_DTYPE_BF16 if g["A_log"].dtype == torch.bfloat16 else _lib.GDN_DTYPE_F32,
        out.data_ptr(), ns.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_beyond_capacity():
    """Too large for the fixed workspace: refused with a clear message before any launch."""
    lib = _lib.load()
    N, T, Hv = 16, 16 * 8192, 32
    assert ((T + 63) // 64 + N) * Hv * SLOT_BYTES > CAPACITY
    rc = lib.gdn_prefill_noalloc(None, None, None, None, None, None, None, None, None, N, T, 16, Hv,
                                 128, 0.0, 1, 0, None, None, None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT
    msg = lib.gdn_last_error().decode()
    assert "fixed workspace holds" in msg and str(CAPACITY) in msg


@pytest.mark.gpu
def test_noalloc_matches_pooled_entry_point_twice():
    """Two calls in a row (different batches, the second reusing the array the first
    filled) each equal the pooled-workspace entry point bit for bit; the second call
    takes no device memory (free memory does not drop across it)."""
    cases = [([1000, 37, 700, 64], 7), ([2048, 129, 1], 8)]
    for i, (lengths, seed) in enumerate(cases):
        x = W.prefill_inputs(lengths, seed=seed, Hq=16, Hv=32)
        T, N = sum(lengths), len(lengths)
        assert ((T + 63) // 64 + N) * 32 * SLOT_BYTES <= CAPACITY
        g = {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in x.items()}
        o_ref, s_ref = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"],
                                 g["dt_bias"], g["b"], g["cu_seqlens"], g["scale"], method="tcgen05")
        out = torch.full_like(o_ref, 3.0)
        ns = torch.full_like(s_ref, 3.0)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(DEV)[0]
        rc = _noalloc(g, out, ns)
        assert rc == 0, _lib.load().gdn_last_error()
        fk.device_status()
        if i > 0:
            assert torch.cuda.mem_get_info(DEV)[0] >= free_before, "the call took device memory"
        assert torch.equal(out, o_ref)
        assert torch.equal(ns, s_ref)
