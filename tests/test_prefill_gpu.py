"""Prefill kernels on the GPU against the CPU oracle (through the C ABI).

All three prefill kernels are covered: the chunked (C=64) kernel on tcgen05 +
TMEM + TMA, the chunked kernel on mma.sync, and the token-serial CUDA-core kernel."""
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
METHODS = ["tcgen05", "chunked", "recurrent"]
TC_MIN_TOKENS = 64   # the tcgen05 kernel's TMA box is 64 tokens deep


def _gpu(d):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def _prefill(x, method, **kw):
    g = _gpu(x)
    if method == "tcgen05" and g["q"].shape[0] < TC_MIN_TOKENS:
        # Refused before any launch, with the library's "unsupported" status.
        with pytest.raises(NotImplementedError):
            fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"],
                      g["b"], g["cu_seqlens"], g["scale"], method=method, **kw)
        pytest.skip("the tcgen05 kernel needs at least 64 packed tokens")
    o, s = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"],
                     g["b"], g["cu_seqlens"], g["scale"], method=method, **kw)
    fk.device_status()   # synchronizes; raises if a bounded device wait timed out
    return o, s


def _oracle(x):
    return c_oracle.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"],
                            x["dt_bias"], x["b"], x["cu_seqlens"], x["scale"])


def _golden_state(g, s):
    got = s.cpu().reshape(-1).numpy()[g["state_idx"]].astype(np.float64)
    ref = g["state_val"].astype(np.float64)
    return np.abs(got - ref).max() / np.abs(ref).max()


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("name", ["prefill_qk16_v32_ragged", "prefill_qk16_v32_chunk_edges",
                                  "prefill_qk4_v8_long_memory"])
def test_prefill_golden_fixtures(method, name):
    g = fixtures.load(name)
    o, s = _prefill(fixtures.make_inputs(name), method)
    ref_o = torch.from_numpy(g["out"].view(np.int16).copy()).view(torch.bfloat16).reshape(
        tuple(g["out_shape"]))
    assert _golden_state(g, s) <= 1e-3
    assert ((o.cpu().float() - ref_o.float()).abs() <= 2e-2 + 2e-2 * ref_o.float().abs()).all()


def test_prefill_reference_test_fixture_recurrent():
    """The reference test's own fixture (local_test/test_cuda_kernel_direct.py:91-116):
    unnormalised randn keys amplify the state ~1e6-fold in 9 tokens, so only the
    fp32 token-serial kernel is held to it, at the fp32-reordering level."""
    name = "prefill_qk4_v8_t17"
    g = fixtures.load(name)
    o, s = _prefill(fixtures.make_inputs(name), "recurrent")
    assert _golden_state(g, s) <= 1e-3


@pytest.mark.parametrize("method", METHODS)
def test_prefill_varlen_benchmark_case(method):
    """4 sequences, lengths U[64,512], sequences 1 and 3 with an initial state."""
    x = W.prefill_varlen(seed=1)
    o, s = _prefill(x, method)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("lengths", [[1], [63], [64], [65], [127, 128, 129], [0, 5, 0],
                                     [200, 1, 64, 3]])
def test_prefill_lengths(method, lengths):
    x = W.prefill_inputs(lengths, seed=sum(lengths) + len(lengths), Hq=4, Hv=8)
    o, s = _prefill(x, method)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("method", METHODS)
def test_prefill_no_state(method):
    x = W.prefill_inputs([100, 37], seed=8, state_mask=[False, False])
    assert x["state"] is None
    o, s = _prefill(x, method)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("decay", [(0.5, 0.999), (0.99, 0.9999), (0.999, 1.0)])
def test_prefill_long_sequences(method, decay):
    """Long-prefill statistics (nonzero state, slow decay) on 2 sequences x 1536 tokens."""
    x = W.prefill_inputs([1536, 1000], seed=33, Hq=4, Hv=8, decay_range=decay)
    o, s = _prefill(x, method)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("method", METHODS)
def test_prefill_f32_gates_bf16_params(method):
    x = W.prefill_inputs([90, 40], seed=12, Hq=4, Hv=8)
    x["a"] = x["a"].float() * 1.5
    x["b"] = x["b"].float()
    x["A_log"] = x["A_log"].to(torch.bfloat16)
    x["dt_bias"] = x["dt_bias"].to(torch.bfloat16)
    o, s = _prefill(x, method)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("method", METHODS)
def test_prefill_gva_ratios(method):
    for Hq, Hv in [(8, 8), (2, 8), (1, 4)]:
        x = W.prefill_inputs([70, 30], seed=Hq * 10 + Hv, Hq=Hq, Hv=Hv)
        o, s = _prefill(x, method)
        ro, rs = _oracle(x)
        assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_long_prefill_full_size_against_oracle():
    """The whole 16 x 8192 long-prefill workload (131072 tokens, Hq 16, Hv 32, nonzero
    state, decay in [0.5, 0.999]) through auto (the tcgen05 pipeline) and the two other
    CUDA kernels, every output element and the full new state against the C oracle."""
    x = W.prefill_long(seed=3)
    assert fk.prefill_method(16 * 8192, num_seqs=16) == "tcgen05"
    ro, rs = _oracle(x)
    for m in ("auto", "chunked", "recurrent"):
        o, s = _prefill(x, m)
        assert_parity(o.cpu(), ro, s.cpu(), rs)
        del o, s


@pytest.mark.parametrize("norm_range", [(0.3, 1.0), (0.5, 1.4)])
def test_unnormalised_keys_auto_at_256_plus_tokens(norm_range):
    """Keys (and queries) that are not unit-norm, with norms in `norm_range` (beta |k|^2
    up to 1.96, so single tokens can flip the sign of the state along k), at >= 256
    packed tokens through auto (the tcgen05 pipeline), against the oracle."""
    x = W.prefill_inputs([700, 300, 257], seed=55, Hq=4, Hv=8, decay_range=(0.9, 0.999))
    g = torch.Generator().manual_seed(56)
    lo, hi = norm_range
    for key in ("q", "k"):
        scale = torch.rand(x[key].shape[:2], generator=g) * (hi - lo) + lo
        x[key] = (x[key].float() * scale[..., None]).to(torch.bfloat16)
    assert fk.prefill_method(x["q"].shape[0], num_seqs=3) == "tcgen05"
    o, s = _prefill(x, "auto")
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_reference_distribution_with_qk_l2norm_auto_at_256_plus_tokens():
    """The reference test's randn inputs at 512 tokens with use_qk_l2norm=True (the
    normalisation Gated DeltaNet layers apply before the recurrence) through auto,
    against the oracle's same option."""
    rng = np.random.Generator(np.random.PCG64(6))
    lengths, Hq, Hv = [300, 212], 4, 8
    T = sum(lengths)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)
    sn = rng.standard_normal
    x = {"q": bf(sn((T, Hq, 128))), "k": bf(sn((T, Hq, 128))), "v": bf(sn((T, Hv, 128))),
         "state": torch.from_numpy(sn((2, Hv, 128, 128)).astype(np.float32)),
         "A_log": torch.from_numpy(sn(Hv).astype(np.float32)), "a": bf(sn((T, Hv))),
         "dt_bias": torch.from_numpy(sn(Hv).astype(np.float32)), "b": bf(sn((T, Hv))),
         "cu_seqlens": torch.tensor([0, 300, T], dtype=torch.int32), "scale": 1.0 / np.sqrt(128)}
    o, s = _prefill(x, "auto", use_qk_l2norm=True)
    ro, rs = c_oracle.prefill(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                              x["b"], x["cu_seqlens"], x["scale"], qk_l2norm=True)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("method", METHODS)
def test_prefill_then_decode_handoff(method):
    """Prefill of T tokens followed by one decode step equals prefill of T+1 tokens."""
    T = 96
    x = W.prefill_inputs([T + 1], seed=44, Hq=4, Hv=8)
    g = _gpu(x)
    o_full, s_full = _prefill(x, method)
    cu = torch.tensor([0, T], dtype=torch.int32, device=DEV)
    sl = lambda t: t[:T]
    o_p, s_p = fk.kernel(sl(g["q"]), sl(g["k"]), sl(g["v"]), g["state"], g["A_log"], sl(g["a"]),
                         g["dt_bias"], sl(g["b"]), cu, g["scale"], method=method)
    o_d, s_d = fk.kernel_decode(g["q"][T:].unsqueeze(0), g["k"][T:].unsqueeze(0),
                                g["v"][T:].unsqueeze(0), s_p, g["A_log"], g["a"][T:].unsqueeze(0),
                                g["dt_bias"], g["b"][T:].unsqueeze(0), g["scale"])
    torch.cuda.synchronize()
    assert_parity(o_d.view(1, 8, 128).cpu(), o_full[T:].cpu(), s_d.cpu(), s_full.cpu())


def test_prefill_output_destination_passing():
    x = W.prefill_inputs([33, 12], seed=5, Hq=4, Hv=8)
    g = _gpu(x)
    out = torch.full((45, 8, 128), 7.0, dtype=torch.bfloat16, device=DEV)
    ns = torch.full((2, 8, 128, 128), 7.0, device=DEV)
    fk.kernel_dps(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                  g["cu_seqlens"], g["scale"], out, ns)
    torch.cuda.synchronize()
    ro, rs = _oracle(x)
    assert_parity(out.cpu(), ro, ns.cpu(), rs)


def test_auto_method_resolution():
    """auto: the tcgen05 pipeline from 256 packed tokens, the mma.sync kernel below, the
    token-serial kernel for at most 32 tokens or under 4 tokens per sequence."""
    assert fk.prefill_method(256) == "tcgen05"
    assert fk.prefill_method(131072, num_seqs=16) == "tcgen05"
    assert fk.prefill_method(255) == "chunked"
    assert fk.prefill_method(33) == "chunked"
    assert fk.prefill_method(32) == "recurrent"
    assert fk.prefill_method(1) == "recurrent"
    assert fk.prefill_method(300, num_seqs=100) == "recurrent"
    assert fk.prefill_method(5000, "recurrent") == "recurrent"


def test_prefill_reference_test_fixture_auto():
    """The reference test's fixture (T = 17, unnormalised keys) through auto, which
    picks the token-serial fp32 kernel for it."""
    name = "prefill_qk4_v8_t17"
    g = fixtures.load(name)
    o, s = _prefill(fixtures.make_inputs(name), "auto")
    assert _golden_state(g, s) <= 1e-3


def test_prefill_caller_workspace():
    """gdn_prefill_ws with a caller-provided workspace equals the pooled-workspace call."""
    import ctypes
    from fastaf_kernel_b200 import _lib
    x = W.prefill_inputs([300, 70, 129], seed=21, Hq=4, Hv=8)
    g = _gpu(x)
    o_ref, s_ref = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"],
                             g["b"], g["cu_seqlens"], g["scale"], method="tcgen05")
    lib = _lib.load()
    T, N = g["q"].shape[0], 3
    nbytes = lib.gdn_prefill_workspace_size(N, T, 8)
    assert nbytes == ((T + 63) // 64 + N) * 8 * 41984
    ws = torch.full((nbytes // 4,), float("nan"), device=DEV)
    out = torch.empty_like(o_ref)
    ns = torch.empty_like(s_ref)
    rc = lib.gdn_prefill_ws(g["q"].data_ptr(), g["k"].data_ptr(), g["v"].data_ptr(), g["state"].data_ptr(),
                            g["A_log"].data_ptr(), g["a"].data_ptr(), g["dt_bias"].data_ptr(),
                            g["b"].data_ptr(), g["cu_seqlens"].data_ptr(), N, T, 4, 8, 128,
                            float(g["scale"]), _lib.GDN_DTYPE_BF16, _lib.GDN_DTYPE_F32, out.data_ptr(),
                            ns.data_ptr(), _lib.GDN_PREFILL_TCGEN05, ws.data_ptr(), nbytes,
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.gdn_last_error()
    small = lib.gdn_prefill_ws(g["q"].data_ptr(), g["k"].data_ptr(), g["v"].data_ptr(), g["state"].data_ptr(),
                               g["A_log"].data_ptr(), g["a"].data_ptr(), g["dt_bias"].data_ptr(),
                               g["b"].data_ptr(), g["cu_seqlens"].data_ptr(), N, T, 4, 8, 128,
                               float(g["scale"]), _lib.GDN_DTYPE_BF16, _lib.GDN_DTYPE_F32, out.data_ptr(),
                               ns.data_ptr(), _lib.GDN_PREFILL_TCGEN05, ws.data_ptr(), nbytes - 16,
                               torch.cuda.current_stream().cuda_stream)
    assert small == _lib.GDN_ERR_INVALID_ARGUMENT
    fk.device_status()
    assert torch.equal(out, o_ref) and torch.equal(ns, s_ref)


def _ws_call(g, N, Hq, Hv):
    """The tcgen05 prefill through gdn_prefill_ws (caller workspace: one stream, no split)."""
    from fastaf_kernel_b200 import _lib
    lib = _lib.load()
    T = g["q"].shape[0]
    nbytes = lib.gdn_prefill_workspace_size(N, T, Hv)
    ws = torch.empty((nbytes,), dtype=torch.uint8, device=DEV)
    out = torch.empty((T, Hv, 128), dtype=torch.bfloat16, device=DEV)
    ns = torch.empty((N, Hv, 128, 128), dtype=torch.float32, device=DEV)
    st = g["state"]
    rc = lib.gdn_prefill_ws(g["q"].data_ptr(), g["k"].data_ptr(), g["v"].data_ptr(),
                            None if st is None else st.data_ptr(), g["A_log"].data_ptr(), g["a"].data_ptr(),
                            g["dt_bias"].data_ptr(), g["b"].data_ptr(), g["cu_seqlens"].data_ptr(), N, T, Hq, Hv,
                            128, float(g["scale"]), _lib.GDN_DTYPE_BF16, _lib.GDN_DTYPE_F32, out.data_ptr(),
                            ns.data_ptr(), _lib.GDN_PREFILL_TCGEN05, ws.data_ptr(), nbytes,
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.gdn_last_error()
    return out, ns


@pytest.mark.parametrize("lengths,Hq,Hv", [
    ([300, 128, 257, 64, 200], 16, 32),                       # 160 chains: two v-heads per prep CTA
    ([90, 64, 130, 70, 65, 200, 64, 100, 64, 77, 64, 150, 64], 4, 12),   # 156 chains: one per prep CTA
    ([256, 0, 191, 64, 300], 16, 32),                         # an empty sequence among them
])
def test_prefill_tc_wave_split_matches_single_stream(lengths, Hq, Hv):
    """A batch of more chains than SMs with a partial last wave: the pooled call splits the
    last (chains mod SMs) chains onto the library's second stream; the result is bit-for-bit
    that of the one-stream launch (caller workspace) and within tolerance of the oracle."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    chains = len(lengths) * Hv
    assert chains > sms and chains % sms > 0, "the case must exercise the split"
    x = W.prefill_inputs(lengths, seed=33, Hq=Hq, Hv=Hv)
    g = _gpu(x)
    o, s = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                     g["cu_seqlens"], g["scale"], method="tcgen05")
    o1, s1 = _ws_call(g, len(lengths), Hq, Hv)
    fk.device_status()
    assert torch.equal(o, o1) and torch.equal(s, s1)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


@pytest.mark.parametrize("n_seqs,Hq,Hv,seed", [
    (37, 4, 8, 61),      # 296 chains = 2 x 148: every sequence ranked, no split
    (300, 4, 8, 62),     # 2400 chains: split tail of 32 chains, the other 296 sequences ranked
])
def test_prefill_tc_longest_first_order_matches_index_order(n_seqs, Hq, Hv, seed):
    """Shuffled lengths (empty, one-token, chunk-boundary and long sequences): the pooled call
    ranks the sequences longest first on the device before its chains; the result is bit for
    bit that of the caller-workspace call, whose chains run in sequence order on one stream,
    and within tolerance of the oracle."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    assert n_seqs * Hv > sms
    rng = np.random.default_rng(seed)
    lengths = [int(v) for v in rng.integers(0, 400, size=n_seqs)]
    lengths[:6] = [0, 1, 64, 65, 128, 0]
    rng.shuffle(lengths)
    x = W.prefill_inputs(lengths, seed=seed, Hq=Hq, Hv=Hv)
    g = _gpu(x)
    o, s = fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                     g["cu_seqlens"], g["scale"], method="tcgen05")
    o1, s1 = _ws_call(g, n_seqs, Hq, Hv)
    fk.device_status()
    assert torch.equal(o, o1) and torch.equal(s, s1)
    ro, rs = _oracle(x)
    assert_parity(o.cpu(), ro, s.cpu(), rs)


def test_prefill_tc_wave_split_under_graph_capture():
    """The split launch (fork onto the library's second stream, join back) records into a
    CUDA graph, and replaying it reproduces the eager result."""
    x = W.prefill_inputs([300, 128, 257, 64, 200], seed=34)
    g = _gpu(x)
    run = lambda: fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                            g["cu_seqlens"], g["scale"], method="tcgen05", validate=False)
    o, s = run()
    torch.cuda.synchronize()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cs):
        og, sg = run()
    graph.replay()
    torch.cuda.synchronize()
    fk.device_status()
    assert torch.equal(og, o) and torch.equal(sg, s)
    del graph


def test_prefill_tc_eager_call_during_a_capture_that_holds_the_split():
    """A capture that contains a split call (the library's second stream joins that
    capture) and, before the capture ends, an eager 160-chain call on another stream:
    the eager call must not touch the captured second stream (it runs unsplit on its own
    stream), and both it and the graph's replay equal the plain eager result."""
    x = W.prefill_inputs([300, 128, 257, 64, 200], seed=36)
    g = _gpu(x)

    def run(out=None, ns=None):
        return fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                         g["cu_seqlens"], g["scale"], method="tcgen05", output=out, new_state=ns)

    o_ref, s_ref = run()
    torch.cuda.synchronize()
    o_eager = torch.empty_like(o_ref)
    s_eager = torch.empty_like(s_ref)
    other = torch.cuda.Stream()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    other.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cs, capture_error_mode="relaxed"):
        og, sg = run()
        with torch.cuda.stream(other):
            run(o_eager, s_eager)
    other.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    fk.device_status()
    assert torch.equal(o_eager, o_ref) and torch.equal(s_eager, s_ref)
    assert torch.equal(og, o_ref) and torch.equal(sg, s_ref)
    del graph


@pytest.mark.parametrize("n_seqs", [3, 16])
def test_prefill_tc_launch_count_matches_query(n_seqs):
    """The kernels one pooled tcgen05 call launches (counted by the profiler) are what
    gdn_prefill_tc_launches reports: 2 below the wave-split threshold; above it 4, plus the
    kernel that ranks the sequences longest first."""
    from torch.profiler import ProfilerActivity, profile
    from fastaf_kernel_b200 import _lib
    x = W.prefill_inputs([128] * n_seqs, seed=35)
    g = _gpu(x)
    run = lambda: fk.kernel(g["q"], g["k"], g["v"], g["state"], g["A_log"], g["a"], g["dt_bias"], g["b"],
                            g["cu_seqlens"], g["scale"], method="tcgen05", validate=False)
    run()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ours = [n for n in names if "chunk_prep_kernel" in n or "prefill_tc_kernel" in n or "chain_order_kernel" in n]
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    assert len(ours) == _lib.load().gdn_prefill_tc_launches(n_seqs, 16, 32, sms), names
