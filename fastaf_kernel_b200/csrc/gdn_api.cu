// gdn_api.cu -- the C ABI declared in include/gdn_b200.h.
//
// Validates arguments on the host (the reference does no validation; its
// harness maps Python exceptions to RUNTIME_ERROR, scripts/run_local_modify.py:280-286),
// selects the kernel and launches it on the caller's stream.  Nothing here
// allocates device memory or synchronizes.
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>

#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace {

thread_local char g_last_error[512] = "";
// From 256 packed tokens the tcgen05 pipeline beats the single-launch mma.sync kernel
// on B200 (256 tokens 43 vs 51 us, 1024 tokens 56 vs 84 us at Hq 16 / Hv 32); below it
// the extra prep launch does not pay off (64-128 tokens: 42 vs 32 us).
constexpr int64_t kAutoTcMinTokens = 256;
constexpr int64_t kAutoRecurrentMaxTokens = 32;

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool ranges_overlap(const void *a, size_t na, const void *b, size_t nb) {
    const auto x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + nb && y < x + na;
}

int check_common(int Hq, int Hv, int D, int gate_dtype, int param_dtype, const void *q,
                 const void *k, const void *v, const void *A_log, const void *a,
                 const void *dt_bias, const void *b, const void *out, const float *new_state) {
    if (D != gdn::kHeadDim)
        return fail(GDN_ERR_UNSUPPORTED, "head_size=%d is not supported (only 128)", D);
    if (Hq <= 0 || Hv <= 0 || Hv % Hq != 0)
        return fail(GDN_ERR_INVALID_ARGUMENT,
                    "num_v_heads=%d must be a positive multiple of num_qk_heads=%d", Hv, Hq);
    if ((gate_dtype != GDN_DTYPE_F32 && gate_dtype != GDN_DTYPE_BF16) ||
        (param_dtype != GDN_DTYPE_F32 && param_dtype != GDN_DTYPE_BF16))
        return fail(GDN_ERR_INVALID_ARGUMENT, "gate_dtype/param_dtype must be 0 (f32) or 1 (bf16)");
    if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state)
        return fail(GDN_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(new_state))
        return fail(GDN_ERR_INVALID_ARGUMENT, "q/k/v/output/new_state must be 16-byte aligned");
    return GDN_OK;
}

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return GDN_OK;
    return fail(GDN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Stream-ordered workspace for callers that pass none: a library-owned memory pool
// per device whose release threshold keeps its memory between calls, so a
// steady-state call takes its workspace from the pool without a driver allocation.
cudaError_t pool_alloc(void **ptr, size_t bytes, cudaStream_t stream) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static cudaMemPool_t pools[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (pools[dev] == nullptr) {
            cudaMemPoolProps props;
            std::memset(&props, 0, sizeof(props));
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            e = cudaMemPoolCreate(&pools[dev], &props);
            if (e != cudaSuccess) {
                pools[dev] = nullptr;
                return e;
            }
            uint64_t keep = ~uint64_t(0);
            cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
        }
        pool = pools[dev];
    }
    return cudaMallocFromPoolAsync(ptr, bytes, pool, stream);
}

}  // namespace

namespace gdn {
void set_last_error(const char *msg) { std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }
}  // namespace gdn

extern "C" {

const char *gdn_last_error(void) { return g_last_error; }

const char *gdn_version(void) { return "gdn_b200 0.1.0 sm_100a"; }

int gdn_device_status(void *stream) {
    g_last_error[0] = '\0';
    int code = 0;
    const cudaError_t e = gdn::read_device_status(static_cast<cudaStream_t>(stream), &code, true);
    if (e != cudaSuccess) return cuda_status(e, "gdn_device_status");
    if (code == gdn::kErrCuSeqlens)
        return fail(GDN_ERR_INVALID_ARGUMENT,
                    "cu_seqlens was not an offsets array over [0, total_tokens] (an entry out of range, "
                    "a decreasing pair, or a first entry != 0 / last entry != total_tokens); the kernels "
                    "clamped it, the results of the affected sequences are meaningless");
    if (code != 0)
        return fail(GDN_ERR_DEVICE_TIMEOUT, "a prefill CTA timed out waiting at site %d", code);
    return GDN_OK;
}

uint64_t gdn_set_wait_limit_ns(uint64_t ns) { return gdn::set_wait_limit_ns(ns); }

int gdn_decode(const void *q, const void *k, const void *v, const float *state,
               const void *A_log, const void *a, const void *dt_bias, const void *b,
               int64_t batch, int num_qk_heads, int num_v_heads, int head_size, float scale,
               int gate_dtype, int param_dtype, void *output, float *new_state,
               void *stream) {
    return gdn_decode_flags(q, k, v, state, A_log, a, dt_bias, b, batch, num_qk_heads, num_v_heads,
                            head_size, scale, gate_dtype, param_dtype, output, new_state, 0, stream);
}

int gdn_decode_flags(const void *q, const void *k, const void *v, const float *state,
                     const void *A_log, const void *a, const void *dt_bias, const void *b,
                     int64_t batch, int num_qk_heads, int num_v_heads, int head_size, float scale,
                     int gate_dtype, int param_dtype, void *output, float *new_state, int flags,
                     void *stream) {
    return gdn_decode_strided(q, k, v, state, A_log, a, dt_bias, b, batch, num_qk_heads, num_v_heads, head_size,
                              scale, gate_dtype, param_dtype, output, new_state, 0, 0, flags, stream);
}

int gdn_decode_strided(const void *q, const void *k, const void *v, const float *state,
                       const void *A_log, const void *a, const void *dt_bias, const void *b,
                       int64_t batch, int num_qk_heads, int num_v_heads, int head_size, float scale,
                       int gate_dtype, int param_dtype, void *output, float *new_state,
                       int64_t a_row_stride, int64_t b_row_stride, int flags, void *stream) {
    g_last_error[0] = '\0';
    if ((a_row_stride != 0 && a_row_stride < num_v_heads) || (b_row_stride != 0 && b_row_stride < num_v_heads) ||
        a_row_stride > 0x7fffffff || b_row_stride > 0x7fffffff)
        return fail(GDN_ERR_INVALID_ARGUMENT,
                    "a/b row strides (%lld, %lld) must be 0 or in [num_v_heads=%d, 2^31)",
                    (long long)a_row_stride, (long long)b_row_stride, num_v_heads);
    if (flags & ~GDN_FLAG_QK_L2NORM) return fail(GDN_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
    int rc = check_common(num_qk_heads, num_v_heads, head_size, gate_dtype, param_dtype, q, k, v,
                          A_log, a, dt_bias, b, output, new_state);
    if (rc) return rc;
    if (batch < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "batch=%lld < 0", (long long)batch);
    const size_t state_bytes = static_cast<size_t>(batch) * num_v_heads * head_size * head_size * 4;
    if (state) {
        if (!aligned16(state)) return fail(GDN_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
        if (state != new_state && ranges_overlap(state, state_bytes, new_state, state_bytes))
            return fail(GDN_ERR_INVALID_ARGUMENT,
                        "new_state partially overlaps state (only exact aliasing is allowed)");
    }
    if (batch == 0) return GDN_OK;
    gdn::DecodeArgs p{q, k, v, state, A_log, a, dt_bias, b, batch, num_qk_heads, num_v_heads,
                      scale == 0.0f ? 1.0f / sqrtf(static_cast<float>(head_size)) : scale,
                      gate_dtype, param_dtype, output, new_state, (flags & GDN_FLAG_QK_L2NORM) ? 1 : 0};
    p.a_stride = a_row_stride;
    p.b_stride = b_row_stride;
    return cuda_status(gdn::launch_decode(p, static_cast<cudaStream_t>(stream)), "gdn_decode launch");
}

// The optional gated RMSNorm of the output, as its own pass after the prefill kernels
// that do not fuse it (the tcgen05 chains apply it in their output stores).
static int gate_output(const gdn::PrefillArgs &p, cudaStream_t s) {
    if (!p.out_gate) return GDN_OK;
    return cuda_status(gdn::launch_output_gate(p.out, p.out_gate, p.norm_w, p.norm_w_dtype,
                                               p.total_tokens * p.Hv, p.norm_eps, s),
                       "gdn_prefill output gate launch");
}

// The tcgen05 prefill of a validated call: workspace from the caller or the pool.
static int prefill_tc_call(const gdn::PrefillArgs &p, void *workspace, size_t workspace_bytes, cudaStream_t s) {
    if (!gdn::prefill_tc_supported(p))
        return fail(GDN_ERR_UNSUPPORTED,
                    "the tcgen05 prefill needs an sm_100 device and total_tokens >= 64");
    const size_t need = gdn::prefill_tc_workspace_bytes(p);
    if (workspace) {
        if (workspace_bytes < need)
            return fail(GDN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is smaller than the %zu needed",
                        workspace_bytes, need);
        const cudaError_t e = gdn::launch_prefill_tc(p, workspace, s);   // (gating fused into its stores)
        if (e != cudaSuccess) return cuda_status(e, "gdn_prefill (tcgen05) launch");
        return GDN_OK;
    }
    // The pool block also holds the sequences' launch order (need is a multiple of 256 bytes).
    void *ws = nullptr;
    cudaError_t e = pool_alloc(&ws, need + static_cast<size_t>(p.num_seqs) * sizeof(int32_t), s);
    if (e != cudaSuccess) return cuda_status(e, "gdn_prefill (tcgen05) workspace");
    e = gdn::launch_prefill_tc(p, ws, s, /*overlap=*/true,
                               reinterpret_cast<int32_t *>(static_cast<char *>(ws) + need));
    const cudaError_t ef = cudaFreeAsync(ws, s);
    if (e != cudaSuccess) return cuda_status(e, "gdn_prefill (tcgen05) launch");
    if (ef != cudaSuccess) return cuda_status(ef, "gdn_prefill (tcgen05) workspace release");
    return GDN_OK;   // (the chains' stores applied the gating)
}

static int prefill_impl(const void *q, const void *k, const void *v, const float *state,
                        const void *A_log, const void *a, const void *dt_bias, const void *b,
                        const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                        int num_qk_heads, int num_v_heads, int head_size, float scale,
                        int gate_dtype, int param_dtype, void *output, float *new_state,
                        int method, void *workspace, size_t workspace_bytes, void *stream,
                        int flags = 0, const void *out_gate = nullptr, const void *norm_w = nullptr,
                        int norm_w_dtype = 0, float norm_eps = 0.0f, int64_t a_stride = 0,
                        int64_t b_stride = 0) {
    g_last_error[0] = '\0';
    if (flags & ~GDN_FLAG_QK_L2NORM) return fail(GDN_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
    if ((a_stride != 0 && a_stride < num_v_heads) || (b_stride != 0 && b_stride < num_v_heads) ||
        a_stride > 0x7fffffff || b_stride > 0x7fffffff)
        return fail(GDN_ERR_INVALID_ARGUMENT,
                    "a/b row strides (%lld, %lld) must be 0 or in [num_v_heads=%d, 2^31)",
                    (long long)a_stride, (long long)b_stride, num_v_heads);
    int rc = check_common(num_qk_heads, num_v_heads, head_size, gate_dtype, param_dtype, q, k, v,
                          A_log, a, dt_bias, b, output, new_state);
    if (rc) return rc;
    if (num_seqs < 0 || total_tokens < 0)
        return fail(GDN_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0");
    if (total_tokens >= (int64_t(1) << 31))
        return fail(GDN_ERR_INVALID_ARGUMENT, "total_tokens must fit in int32 (cu_seqlens is int32)");
    if (!cu_seqlens) return fail(GDN_ERR_INVALID_ARGUMENT, "null cu_seqlens");
    const size_t state_bytes = static_cast<size_t>(num_seqs) * num_v_heads * head_size * head_size * 4;
    if (state) {
        if (!aligned16(state)) return fail(GDN_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
        if (ranges_overlap(state, state_bytes, new_state, state_bytes))
            return fail(GDN_ERR_INVALID_ARGUMENT, "prefill new_state must not overlap state");
    }
    if (method != GDN_PREFILL_AUTO && method != GDN_PREFILL_CHUNKED && method != GDN_PREFILL_RECURRENT &&
        method != GDN_PREFILL_TCGEN05)
        return fail(GDN_ERR_INVALID_ARGUMENT, "unknown prefill method %d", method);
    if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return fail(GDN_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    if (num_seqs == 0) return GDN_OK;
    gdn::PrefillArgs p{q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                       num_qk_heads, num_v_heads,
                       scale == 0.0f ? 1.0f / sqrtf(static_cast<float>(head_size)) : scale,
                       gate_dtype, param_dtype, output, new_state};
    p.out_gate = out_gate;
    p.norm_w = norm_w;
    p.norm_w_dtype = norm_w_dtype;
    p.norm_eps = norm_eps;
    p.status = gdn::device_status_word();
    p.a_stride = a_stride;
    p.b_stride = b_stride;
    const auto s = static_cast<cudaStream_t>(stream);
    if (flags & GDN_FLAG_QK_L2NORM) {
        // Normalised q and k into pool scratch, then the prefill on them.
        const size_t qk_bytes = static_cast<size_t>(total_tokens) * num_qk_heads * head_size * 2;
        if (qk_bytes == 0)
            return prefill_impl(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                                num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                                new_state, method, workspace, workspace_bytes, stream, 0, out_gate, norm_w,
                                norm_w_dtype, norm_eps, a_stride, b_stride);
        void *qk = nullptr;
        cudaError_t e = pool_alloc(&qk, 2 * qk_bytes, s);
        if (e != cudaSuccess) return cuda_status(e, "gdn_prefill (qk l2norm) scratch");
        void *qn = qk, *kn = static_cast<char *>(qk) + qk_bytes;
        e = gdn::launch_qk_l2norm(q, k, total_tokens * num_qk_heads, qn, kn, s);
        int rc2 = e != cudaSuccess ? cuda_status(e, "gdn_prefill (qk l2norm) launch")
                                   : prefill_impl(qn, kn, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs,
                                                  total_tokens, num_qk_heads, num_v_heads, head_size, scale,
                                                  gate_dtype, param_dtype, output, new_state, method, workspace,
                                                  workspace_bytes, stream, 0, out_gate, norm_w, norm_w_dtype,
                                                  norm_eps, a_stride, b_stride);
        const cudaError_t ef = cudaFreeAsync(qk, s);
        if (rc2 != GDN_OK) return rc2;
        return cuda_status(ef, "gdn_prefill (qk l2norm) scratch release");
    }
    // auto: gdn_prefill_resolve's choice
    if (method == GDN_PREFILL_AUTO) method = gdn_prefill_resolve(total_tokens, num_seqs, method);
    if (method == GDN_PREFILL_TCGEN05) return prefill_tc_call(p, workspace, workspace_bytes, s);
    const bool chunked_ok = gdn::prefill_chunked_supported(p);
    if (method == GDN_PREFILL_CHUNKED && !chunked_ok)
        return fail(GDN_ERR_UNSUPPORTED, "the chunked tensor-core prefill is not available here");
    const bool recurrent = method == GDN_PREFILL_RECURRENT || (method == GDN_PREFILL_AUTO && !chunked_ok);
    cudaError_t e = recurrent ? gdn::launch_prefill_recurrent(p, s) : gdn::launch_prefill_chunked(p, s);
    if (e != cudaSuccess) return cuda_status(e, recurrent ? "gdn_prefill (recurrent) launch" : "gdn_prefill (chunked) launch");
    return gate_output(p, s);
}

int gdn_prefill_ex(const void *q, const void *k, const void *v, const float *state,
                   const void *A_log, const void *a, const void *dt_bias, const void *b,
                   const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                   int num_qk_heads, int num_v_heads, int head_size, float scale,
                   int gate_dtype, int param_dtype, void *output, float *new_state,
                   int method, void *stream) {
    return prefill_impl(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                        num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                        new_state, method, nullptr, 0, stream);
}

int gdn_prefill_flags(const void *q, const void *k, const void *v, const float *state,
                      const void *A_log, const void *a, const void *dt_bias, const void *b,
                      const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                      int num_qk_heads, int num_v_heads, int head_size, float scale,
                      int gate_dtype, int param_dtype, void *output, float *new_state,
                      int method, int flags, void *stream) {
    return prefill_impl(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                        num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                        new_state, method, nullptr, 0, stream, flags);
}

int gdn_prefill_strided(const void *q, const void *k, const void *v, const float *state,
                        const void *A_log, const void *a, const void *dt_bias, const void *b,
                        const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                        int num_qk_heads, int num_v_heads, int head_size, float scale,
                        int gate_dtype, int param_dtype, void *output, float *new_state,
                        int64_t a_row_stride, int64_t b_row_stride, int method, int flags, void *stream) {
    return prefill_impl(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                        num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                        new_state, method, nullptr, 0, stream, flags, nullptr, nullptr, 0, 0.0f, a_row_stride,
                        b_row_stride);
}

int gdn_prefill_gated(const void *q, const void *k, const void *v, const float *state,
                      const void *A_log, const void *a, const void *dt_bias, const void *b,
                      const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                      int num_qk_heads, int num_v_heads, int head_size, float scale,
                      int gate_dtype, int param_dtype, void *output, float *new_state,
                      const void *out_gate, const void *norm_weight, int norm_weight_dtype, float eps,
                      int method, int flags, void *stream) {
    g_last_error[0] = '\0';
    if (!out_gate || !norm_weight) return fail(GDN_ERR_INVALID_ARGUMENT, "null gate or norm weight");
    if (!aligned16(out_gate)) return fail(GDN_ERR_INVALID_ARGUMENT, "gate must be 16-byte aligned");
    if (norm_weight_dtype != GDN_DTYPE_F32 && norm_weight_dtype != GDN_DTYPE_BF16)
        return fail(GDN_ERR_INVALID_ARGUMENT, "unknown norm_weight_dtype %d", norm_weight_dtype);
    if (!(eps >= 0.0f)) return fail(GDN_ERR_INVALID_ARGUMENT, "eps must be >= 0");
    return prefill_impl(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                        num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                        new_state, method, nullptr, 0, stream, flags, out_gate, norm_weight, norm_weight_dtype,
                        eps);
}

int gdn_prefill_ws(const void *q, const void *k, const void *v, const float *state,
                   const void *A_log, const void *a, const void *dt_bias, const void *b,
                   const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                   int num_qk_heads, int num_v_heads, int head_size, float scale,
                   int gate_dtype, int param_dtype, void *output, float *new_state,
                   int method, void *workspace, size_t workspace_bytes, void *stream) {
    return prefill_impl(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                        num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                        new_state, method, workspace, workspace_bytes, stream);
}

int gdn_output_gate(void *output, const void *gate, const void *weight, int weight_dtype, int64_t num_vectors,
                    int head_size, float eps, void *stream) {
    g_last_error[0] = '\0';
    if (head_size != 128) return fail(GDN_ERR_UNSUPPORTED, "head_size=%d (only 128 is built)", head_size);
    if (num_vectors < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "num_vectors=%lld < 0", (long long)num_vectors);
    if (weight_dtype != GDN_DTYPE_F32 && weight_dtype != GDN_DTYPE_BF16)
        return fail(GDN_ERR_INVALID_ARGUMENT, "unknown weight_dtype %d", weight_dtype);
    if (!(eps >= 0.0f)) return fail(GDN_ERR_INVALID_ARGUMENT, "eps must be >= 0");
    if (num_vectors == 0) return GDN_OK;
    if (!output || !gate || !weight) return fail(GDN_ERR_INVALID_ARGUMENT, "null output, gate or weight");
    if (!aligned16(output) || !aligned16(gate))
        return fail(GDN_ERR_INVALID_ARGUMENT, "output and gate must be 16-byte aligned");
    return cuda_status(gdn::launch_output_gate(output, gate, weight, weight_dtype, num_vectors, eps,
                                               static_cast<cudaStream_t>(stream)),
                       "gdn_output_gate launch");
}

int gdn_prefill_tc_launches(int64_t num_seqs, int num_qk_heads, int num_v_heads, int num_sms) {
    if (num_seqs <= 0 || num_qk_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_qk_heads != 0) return 0;
    const int nh = ((num_v_heads / num_qk_heads) % 2 == 0) ? 2 : 1;
    return (gdn::prefill_tc_overlap_tail(num_seqs * num_v_heads, num_sms, nh) > 0 ? 4 : 2) +
           (gdn::prefill_tc_orders_chains(num_seqs, num_v_heads, num_sms) ? 1 : 0);
}

int gdn_prefill_resolve(int64_t total_tokens, int64_t num_seqs, int method) {
    gdn::PrefillArgs p{};
    p.total_tokens = total_tokens;
    p.num_seqs = num_seqs;
    if (method == GDN_PREFILL_AUTO) {
        // Tiny batches and batches of very short sequences: the token-serial fp32 kernel
        // costs the same or less there (T <= 32: equal; 64 sequences of 1 token: 101 vs
        // 210 us) and follows the reference's fp32 recurrence exactly, also on inputs
        // with unnormalised keys that amplify the state.
        if (total_tokens <= kAutoRecurrentMaxTokens || total_tokens < 4 * num_seqs) return GDN_PREFILL_RECURRENT;
        if (total_tokens >= kAutoTcMinTokens && gdn::prefill_tc_supported(p)) return GDN_PREFILL_TCGEN05;
        return gdn::prefill_chunked_supported(p) ? GDN_PREFILL_CHUNKED : GDN_PREFILL_RECURRENT;
    }
    return method;
}

size_t gdn_prefill_workspace_size(int64_t num_seqs, int64_t total_tokens, int num_v_heads) {
    if (num_seqs < 0 || total_tokens < 0 || num_v_heads <= 0) return 0;
    gdn::PrefillArgs p{};
    p.num_seqs = num_seqs;
    p.total_tokens = total_tokens;
    p.Hv = num_v_heads;
    return gdn::prefill_tc_workspace_bytes(p);
}

int gdn_prefill(const void *q, const void *k, const void *v, const float *state,
                const void *A_log, const void *a, const void *dt_bias, const void *b,
                const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                int num_qk_heads, int num_v_heads, int head_size, float scale, int gate_dtype,
                int param_dtype, void *output, float *new_state, void *stream) {
    return gdn_prefill_ex(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs,
                          total_tokens, num_qk_heads, num_v_heads, head_size, scale, gate_dtype,
                          param_dtype, output, new_state, GDN_PREFILL_AUTO, stream);
}

}  // extern "C"
