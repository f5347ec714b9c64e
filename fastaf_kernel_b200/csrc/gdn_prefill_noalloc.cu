// gdn_prefill_noalloc.cu -- gdn_prefill_noalloc(): the tcgen05 prefill with its
// per-chunk workspace in a fixed-size device array of this library instead of
// memory allocated per call.
//
// Who needs it: callers that must not allocate device memory while serving, e.g.
//   * a serving engine that reserves (nearly) all HBM up front for its own state and
//     cache pools, where any allocation outside them -- even from a stream-ordered
//     pool -- can fail for lack of memory in the middle of a batch;
//   * latency-critical loops that cannot afford the driver allocation a memory pool
//     makes the first time it grows;
//   * callers whose memory accounting forbids allocations outside their own allocator.
// gdn_prefill / gdn_prefill_ex take the workspace from a library-owned memory pool and
// gdn_prefill_ws from the caller; this entry point needs neither.
//
// The array holds kNoAllocWorkspaceBytes (64 MiB), enough for
// (ceil(T/64) + N) * Hv <= 1598 chunk-head slots, e.g. T = 2560 tokens in up to 9
// sequences with 32 v-heads.  Larger calls are rejected before any launch.  Nothing in
// the array has to start at zero: the prep kernel writes every slot the chain kernel
// reads, in the same call.  There is one array per device, so calls whose executions
// overlap on the device (different streams or host threads) race on it.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "gdn_b200.h"
#include "gdn_launch.h"

namespace {

constexpr size_t kNoAllocWorkspaceBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_noalloc_ws[kNoAllocWorkspaceBytes];

// Device address of g_noalloc_ws on the current device.  Outside a stream capture it is
// looked up on every call (cudaGetSymbolAddress with that device current: a table lookup
// once the module is loaded), so it follows a new primary context after a device reset;
// inside a capture the last address seen on this device is used, since loading the module
// there is not allowed -- so the device's first call must come before any capture.
cudaError_t noalloc_workspace(void **ptr, cudaStream_t stream) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void *addr[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cs);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (cs == cudaStreamCaptureStatusNone || addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_ws);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *ptr = addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" {

int gdn_prefill_noalloc(const void *q, const void *k, const void *v, const float *state,
                        const void *A_log, const void *a, const void *dt_bias, const void *b,
                        const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                        int num_qk_heads, int num_v_heads, int head_size, float scale,
                        int gate_dtype, int param_dtype, void *output, float *new_state,
                        void *stream) {
    char msg[256];
    if (num_seqs < 0 || total_tokens < 0 || num_v_heads <= 0) {
        gdn::set_last_error("gdn_prefill_noalloc: num_seqs, total_tokens must be >= 0 and num_v_heads > 0");
        return GDN_ERR_INVALID_ARGUMENT;
    }
    const size_t need = gdn_prefill_workspace_size(num_seqs, total_tokens, num_v_heads);
    if (need > kNoAllocWorkspaceBytes) {
        std::snprintf(msg, sizeof(msg),
                      "gdn_prefill_noalloc: %lld sequences of %lld tokens with %d v-heads need %zu bytes "
                      "of workspace; the fixed workspace holds %zu",
                      static_cast<long long>(num_seqs), static_cast<long long>(total_tokens), num_v_heads,
                      need, kNoAllocWorkspaceBytes);
        gdn::set_last_error(msg);
        return GDN_ERR_INVALID_ARGUMENT;
    }
    void *ws = nullptr;
    const cudaError_t e = noalloc_workspace(&ws, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        std::snprintf(msg, sizeof(msg), "gdn_prefill_noalloc: workspace address: %s", cudaGetErrorString(e));
        gdn::set_last_error(msg);
        return GDN_ERR_CUDA;
    }
    return gdn_prefill_ws(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, num_seqs, total_tokens,
                          num_qk_heads, num_v_heads, head_size, scale, gate_dtype, param_dtype, output,
                          new_state, GDN_PREFILL_TCGEN05, ws, kNoAllocWorkspaceBytes, stream);
}

}  // extern "C"
