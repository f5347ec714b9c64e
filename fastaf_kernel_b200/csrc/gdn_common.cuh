// gdn_common.cuh -- shared device helpers for the Gated DeltaNet kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 128;  // the only head size the kernels are built for

// Element types of the gate inputs (a, b) and parameters (A_log, dt_bias);
// the codes match GDN_DTYPE_F32 / GDN_DTYPE_BF16 of the C ABI.
__device__ __forceinline__ float load_scalar(const void *p, int64_t i, int dtype) {
    return dtype == 1 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i])
                      : reinterpret_cast<const float *>(p)[i];
}

// torch.nn.functional.softplus(x) with beta=1, threshold=20: the gate formula
// of solution/gdn_baseline_torch.py:43 (the Triton helper at
// solution/triton/kernel.py:107-119 differs only below x=-20).
__device__ __forceinline__ float softplus_torch(float x) {
    return x > 20.0f ? x : log1pf(expf(x));
}

// log(alpha) = -exp(A_log) * softplus(a + dt_bias)  (solution/gdn_baseline_torch.py:42-43)
__device__ __forceinline__ float log_decay(float exp_A_log, float a, float dt_bias) {
    return -exp_A_log * softplus_torch(a + dt_bias);
}

// Code a prefill kernel records in the library's device status word (read and cleared
// by gdn_device_status) when cu_seqlens is not an offsets array over [0, T]: an entry
// outside [0, T], a decreasing pair, cu_seqlens[0] != 0 or cu_seqlens[N] != T.  The
// kernels clamp such entries, so nothing is read or written out of bounds; the results
// of the affected sequences are then meaningless.  (Bounded-wait give-ups record their
// site, 1..99, in the same word.)
constexpr int kErrCuSeqlens = 100;

// Called by one thread of each CTA that processes sequence n of N: the raw bounds of
// sequence n against the offsets contract (first error kept).
__device__ __forceinline__ void check_seq_bounds(const int32_t *cu, int64_t n, int64_t N, int64_t T, int *status) {
    if (status == nullptr) return;
    const int64_t s0 = cu[n], s1 = cu[n + 1];
    if (s0 < 0 || s1 > T || s1 < s0 || (n == 0 && s0 != 0) || (n == N - 1 && s1 != T))
        atomicCAS(status, 0, kErrCuSeqlens);
}

// beta = sigmoid(b)  (solution/gdn_baseline_torch.py:44)
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float bf16_lo(uint32_t packed) {
    return __uint_as_float(packed << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t packed) {
    return __uint_as_float(packed & 0xffff0000u);
}

// Round-to-nearest-even fp32 -> bf16, two values packed (lo in bits 0-15).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Gated RMSNorm of one 128-element bf16 vector held by an aligned group of 16 lanes,
// 8 elements (one 16-byte word) each: o / sqrt(mean(o^2) + eps) * w * silu(z), fp32,
// rounded to bf16.  ow / zw are this lane's words of o and z, wv its 8 weights.  Every
// lane of the warp must call it (full-warp shuffles).  The reciprocal square root, the
// exponential and the division of silu use the hardware approximations (rsqrtf, __expf,
// __fdividef: a few ulp in fp32, far below the bf16 rounding of the result), so the
// tcgen05 prefill's output-store warps keep up with a chunk in their shared budget; the
// standalone pass uses this same routine, so both give the same bits.
__device__ __forceinline__ uint4 gated_rmsnorm16(uint4 ov, uint4 zv, const float (&wv)[8], float eps) {
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
    float x[8], g[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        x[2 * e] = bf16_lo(ow[e]); x[2 * e + 1] = bf16_hi(ow[e]);
        g[2 * e] = bf16_lo(zw[e]); g[2 * e + 1] = bf16_hi(zw[e]);
    }
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
    for (int m = 1; m < 16; m <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
    uint32_t r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float y[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = 2 * e + u;
            y[u] = x[i] * inv * wv[i] * __fdividef(g[i], 1.0f + __expf(-g[i]));
        }
        r[e] = pack_bf16x2(y[0], y[1]);
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
}

// Streaming (evict-first) 128-bit global accesses for data touched once.
__device__ __forceinline__ float4 ld_stream(const float4 *p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4 *p, float4 v) { __stcs(p, v); }

}  // namespace gdn
