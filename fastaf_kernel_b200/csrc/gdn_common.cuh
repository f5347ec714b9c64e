// gdn_common.cuh -- shared device helpers for the Gated DeltaNet kernels (sm_100a).
#pragma once

#include "gdn_chunk_common.cuh"

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

__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// The hardware's tanh approximation (MUFU; a few units of 2^-11 relative).
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Gated RMSNorm of one 128-element bf16 vector held by an aligned group of 16 lanes,
// 8 elements (one 16-byte word) each: o / sqrt(mean(o^2) + eps) * w * silu(z), fp32,
// rounded to bf16.  ow / zw are this lane's words of o and z, wv its 8 weights.  Every
// lane of the warp must call it (full-warp shuffles).  Built for few instructions, since
// the tcgen05 prefill's output-store warps run it beside the chain's critical path: packed
// f32x2 arithmetic, the hardware reciprocal square root, and sigmoid(z) = (1 + tanh(z/2))/2
// with the hardware tanh -- a few units of 2^-11 relative, below the bf16 rounding of the
// result.  The standalone pass uses this same routine, so both give the same bits.
__device__ __forceinline__ uint4 gated_rmsnorm16(uint4 ov, uint4 zv, const float (&wv)[8], float eps) {
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
    uint64_t x2[4];
    uint64_t ss2 = f2(0.0f, 0.0f);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        x2[e] = f2(bf16_lo(ow[e]), bf16_hi(ow[e]));
        ss2 = fma_f2(x2[e], x2[e], ss2);
    }
    float sa, sb;
    unf2(ss2, sa, sb);
    float ss = sa + sb;
#pragma unroll
    for (int m = 1; m < 16; m <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    const float inv = rsqrtf(ss * (1.0f / 128.0f) + eps);
    const uint64_t inv2 = f2(inv, inv), half2 = f2(0.5f, 0.5f);
    uint32_t r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float g0 = bf16_lo(zw[e]), g1 = bf16_hi(zw[e]);
        const uint64_t g2 = f2(g0, g1);
        const uint64_t sg2 = fma_f2(f2(tanh_approx(0.5f * g0), tanh_approx(0.5f * g1)), half2, half2);
        float y0, y1;
        unf2(mul_f2(mul_f2(mul_f2(x2[e], inv2), f2(wv[2 * e], wv[2 * e + 1])), mul_f2(g2, sg2)), y0, y1);
        r[e] = pack_bf16x2(y0, y1);
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
}

// Streaming (evict-first) 128-bit global accesses for data touched once.
__device__ __forceinline__ float4 ld_stream(const float4 *p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4 *p, float4 v) { __stcs(p, v); }

}  // namespace gdn
