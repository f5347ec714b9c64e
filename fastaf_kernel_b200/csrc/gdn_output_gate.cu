// gdn_output_gate.cu -- the gated RMSNorm that Gated DeltaNet layers apply to the
// recurrence output before the output projection (not part of the reference, whose
// entry points return o itself):
//
//   out = o / sqrt(mean(o^2) + eps) * w * silu(z),   silu(z) = z / (1 + exp(-z)),
//
// per 128-element head vector, in fp32 from the bf16 o and z, rounded to bf16.  It
// reads and writes the output once (in place); 16 lanes own one vector, 8 elements
// (one 16-byte load) each, and reduce the sum of squares with a 16-lane butterfly.
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

__global__ void __launch_bounds__(256)
output_gate_kernel(__nv_bfloat16 *__restrict__ o, const __nv_bfloat16 *__restrict__ z, const void *w,
                   int w_dtype, int64_t vectors, float eps) {
    const int64_t vec = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
    const int l16 = threadIdx.x & 15;
    // Groups past the end work on vector 0 and store nothing, so every lane takes part
    // in the full-warp shuffles.
    const bool live = vec < vectors;
    const int64_t base = (live ? vec : 0) * kHeadDim + l16 * 8;
    const uint4 ov = *reinterpret_cast<const uint4 *>(o + base);
    const uint4 zv = __ldg(reinterpret_cast<const uint4 *>(z + base));
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
    const float inv = 1.0f / sqrtf(ss * (1.0f / kHeadDim) + eps);
    uint32_t r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float y[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = 2 * e + u;
            const float wi = load_scalar(w, l16 * 8 + i, w_dtype);
            const float silu = g[i] / (1.0f + expf(-g[i]));
            y[u] = x[i] * inv * wi * silu;
        }
        r[e] = pack_bf16x2(y[0], y[1]);
    }
    if (live) *reinterpret_cast<uint4 *>(o + base) = make_uint4(r[0], r[1], r[2], r[3]);
}

cudaError_t launch_output_gate(void *o, const void *z, const void *w, int w_dtype, int64_t vectors, float eps,
                               cudaStream_t stream) {
    if (vectors <= 0) return cudaSuccess;
    const int64_t blocks = (vectors * 16 + 255) / 256;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    output_gate_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<__nv_bfloat16 *>(o), static_cast<const __nv_bfloat16 *>(z), w, w_dtype, vectors, eps);
    return cudaGetLastError();
}

}  // namespace gdn
