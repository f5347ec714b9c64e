// gdn_output_gate.cu -- the gated RMSNorm that Gated DeltaNet layers apply to the
// recurrence output before the output projection (not part of the reference, whose
// entry points return o itself):
//
//   out = o / sqrt(mean(o^2) + eps) * w * silu(z),   silu(z) = z / (1 + exp(-z)),
//
// per 128-element head vector, in fp32 from the bf16 o and z, rounded to bf16.  It
// reads and writes the output once (in place); 16 lanes own one vector, 8 elements
// (one 16-byte load) each, and reduce the sum of squares with a 16-lane butterfly
// (gated_rmsnorm16, which the tcgen05 prefill's fused output store shares).
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
    float wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = load_scalar(w, l16 * 8 + i, w_dtype);
    const uint4 y = gated_rmsnorm16(ov, zv, wv, eps);
    if (live) *reinterpret_cast<uint4 *>(o + base) = y;
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
