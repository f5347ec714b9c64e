// gdn_output_gate.cu -- the gated RMSNorm that Gated DeltaNet layers apply to the
// recurrence output before the output projection (not part of the reference, whose
// entry points return o itself):
//
//   out = o / sqrt(mean(o^2) + eps) * w * silu(z),   silu(z) = z / (1 + exp(-z)),
//
// per 128-element head vector, in fp32 from the bf16 o and z (sigmoid from the hardware
// tanh, the hardware reciprocal square root), rounded to bf16.  It reads and writes the
// output once (in place); 16 lanes own one vector, 8 elements (one 16-byte load) each,
// and reduce the sum of squares with a 16-lane butterfly (gated_rmsnorm16, which the
// tcgen05 prefill's fused output store shares, so both give the same bits).
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

// Vectors per 16-lane group: their o and z loads are all issued before any arithmetic,
// so each thread keeps 4 x 16 bytes in flight.  Measured at 16 x 8192 x 32 heads (3.2 GB):
// one vector per group 4.99 TB/s, two 5.32 TB/s, four 4.74 TB/s (the registers of four
// cut the resident warps), four with streaming (.cs) accesses 4.72 TB/s.
constexpr int kGateVecs = 2;

__global__ void __launch_bounds__(256)
output_gate_kernel(__nv_bfloat16 *__restrict__ o, const __nv_bfloat16 *__restrict__ z, const void *w,
                   int w_dtype, int64_t vectors, float eps) {
    const int64_t groups = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 4);
    const int64_t g0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;
    const int l16 = threadIdx.x & 15;
    float wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = load_scalar(w, l16 * 8 + i, w_dtype);
    // group g0 takes vectors g0, g0 + groups, ... (each round over the grid is contiguous);
    // vectors past the end work on vector 0 and store nothing, so every lane takes part
    // in the full-warp shuffles
    int64_t base[kGateVecs];
    bool live[kGateVecs];
    uint4 ov[kGateVecs], zv[kGateVecs];
#pragma unroll
    for (int u = 0; u < kGateVecs; ++u) {
        const int64_t vec = g0 + u * groups;
        live[u] = vec < vectors;
        base[u] = (live[u] ? vec : 0) * kHeadDim + l16 * 8;
        ov[u] = *reinterpret_cast<const uint4 *>(o + base[u]);
        zv[u] = __ldg(reinterpret_cast<const uint4 *>(z + base[u]));
    }
#pragma unroll
    for (int u = 0; u < kGateVecs; ++u) {
        const uint4 y = gated_rmsnorm16(ov[u], zv[u], wv, eps);
        if (live[u]) *reinterpret_cast<uint4 *>(o + base[u]) = y;
    }
}

cudaError_t launch_output_gate(void *o, const void *z, const void *w, int w_dtype, int64_t vectors, float eps,
                               cudaStream_t stream) {
    if (vectors <= 0) return cudaSuccess;
    const int64_t groups = (vectors + kGateVecs - 1) / kGateVecs;
    const int64_t blocks = (groups * 16 + 255) / 256;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    output_gate_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<__nv_bfloat16 *>(o), static_cast<const __nv_bfloat16 *>(z), w, w_dtype, vectors, eps);
    return cudaGetLastError();
}

}  // namespace gdn
