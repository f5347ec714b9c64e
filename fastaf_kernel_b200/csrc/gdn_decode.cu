// gdn_decode.cu -- single-token Gated DeltaNet decode, one state read + one state write.
//
// Replaces _gdn_decode_kernel_v3 (solution/triton/kernel.py:285-409), which reads
// every state tile twice (pass 1 at :366-375 for S k, pass 2 at :386-404 for the
// update).  Here each state row is streamed from HBM once with 128-bit loads,
// both dot products it needs are reduced with warp shuffles while the row sits
// in registers, and the updated row is streamed back:
//
//   S'   = alpha * S                      (solution/gdn_baseline_torch.py:79)
//   u    = k . S'[v, :]                   (:80)
//   vn   = beta * v + (1 - beta) * u      (:81)
//   S[v, :] = (S' - k u) + k vn           (:82-84)
//   o[v] = scale * q . S[v, :]            (:86-87)
//
// Optionally (qk_l2norm) q and k are first L2-normalised per head, the usual step
// before the recurrence in Gated DeltaNet layers (the reference never normalises and
// its benchmark inputs arrive normalised): x <- bf16(x / sqrt(sum x^2 + 1e-6)), in
// fp32 from the bf16 inputs, rounded back to bf16 as an upstream normalisation layer
// would emit it.
//
// The step is HBM-bound (128 KiB of state traffic per (sequence, v-head)
// against ~0.8 KiB of q/k/v/o), so the design goal is a copy-like access pattern: every 8 consecutive
// lanes own one 512-byte state row, lane j holding the four float4 at columns
// 4j + 32m (m = 0..3), so each warp-wide load covers four full 128-byte lines.
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

// L2-normalise a 128-element vector held by an aligned group of 8 lanes, 16 values per
// lane: sum of squares per lane in index order, then a butterfly over the 8 lanes.
__device__ __forceinline__ void l2norm_8lanes(float (&x)[16]) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) ss = fmaf(x[i], x[i], ss);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = __bfloat162float(__float2bfloat16_rn(x[i] * inv));
}

constexpr int kDecodeThreads = 256;            // 32 rows per pass (8 lanes per row)
constexpr int kRowsPerPass = kDecodeThreads / 8;

// Three CTAs (24 warps) per SM keep enough loads in flight to stream the state at the
// HBM rate: the two-rows-per-thread instance must fit 85 registers (at 86 it drops to
// two CTAs per SM and the B = 512 step is 16 % slower).
template <int ROWS_PER_THREAD, bool QK_L2NORM>
__global__ void __launch_bounds__(kDecodeThreads, 3)
decode_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
              const __nv_bfloat16 *__restrict__ v, const float *state, const void *A_log,
              const void *a, const void *dt_bias, const void *b, int Hq, int Hv, float scale,
              int gate_dtype, int param_dtype, __nv_bfloat16 *__restrict__ out,
              float *new_state, int sa, int sb) {
    constexpr int kRowsPerCta = kRowsPerPass * ROWS_PER_THREAD;
    constexpr int kCtasPerHead = kHeadDim / kRowsPerCta;
    const int64_t bh = blockIdx.x / kCtasPerHead;          // (sequence, v-head) index
    const int row_block = blockIdx.x % kCtasPerHead;
    const int64_t bidx = bh / Hv;
    const int h = static_cast<int>(bh % Hv);
    const int hq = h / (Hv / Hq);                           // GVA: solution/triton/kernel.py:331
    const int lane8 = threadIdx.x & 7;
    const int row0 = row_block * kRowsPerCta + (threadIdx.x >> 3);

    const float exp_A = expf(load_scalar(A_log, h, param_dtype));
    const float alpha = expf(log_decay(exp_A, load_scalar(a, bidx * sa + h, gate_dtype),
                                       load_scalar(dt_bias, h, param_dtype)));
    const float beta = sigmoid_f(load_scalar(b, bidx * sb + h, gate_dtype));

    // This lane's 16 columns of k and q.
    float kf[16], qf[16];
    {
        const uint2 *kp = reinterpret_cast<const uint2 *>(k + (bidx * Hq + hq) * kHeadDim);
        const uint2 *qp = reinterpret_cast<const uint2 *>(q + (bidx * Hq + hq) * kHeadDim);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const uint2 kk = __ldg(kp + lane8 + 8 * m);
            const uint2 qq = __ldg(qp + lane8 + 8 * m);
            kf[4 * m + 0] = bf16_lo(kk.x); kf[4 * m + 1] = bf16_hi(kk.x);
            kf[4 * m + 2] = bf16_lo(kk.y); kf[4 * m + 3] = bf16_hi(kk.y);
            qf[4 * m + 0] = bf16_lo(qq.x); qf[4 * m + 1] = bf16_hi(qq.x);
            qf[4 * m + 2] = bf16_lo(qq.y); qf[4 * m + 3] = bf16_hi(qq.y);
        }
        if (QK_L2NORM) {
            l2norm_8lanes(kf);
            l2norm_8lanes(qf);
        }
    }

    const int64_t head_base = bh * kHeadDim * kHeadDim;
    float s[ROWS_PER_THREAD][16];
    // Issue every state load of this thread before any arithmetic.
#pragma unroll
    for (int r = 0; r < ROWS_PER_THREAD; ++r) {
        const int row = row0 + r * kRowsPerPass;
        if (state != nullptr) {
            const float4 *sp = reinterpret_cast<const float4 *>(state + head_base + row * kHeadDim);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float4 x = ld_stream(sp + lane8 + 8 * m);
                s[r][4 * m + 0] = x.x; s[r][4 * m + 1] = x.y;
                s[r][4 * m + 2] = x.z; s[r][4 * m + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) s[r][i] = 0.0f;
        }
    }

#pragma unroll
    for (int r = 0; r < ROWS_PER_THREAD; ++r) {
        const int row = row0 + r * kRowsPerPass;
        const float v_row = __bfloat162float(v[(bidx * Hv + h) * kHeadDim + row]);
        float u = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            s[r][i] *= alpha;
            u = fmaf(kf[i], s[r][i], u);
        }
        u += __shfl_xor_sync(0xffffffffu, u, 1);
        u += __shfl_xor_sync(0xffffffffu, u, 2);
        u += __shfl_xor_sync(0xffffffffu, u, 4);
        const float vn = beta * v_row + (1.0f - beta) * u;
        float y = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            s[r][i] = (s[r][i] - kf[i] * u) + kf[i] * vn;
            y = fmaf(qf[i], s[r][i], y);
        }
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        y += __shfl_xor_sync(0xffffffffu, y, 4);
        float4 *dp = reinterpret_cast<float4 *>(new_state + head_base + row * kHeadDim);
#pragma unroll
        for (int m = 0; m < 4; ++m)
            st_stream(dp + lane8 + 8 * m,
                      make_float4(s[r][4 * m], s[r][4 * m + 1], s[r][4 * m + 2], s[r][4 * m + 3]));
        if (lane8 == 0) out[bh * kHeadDim + row] = __float2bfloat16_rn(scale * y);
    }
}

cudaError_t launch_decode(const DecodeArgs &p, cudaStream_t stream) {
    const int64_t heads = p.batch * p.Hv;
    if (heads == 0) return cudaSuccess;
    // Fewer rows per CTA when there are few (sequence, head) pairs, so small
    // batches still spread over all 148 SMs.
    const int rows_per_thread = heads >= 2048 ? 2 : 1;
    const int64_t ctas = heads * (kHeadDim / (kRowsPerPass * rows_per_thread));
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const dim3 grid(static_cast<unsigned>(ctas));
    const auto *q = static_cast<const __nv_bfloat16 *>(p.q);
    const auto *k = static_cast<const __nv_bfloat16 *>(p.k);
    const auto *v = static_cast<const __nv_bfloat16 *>(p.v);
    auto *o = static_cast<__nv_bfloat16 *>(p.out);
    auto kernel = rows_per_thread == 2 ? (p.qk_l2norm ? decode_kernel<2, true> : decode_kernel<2, false>)
                                       : (p.qk_l2norm ? decode_kernel<1, true> : decode_kernel<1, false>);
    kernel<<<grid, kDecodeThreads, 0, stream>>>(q, k, v, p.state, p.A_log, p.a, p.dt_bias, p.b, p.Hq, p.Hv,
                                                p.scale, p.gate_dtype, p.param_dtype, o, p.new_state,
                                                static_cast<int>(p.a_stride ? p.a_stride : p.Hv),
                                                static_cast<int>(p.b_stride ? p.b_stride : p.Hv));
    return cudaGetLastError();
}

// One 8-lane group per 128-element vector (4 per warp), the layout of the decode
// kernel, so both produce the same bits.
__global__ void __launch_bounds__(256) qk_l2norm_kernel(const __nv_bfloat16 *__restrict__ q,
                                                        const __nv_bfloat16 *__restrict__ k, int64_t rows,
                                                        __nv_bfloat16 *__restrict__ qn,
                                                        __nv_bfloat16 *__restrict__ kn) {
    const int64_t vec = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
    const int lane8 = threadIdx.x & 7;
    const bool is_k = vec >= rows;
    const int64_t r0 = is_k ? vec - rows : vec;
    // Groups past the end compute on row 0 and store nothing: every lane stays for the
    // full-warp shuffles.
    const bool live = r0 < rows;
    const int64_t r = live ? r0 : 0;
    const __nv_bfloat16 *src = (is_k ? k : q) + r * kHeadDim;
    __nv_bfloat16 *dst = (is_k ? kn : qn) + r * kHeadDim;
    float x[16];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const uint2 w = __ldg(reinterpret_cast<const uint2 *>(src) + lane8 + 8 * m);
        x[4 * m + 0] = bf16_lo(w.x); x[4 * m + 1] = bf16_hi(w.x);
        x[4 * m + 2] = bf16_lo(w.y); x[4 * m + 3] = bf16_hi(w.y);
    }
    l2norm_8lanes(x);
    if (!live) return;
#pragma unroll
    for (int m = 0; m < 4; ++m)
        reinterpret_cast<uint2 *>(dst)[lane8 + 8 * m] =
            make_uint2(pack_bf16x2(x[4 * m], x[4 * m + 1]), pack_bf16x2(x[4 * m + 2], x[4 * m + 3]));
}

cudaError_t launch_qk_l2norm(const void *q, const void *k, int64_t rows, void *qn, void *kn,
                             cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int64_t threads = 2 * rows * 8;
    const int64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    qk_l2norm_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(q), static_cast<const __nv_bfloat16 *>(k), rows,
        static_cast<__nv_bfloat16 *>(qn), static_cast<__nv_bfloat16 *>(kn));
    return cudaGetLastError();
}

}  // namespace gdn
