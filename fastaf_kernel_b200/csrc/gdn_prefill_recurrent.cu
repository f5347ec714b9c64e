// gdn_prefill_recurrent.cu -- token-serial Gated DeltaNet prefill on CUDA cores.
//
// The direct form of the recurrence (solution/gdn_baseline_torch.py:71-87), kept
// as the second, independent CUDA implementation of the prefill: it covers any
// sequence layout with plain fp32 FMAs and serves as a cross-check for the
// chunked tensor-core kernel.  It is the algorithm of _gdn_prefill_kernel_v2
// (solution/triton/kernel.py:138-278) written B200-first: the state slab stays
// in registers for the whole sequence, tokens are staged through shared memory
// in blocks of 16 (k/q converted to fp32 once per block, next block prefetched
// into registers while the current one is processed), and the two halves of
// every state row are reduced with one shuffle.
//
// CTA = 128 threads = 64 state rows x 2 column halves of one (sequence, v-head).
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {
namespace {

constexpr int kRecThreads = 128;
constexpr int kRecRows = 64;          // state rows per CTA (2 CTAs per head)
constexpr int kTokBlock = 16;         // tokens staged per shared-memory block
constexpr int kHalfPad = 68;          // floats per half-row of staged k/q (bank offset 4)

struct Prefetch {
    uint4 kq[4];   // 16 tokens x 128 bf16 of k and q = 2 x 4 KiB over 128 threads
    uint4 vv;      // 16 tokens x 64 bf16 of this CTA's v rows = 2 KiB
    float a, b;    // gate inputs of token (threadIdx.x) when threadIdx.x < 16
};

__device__ __forceinline__ void prefetch_block(Prefetch &pf, const __nv_bfloat16 *q,
                                               const __nv_bfloat16 *k, const __nv_bfloat16 *v,
                                               const void *a, const void *b, int gate_dtype,
                                               int64_t t0, int64_t t_end, int Hq, int Hv, int hq,
                                               int h, int row_base, int sa, int sb) {
    const int tid = threadIdx.x;
    // k, q: 16 tokens x 16 uint4 each; thread covers 2 uint4 of k and 2 of q.
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int idx = tid + j * kRecThreads;           // 0..255
        const int tok = idx >> 4, part = idx & 15;
        const int64_t t = t0 + tok;
        if (t < t_end) {
            pf.kq[j] = __ldg(reinterpret_cast<const uint4 *>(k + (t * Hq + hq) * kHeadDim) + part);
            pf.kq[2 + j] = __ldg(reinterpret_cast<const uint4 *>(q + (t * Hq + hq) * kHeadDim) + part);
        } else {
            pf.kq[j] = make_uint4(0, 0, 0, 0);
            pf.kq[2 + j] = make_uint4(0, 0, 0, 0);
        }
    }
    {   // v: 16 tokens x 8 uint4 (64 rows)
        const int tok = tid >> 3, part = tid & 7;
        const int64_t t = t0 + tok;
        pf.vv = t < t_end ? __ldg(reinterpret_cast<const uint4 *>(v + (t * Hv + h) * kHeadDim + row_base) + part)
                          : make_uint4(0, 0, 0, 0);
    }
    if (tid < kTokBlock) {
        const int64_t t = t0 + tid;
        pf.a = t < t_end ? load_scalar(a, t * sa + h, gate_dtype) : 0.0f;
        pf.b = t < t_end ? load_scalar(b, t * sb + h, gate_dtype) : 0.0f;
    }
}

__global__ void __launch_bounds__(kRecThreads)
prefill_recurrent_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                         const __nv_bfloat16 *__restrict__ v, const float *__restrict__ state,
                         const void *A_log, const void *a, const void *dt_bias, const void *b,
                         const int32_t *__restrict__ cu_seqlens, int64_t N, int64_t T, int Hq, int Hv,
                         float scale, int gate_dtype, int param_dtype,
                         __nv_bfloat16 *__restrict__ out, float *__restrict__ new_state, int *status,
                         int sa, int sb) {
    __shared__ __align__(16) float k_s[kTokBlock][2][kHalfPad];
    __shared__ __align__(16) float q_s[kTokBlock][2][kHalfPad];
    __shared__ float v_s[kTokBlock][kRecRows];
    __shared__ float alpha_s[kTokBlock], beta_s[kTokBlock];

    const int slab = blockIdx.x & 1;
    const int64_t sh = blockIdx.x >> 1;                  // (sequence, v-head)
    const int64_t n = sh / Hv;
    const int h = static_cast<int>(sh % Hv);
    const int hq = h / (Hv / Hq);
    const int tid = threadIdx.x;
    const int half = tid & 1;
    const int row_base = slab * kRecRows;
    const int row = row_base + (tid >> 1);

    if (tid == 0 && blockIdx.x % (2 * Hv) == 0) check_seq_bounds(cu_seqlens, n, N, T, status);
    int64_t s0 = cu_seqlens[n], s1 = cu_seqlens[n + 1];
    s0 = s0 < 0 ? 0 : (s0 > T ? T : s0);
    s1 = s1 < s0 ? s0 : (s1 > T ? T : s1);

    float *dst = new_state + (sh * kHeadDim + row) * kHeadDim + half * 64;
    float S[64];
    if (s1 <= s0) {   // empty sequence: zero new state (solution/gdn_baseline_torch.py:61-62)
#pragma unroll
        for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4 *>(dst + i) = make_float4(0, 0, 0, 0);
        return;
    }
    if (state != nullptr) {
        const float *src = state + (sh * kHeadDim + row) * kHeadDim + half * 64;
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(src + i);
            S[i] = x.x; S[i + 1] = x.y; S[i + 2] = x.z; S[i + 3] = x.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) S[i] = 0.0f;
    }
    const float exp_A = expf(load_scalar(A_log, h, param_dtype));
    const float dtb = load_scalar(dt_bias, h, param_dtype);

    Prefetch pf;
    prefetch_block(pf, q, k, v, a, b, gate_dtype, s0, s1, Hq, Hv, hq, h, row_base, sa, sb);
    for (int64_t t0 = s0; t0 < s1; t0 += kTokBlock) {
        __syncthreads();   // the previous block is no longer being read
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int idx = tid + j * kRecThreads;
            const int tok = idx >> 4, part = idx & 15;        // part: 8 bf16 at column 8*part
            const int hh = part >> 3, c = (part & 7) * 8;
            const uint4 kk = pf.kq[j], qq = pf.kq[2 + j];
            float *kd = &k_s[tok][hh][c];
            float *qd = &q_s[tok][hh][c];
            kd[0] = bf16_lo(kk.x); kd[1] = bf16_hi(kk.x); kd[2] = bf16_lo(kk.y); kd[3] = bf16_hi(kk.y);
            kd[4] = bf16_lo(kk.z); kd[5] = bf16_hi(kk.z); kd[6] = bf16_lo(kk.w); kd[7] = bf16_hi(kk.w);
            qd[0] = bf16_lo(qq.x); qd[1] = bf16_hi(qq.x); qd[2] = bf16_lo(qq.y); qd[3] = bf16_hi(qq.y);
            qd[4] = bf16_lo(qq.z); qd[5] = bf16_hi(qq.z); qd[6] = bf16_lo(qq.w); qd[7] = bf16_hi(qq.w);
        }
        {
            const int tok = tid >> 3, c = (tid & 7) * 8;
            const uint4 vv = pf.vv;
            float *vd = &v_s[tok][c];
            vd[0] = bf16_lo(vv.x); vd[1] = bf16_hi(vv.x); vd[2] = bf16_lo(vv.y); vd[3] = bf16_hi(vv.y);
            vd[4] = bf16_lo(vv.z); vd[5] = bf16_hi(vv.z); vd[6] = bf16_lo(vv.w); vd[7] = bf16_hi(vv.w);
        }
        if (tid < kTokBlock) {
            alpha_s[tid] = expf(log_decay(exp_A, pf.a, dtb));
            beta_s[tid] = sigmoid_f(pf.b);
        }
        __syncthreads();
        const int64_t nxt = t0 + kTokBlock;
        if (nxt < s1) prefetch_block(pf, q, k, v, a, b, gate_dtype, nxt, s1, Hq, Hv, hq, h, row_base, sa, sb);

        const int ntok = static_cast<int>(s1 - t0 < kTokBlock ? s1 - t0 : kTokBlock);
        for (int tt = 0; tt < ntok; ++tt) {
            const float g = alpha_s[tt], bt = beta_s[tt];
            const float4 *kr = reinterpret_cast<const float4 *>(&k_s[tt][half][0]);
            const float4 *qr = reinterpret_cast<const float4 *>(&q_s[tt][half][0]);
            float u = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float4 kv = kr[i];
                S[4 * i] *= g; S[4 * i + 1] *= g; S[4 * i + 2] *= g; S[4 * i + 3] *= g;
                u = fmaf(kv.x, S[4 * i], u); u = fmaf(kv.y, S[4 * i + 1], u);
                u = fmaf(kv.z, S[4 * i + 2], u); u = fmaf(kv.w, S[4 * i + 3], u);
            }
            u += __shfl_xor_sync(0xffffffffu, u, 1);
            const float vn = bt * v_s[tt][tid >> 1] + (1.0f - bt) * u;
            float y = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float4 kv = kr[i], qv = qr[i];
                S[4 * i] = (S[4 * i] - kv.x * u) + kv.x * vn;
                S[4 * i + 1] = (S[4 * i + 1] - kv.y * u) + kv.y * vn;
                S[4 * i + 2] = (S[4 * i + 2] - kv.z * u) + kv.z * vn;
                S[4 * i + 3] = (S[4 * i + 3] - kv.w * u) + kv.w * vn;
                y = fmaf(qv.x, S[4 * i], y); y = fmaf(qv.y, S[4 * i + 1], y);
                y = fmaf(qv.z, S[4 * i + 2], y); y = fmaf(qv.w, S[4 * i + 3], y);
            }
            y += __shfl_xor_sync(0xffffffffu, y, 1);
            if (half == 0) out[((t0 + tt) * Hv + h) * kHeadDim + row] = __float2bfloat16_rn(scale * y);
        }
    }
#pragma unroll
    for (int i = 0; i < 64; i += 4)
        *reinterpret_cast<float4 *>(dst + i) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
}

}  // namespace

cudaError_t launch_prefill_recurrent(const PrefillArgs &p, cudaStream_t stream) {
    const int64_t ctas = p.num_seqs * p.Hv * 2;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    prefill_recurrent_kernel<<<static_cast<unsigned>(ctas), kRecThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(p.q), static_cast<const __nv_bfloat16 *>(p.k),
        static_cast<const __nv_bfloat16 *>(p.v), p.state, p.A_log, p.a, p.dt_bias, p.b,
        p.cu_seqlens, p.num_seqs, p.total_tokens, p.Hq, p.Hv, p.scale, p.gate_dtype, p.param_dtype,
        static_cast<__nv_bfloat16 *>(p.out), p.new_state, p.status,
        static_cast<int>(p.a_stride ? p.a_stride : p.Hv), static_cast<int>(p.b_stride ? p.b_stride : p.Hv));
    return cudaGetLastError();
}

}  // namespace gdn
