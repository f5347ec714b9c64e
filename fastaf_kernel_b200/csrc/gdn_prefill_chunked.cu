// gdn_prefill_chunked.cu -- chunked (C = 64) Gated DeltaNet prefill on the tensor cores.
//
// Replaces the token-serial _gdn_prefill_kernel_v2 (solution/triton/kernel.py:138-278)
// with the chunked WY/UT form of the same recurrence
// (solution/gdn_baseline_torch.py:71-87).  For one (sequence, v-head) chain and a
// chunk of tokens i, j = 0..63 with state S0 (k-last, [v][k]) at its start:
//
//   gamma_i = sum_{j<=i} log alpha_j,  Gamma_i = exp(gamma_i)
//   A[i][j] = beta_i exp(gamma_i - gamma_j) k_i.k_j  (j < i),   T = (I + A)^-1
//   R       = K S0^T                                   (the state's prediction of v)
//   X       = diag(beta) (V - diag(Gamma) R)
//   delta   = T X                                      (per-token innovations, [i][v])
//             computed block-wise over 16-token blocks b as
//             delta_b = T_bb (X_b - sum_{c<b} A_bc delta_c),  T_bb = (I + A_bb)^-1
//   O       = scale (diag(Gamma) Q S0^T + P delta),    P[i][j] = exp(gamma_i - gamma_j) q_i.k_j (j <= i)
//   S_end   = Gamma_63 S0 + sum_i exp(gamma_63 - gamma_i) delta_i k_i^T
//
// which is exactly S_t = alpha_t S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T
// applied token by token.  Padding tokens of a partial chunk get beta = 0 and
// log alpha = 0 (identity rows of T, zero innovations), so K/Q/V need no masking.
//
// Precision: every product with an fp32 operand (S0, X, T, delta') splits that
// operand into bf16 hi + lo (~16 significant bits), so the fp32 state tracks the
// fp32 recurrence to ~1e-5 relative; q/k/v are exact in bf16.  Only the output
// path (Q S0^T and P delta) uses single bf16, within the bf16 output tolerance.
//
// Layout: one CTA per chain, 8 warps; warp w owns state rows v = 16w..16w+15 and
// keeps them, all 128 k columns, as fp32 mma.sync accumulators in registers for
// the whole sequence.  The products in which v is the row index (R, Q S0^T, the
// blocked delta recursion, O, the state update) run per warp; only the
// chunk-wide pieces (gates, K K^T / Q K^T and the four 16x16 diagonal inverses)
// are shared through swizzled shared memory.  q/k/v tiles are double-buffered
// with cp.async and the gate inputs of the next chunk are prefetched into
// registers, so the only serial work per chunk is one 16-step substitution.
#include <cuda_bf16.h>

#include "gdn_chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_launch.h"
#include "gdn_mma_sync.cuh"

namespace gdn {
namespace {

using namespace msync;

constexpr int kC = 64;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Shared memory map (bytes).
constexpr uint32_t TILE = 64 * 256;                 // one [64][128] bf16 tile
constexpr uint32_t OFF_K = 0;                       // 2 stages
constexpr uint32_t OFF_Q = 2 * TILE;                // 2 stages
constexpr uint32_t OFF_V = 4 * TILE;                // 2 stages
constexpr uint32_t OFF_O = 6 * TILE;                // output staging [i][v]
constexpr uint32_t OFF_P = 7 * TILE;                // [64][64] bf16
constexpr uint32_t OFF_MH = OFF_P + 8192;           // M hi [i][j]: -A off the diagonal blocks, T_bb on them
constexpr uint32_t OFF_ML = OFF_MH + 8192;          // M lo
constexpr uint32_t OFF_AD = OFF_ML + 8192;          // fp32 diagonal blocks of A: 4 x [16][17]
constexpr uint32_t AD_STRIDE = 17;
constexpr uint32_t OFF_GATE = OFF_AD + 4 * 16 * AD_STRIDE * 4;   // beta, gamma, Gamma, decay-to-end
constexpr uint32_t SMEM_BYTES = OFF_GATE + 1024;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

struct ChunkParams {
    const __nv_bfloat16 *q, *k, *v;
    const float *state;
    const void *A_log, *a, *dt_bias, *b;
    const int32_t *cu_seqlens;
    int64_t T;
    int Hq, Hv;
    float scale;
    int gate_dtype, param_dtype;
    __nv_bfloat16 *out;
    float *new_state;
    int64_t num_seqs;
    int *status;     // device status word (malformed cu_seqlens), or nullptr
    int sa, sb;      // elements between consecutive tokens' gate inputs in a, b
};

// Issue the cp.async copies of chunk tokens [t0, t0+64) into stage `st`.
__device__ __forceinline__ void load_chunk(const ChunkParams &p, uint32_t sbase, int st,
                                           int64_t t0, int hq, int h) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int u = 0; u < (64 * 16) / kThreads; ++u) {
        const int idx = tid + u * kThreads;
        const int j = idx >> 4, ch = idx & 15;
        const int64_t t = t0 + j;
        const bool ok = t < p.T;
        const int64_t tt = ok ? t : 0;
        const uint32_t off = j * 256 + (((ch ^ (j & 7))) << 4);
        cp_async16(sbase + OFF_K + st * TILE + off, p.k + (tt * p.Hq + hq) * kHeadDim + ch * 8, ok ? 16 : 0);
        cp_async16(sbase + OFF_Q + st * TILE + off, p.q + (tt * p.Hq + hq) * kHeadDim + ch * 8, ok ? 16 : 0);
        cp_async16(sbase + OFF_V + st * TILE + off, p.v + (tt * p.Hv + h) * kHeadDim + ch * 8, ok ? 16 : 0);
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(kThreads, 1) prefill_chunked_mma_kernel(const ChunkParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;   // mma fragment row group / column pair
    const int64_t chain = blockIdx.x;
    const int64_t n = chain / p.Hv;
    const int h = static_cast<int>(chain % p.Hv);
    const int hq = h / (p.Hv / p.Hq);
    if (tid == 0 && h == 0) check_seq_bounds(p.cu_seqlens, n, p.num_seqs, p.T, p.status);
    int64_t s0 = p.cu_seqlens[n], s1 = p.cu_seqlens[n + 1];
    s0 = s0 < 0 ? 0 : (s0 > p.T ? p.T : s0);
    s1 = s1 < s0 ? s0 : (s1 > p.T ? p.T : s1);
    const int nch = static_cast<int>((s1 - s0 + kC - 1) / kC);
    float *dst_state = p.new_state + chain * kHeadDim * kHeadDim;

    if (nch == 0) {   // empty sequence: zero new state (solution/gdn_baseline_torch.py:61-62)
        for (int i = tid; i < kHeadDim * kHeadDim / 4; i += kThreads)
            reinterpret_cast<float4 *>(dst_state)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }

    const uint32_t sbase = smem_u32(sm);
    float *A_d = reinterpret_cast<float *>(sm + OFF_AD);
    float *g_beta = reinterpret_cast<float *>(sm + OFF_GATE);
    float *g_gam = g_beta + 64, *g_Gam = g_beta + 128, *g_dec = g_beta + 192;

    // State rows v0 = 16*warp + g and v0 + 8, columns 8*nt + 2*t4 (+1): fp32 accumulators.
    const int v0 = warp * 16 + g;
    float S[16][4];
    {
        const float *src = p.state ? p.state + chain * kHeadDim * kHeadDim : nullptr;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
            const int col = nt * 8 + 2 * t4;
            float2 x0 = make_float2(0.f, 0.f), x1 = make_float2(0.f, 0.f);
            if (src) {
                x0 = *reinterpret_cast<const float2 *>(src + v0 * kHeadDim + col);
                x1 = *reinterpret_cast<const float2 *>(src + (v0 + 8) * kHeadDim + col);
            }
            S[nt][0] = x0.x; S[nt][1] = x0.y; S[nt][2] = x1.x; S[nt][3] = x1.y;
        }
    }
    const float exp_A = expf(load_scalar(p.A_log, h, p.param_dtype));
    const float dtb = load_scalar(p.dt_bias, h, p.param_dtype);

    load_chunk(p, sbase, 0, s0, hq, h);
    if (nch > 1) load_chunk(p, sbase, 1, s0 + kC, hq, h);

    // Warp 0 keeps the next chunk's raw gate inputs in registers (loaded one chunk ahead).
    float ga[2] = {0.f, 0.f}, gb[2] = {0.f, 0.f};
    auto fetch_gates = [&](int64_t tbase, int nvalid) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = lane + 32 * u;
            if (i < nvalid) {
                ga[u] = load_scalar(p.a, (tbase + i) * p.sa + h, p.gate_dtype);
                gb[u] = load_scalar(p.b, (tbase + i) * p.sb + h, p.gate_dtype);
            }
        }
    };
    if (warp == 0) fetch_gates(s0, static_cast<int>(s1 - s0 < kC ? s1 - s0 : kC));

    for (int c = 0; c < nch; ++c) {
        const int st = c & 1;
        const int64_t t0 = s0 + static_cast<int64_t>(c) * kC;
        const int nt_valid = static_cast<int>(s1 - t0 < kC ? s1 - t0 : kC);
        const uint32_t sK = sbase + OFF_K + st * TILE;
        const uint32_t sQ = sbase + OFF_Q + st * TILE;
        const uint8_t *pV = sm + OFF_V + st * TILE;

        if (c + 1 < nch) cp_async_wait<1>(); else cp_async_wait<0>();
        // ---- gates (warp 0): beta, inclusive cumsum gamma of log alpha, Gamma, decay to chunk end
        if (warp == 0) {
            float lg[2], bt[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int i = lane + 32 * u;
                lg[u] = 0.0f;
                bt[u] = 0.0f;
                if (i < nt_valid) {
                    lg[u] = log_decay(exp_A, ga[u], dtb);
                    bt[u] = sigmoid_f(gb[u]);
                }
            }
            if (c + 1 < nch) {
                const int64_t tn = t0 + kC;
                fetch_gates(tn, static_cast<int>(s1 - tn < kC ? s1 - tn : kC));
            }
            float x0 = lg[0], x1 = lg[1];
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float y0 = __shfl_up_sync(0xffffffffu, x0, off);
                const float y1 = __shfl_up_sync(0xffffffffu, x1, off);
                if (lane >= off) { x0 += y0; x1 += y1; }
            }
            x1 += __shfl_sync(0xffffffffu, x0, 31);
            const float gend = __shfl_sync(0xffffffffu, x1, 31);
            g_beta[lane] = bt[0]; g_beta[lane + 32] = bt[1];
            g_gam[lane] = x0; g_gam[lane + 32] = x1;
            g_Gam[lane] = expf(x0); g_Gam[lane + 32] = expf(x1);
            g_dec[lane] = expf(gend - x0); g_dec[lane + 32] = expf(gend - x1);
        }
        __syncthreads();

        // ---- K K^T (warps 0-3) and Q K^T (warps 4-7): rows 16*(warp&3).., all 64 columns
        {
            const int r0 = (warp & 3) * 16;
            const uint32_t sA = warp < 4 ? sK : sQ;
            float acc[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t af[4];
                ldsm_x4(af, a_addr<256>(sA, r0, kk * 16, lane));
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t bf[4];
                    ldsm_x4(bf, b_addr_nk<256>(sK, np * 16, kk * 16, lane));
                    mma16816(acc[2 * np], af, bf[0], bf[1]);
                    mma16816(acc[2 * np + 1], af, bf[2], bf[3]);
                }
            }
            // Epilogue.  Warps 0-3 (K K^T, row block w): the diagonal block of A in fp32
            // for the 16x16 inverse, -A as bf16 hi/lo on the blocks left of it, zeros
            // to its right.  Warps 4-7 (Q K^T): P in bf16.
            const int blk = warp & 3;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int j0 = nt * 8 + 2 * t4;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int i = r0 + g + half * 8;
                    const float gi = g_gam[i];
                    float vals[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int j = j0 + u;
                        const float dec = j <= i ? expf(gi - g_gam[j]) : 0.0f;
                        vals[u] = dec * acc[nt][2 * half + u];
                    }
                    if (warp < 4) {
                        const int jb = nt >> 1;   // column block of j0, j0+1
                        if (jb == blk) {
#pragma unroll
                            for (int u = 0; u < 2; ++u) {
                                const int j = j0 + u;
                                A_d[(blk * 16 + (i & 15)) * AD_STRIDE + (j & 15)] =
                                    j < i ? g_beta[i] * vals[u] : 0.0f;
                            }
                        } else {
                            float h0 = 0.f, l0 = 0.f, h1 = 0.f, l1 = 0.f;
                            if (jb < blk) {
                                split_bf16(-g_beta[i] * vals[0], h0, l0);
                                split_bf16(-g_beta[i] * vals[1], h1, l1);
                            }
                            *reinterpret_cast<uint32_t *>(sm + OFF_MH + swz<128>(i, j0)) = pack_bf16x2(h0, h1);
                            *reinterpret_cast<uint32_t *>(sm + OFF_ML + swz<128>(i, j0)) = pack_bf16x2(l0, l1);
                        }
                    } else {
                        *reinterpret_cast<uint32_t *>(sm + OFF_P + swz<128>(i, j0)) = pack_bf16x2(vals[0], vals[1]);
                    }
                }
            }
        }
        __syncthreads();

        // ---- T_bb = (I + A_bb)^-1 for the four 16x16 diagonal blocks (threads 0-63,
        //      one column each, forward substitution in fp32) -> bf16 hi/lo into M
        if (tid < 64) {
            const int b = tid >> 4, col = tid & 15;
            const float *Ab = A_d + b * 16 * AD_STRIDE;
            float x[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float acc = (r == col) ? 1.0f : 0.0f;
#pragma unroll
                for (int j = 0; j < r; ++j) acc = fmaf(-Ab[r * AD_STRIDE + j], x[j], acc);
                x[r] = acc;
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float hx, lx;
                split_bf16(x[r], hx, lx);
                const uint32_t off = swz<128>(b * 16 + r, b * 16 + col);
                *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_MH + off) = __float2bfloat16_rn(hx);
                *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_ML + off) = __float2bfloat16_rn(lx);
            }
        }

        // ---- per warp: R^T = S K^T (split S), Y^T = S_hi Q^T   (rows v, columns tokens)
        float R[8][4], Y[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) R[i][e] = Y[i][e] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            uint32_t shi[4], slo[4];
            acc_to_a_split(S[2 * kk], S[2 * kk + 1], shi, slo);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t bk[4], bq[4];
                ldsm_x4(bk, b_addr_nk<256>(sK, np * 16, kk * 16, lane));
                ldsm_x4(bq, b_addr_nk<256>(sQ, np * 16, kk * 16, lane));
                mma16816(R[2 * np], shi, bk[0], bk[1]);
                mma16816(R[2 * np + 1], shi, bk[2], bk[3]);
                mma16816(R[2 * np], slo, bk[0], bk[1]);
                mma16816(R[2 * np + 1], slo, bk[2], bk[3]);
                mma16816(Y[2 * np], shi, bq[0], bq[1]);
                mma16816(Y[2 * np + 1], shi, bq[2], bq[3]);
            }
        }

        // ---- X = beta (V - Gamma R), in place in R
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = nt * 8 + 2 * t4 + (e & 1);
                const int v = v0 + ((e >> 1) << 3);
                const float vv = __bfloat162float(
                    *reinterpret_cast<const __nv_bfloat16 *>(pV + swz<256>(j, v)));
                R[nt][e] = g_beta[j] * (vv - g_Gam[j] * R[nt][e]);
            }

        __syncthreads();   // M (diagonal inverses) and P are complete

        // ---- delta^T block by block: delta_b^T = (X_b^T - sum_{c<b} delta_c^T A_bc^T) T_bb^T
        float D[8][4];
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            float Z[2][4];
#pragma unroll
            for (int e = 0; e < 4; ++e) { Z[0][e] = R[2 * bb][e]; Z[1][e] = R[2 * bb + 1][e]; }
#pragma unroll
            for (int cc = 0; cc < bb; ++cc) {
                uint32_t dhi[4], dlo[4], mh[4], ml[4];
                acc_to_a_split(D[2 * cc], D[2 * cc + 1], dhi, dlo);
                ldsm_x4(mh, b_addr_nk<128>(sbase + OFF_MH, bb * 16, cc * 16, lane));
                ldsm_x4(ml, b_addr_nk<128>(sbase + OFF_ML, bb * 16, cc * 16, lane));
                mma16816(Z[0], dhi, mh[0], mh[1]);
                mma16816(Z[1], dhi, mh[2], mh[3]);
                mma16816(Z[0], dlo, mh[0], mh[1]);
                mma16816(Z[1], dlo, mh[2], mh[3]);
                mma16816(Z[0], dhi, ml[0], ml[1]);
                mma16816(Z[1], dhi, ml[2], ml[3]);
            }
            uint32_t zhi[4], zlo[4], th[4], tl[4];
            acc_to_a_split(Z[0], Z[1], zhi, zlo);
            ldsm_x4(th, b_addr_nk<128>(sbase + OFF_MH, bb * 16, bb * 16, lane));
            ldsm_x4(tl, b_addr_nk<128>(sbase + OFF_ML, bb * 16, bb * 16, lane));
#pragma unroll
            for (int e = 0; e < 4; ++e) D[2 * bb][e] = D[2 * bb + 1][e] = 0.0f;
            mma16816(D[2 * bb], zhi, th[0], th[1]);
            mma16816(D[2 * bb + 1], zhi, th[2], th[3]);
            mma16816(D[2 * bb], zlo, th[0], th[1]);
            mma16816(D[2 * bb + 1], zlo, th[2], th[3]);
            mma16816(D[2 * bb], zhi, tl[0], tl[1]);
            mma16816(D[2 * bb + 1], zhi, tl[2], tl[3]);
        }

        // ---- O^T = Gamma Y^T + delta^T P^T  (delta in bf16: output path)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) Y[nt][e] *= g_Gam[nt * 8 + 2 * t4 + (e & 1)];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t da[4];
            acc_to_a_bf16(D[2 * kk], D[2 * kk + 1], da);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t pb[4];
                ldsm_x4(pb, b_addr_nk<128>(sbase + OFF_P, np * 16, kk * 16, lane));
                mma16816(Y[2 * np], da, pb[0], pb[1]);
                mma16816(Y[2 * np + 1], da, pb[2], pb[3]);
            }
        }
        // stage O as [token i][v] bf16 for coalesced row stores
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = nt * 8 + 2 * t4 + (e & 1);
                const int v = v0 + ((e >> 1) << 3);
                *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_O + swz<256>(i, v)) =
                    __float2bfloat16_rn(p.scale * Y[nt][e]);
            }

        // ---- S = Gamma_63 S + (exp(gamma_63 - gamma_i) delta_i)^T K  (split delta')
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) D[i][e] *= g_dec[i * 8 + 2 * t4 + (e & 1)];
        {
            const float GamC = g_Gam[63];
#pragma unroll
            for (int i = 0; i < 16; ++i)
#pragma unroll
                for (int e = 0; e < 4; ++e) S[i][e] *= GamC;
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t dhi[4], dlo[4];
            acc_to_a_split(D[2 * kk], D[2 * kk + 1], dhi, dlo);
#pragma unroll
            for (int np = 0; np < 8; ++np) {
                uint32_t bk[4];
                ldsm_x4_t(bk, b_addr_kn<256>(sK, np * 16, kk * 16, lane));
                mma16816(S[2 * np], dhi, bk[0], bk[1]);
                mma16816(S[2 * np + 1], dhi, bk[2], bk[3]);
                mma16816(S[2 * np], dlo, bk[0], bk[1]);
                mma16816(S[2 * np + 1], dlo, bk[2], bk[3]);
            }
        }
        __syncthreads();   // all warps done with stage st and the staged output

        // ---- store the chunk's output rows; refill stage st with chunk c+2
        for (int idx = tid; idx < 64 * 16; idx += kThreads) {
            const int i = idx >> 4, ch = idx & 15;
            if (i < nt_valid) {
                const uint4 x = *reinterpret_cast<const uint4 *>(sm + OFF_O + i * 256 + ((ch ^ (i & 7)) << 4));
                *reinterpret_cast<uint4 *>(p.out + ((t0 + i) * p.Hv + h) * kHeadDim + ch * 8) = x;
            }
        }
        if (c + 2 < nch) load_chunk(p, sbase, st, t0 + 2 * kC, hq, h);
    }

    // Final state.
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
        const int col = nt * 8 + 2 * t4;
        *reinterpret_cast<float2 *>(dst_state + v0 * kHeadDim + col) = make_float2(S[nt][0], S[nt][1]);
        *reinterpret_cast<float2 *>(dst_state + (v0 + 8) * kHeadDim + col) = make_float2(S[nt][2], S[nt][3]);
    }
}

int g_sm100_device = -2;

bool device_is_sm100() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (g_sm100_device == dev) return true;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major == 10 && minor == 0) {
        g_sm100_device = dev;
        return true;
    }
    return false;
}

}  // namespace

bool prefill_chunked_supported(const PrefillArgs &p) {
    return p.total_tokens > 0 && device_is_sm100();
}

cudaError_t launch_prefill_chunked(const PrefillArgs &p, cudaStream_t stream) {
    const int64_t ctas = p.num_seqs * p.Hv;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(prefill_chunked_mma_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    ChunkParams cp{static_cast<const __nv_bfloat16 *>(p.q), static_cast<const __nv_bfloat16 *>(p.k),
                   static_cast<const __nv_bfloat16 *>(p.v), p.state, p.A_log, p.a, p.dt_bias, p.b,
                   p.cu_seqlens, p.total_tokens, p.Hq, p.Hv, p.scale, p.gate_dtype, p.param_dtype,
                   static_cast<__nv_bfloat16 *>(p.out), p.new_state, p.num_seqs, p.status,
                   static_cast<int>(p.a_stride ? p.a_stride : p.Hv), static_cast<int>(p.b_stride ? p.b_stride : p.Hv)};
    prefill_chunked_mma_kernel<<<static_cast<unsigned>(ctas), kThreads, SMEM_BYTES, stream>>>(cp);
    return cudaGetLastError();
}

}  // namespace gdn
