// gdn_chunk_prep.cu -- the state-independent half of the chunked prefill, for every
// chunk of every sequence at once: the chunk's gates, T = (I + A)^-1 scaled into the
// bf16 hi/lo operand tiles T' = T diag(beta) and T'' = T diag(beta Gamma), and the
// decayed Q K^T tile P, written to the workspace of gdn_tc_workspace.h that the
// tcgen05 chain kernel (gdn_prefill_tc.cu) streams in.
//
// For a chunk of tokens i, j = 0..63 (solution/gdn_baseline_torch.py:42-44, 71-87):
//   log alpha_i = -exp(A_log) softplus(a_i + dt_bias),  beta_i = sigmoid(b_i)
//   gamma_i = sum_{j<=i} log alpha_j,   Gamma_i = exp(gamma_i)
//   A[i][j] = beta_i exp(gamma_i - gamma_j) k_i.k_j  (j < i),   T = (I + A)^-1
//   P[i][j] = exp(gamma_i - gamma_j) q_i.k_j            (j <= i)
// None of it depends on the recurrent state, so all chunks run in parallel here and
// the chain kernel keeps only the state path on its serial critical path.
//
// The work of one chunk is a chain of short dependent steps, so the kernel is built
// for many chunks in flight per SM: CTAs of 4 warps with ~55 KB of shared memory
// (4 per SM), each handling chunks g, g + G, g + 2G, ... of one sequence and NH v-heads
// that share a q/k head (NH = 2 when the number of v-heads per q/k head is even, else 1):
// K K^T, Q K^T and the K/Q tile loads, which depend only on the q/k head, are done once
// for the NH v-heads.  Warp w owns rows 16w..16w+15 of the chunk:
//   * K K^T and Q K^T on mma.sync (bf16 inputs are exact, fp32 accumulation); K K^T stays
//     in the accumulator registers that computed it and each v-head's A is formed from
//     it in registers, its 16x16 diagonal block also goes to shared memory in fp32; each
//     v-head's P goes from the Q K^T registers to the workspace as bf16;
//   * the four diagonal blocks D_b = (I + A_bb)^-1 by fp32 forward substitution;
//   * then, block-recursively on mma.sync with every fp32 operand split into bf16
//     hi + lo (hi*hi + hi*lo + lo*hi):
//       T_10 = -D_1 A_10 D_0,  T_32 = -D_3 A_32 D_2       (T_a, T_b: the 32x32 halves)
//       T_ba = -T_b A_ba T_a                              (the 32x32 lower-left block)
//     where the A blocks come straight from the registers of warps 1, 3 and 2-3.
#include <cuda_bf16.h>

#include "gdn_chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_launch.h"
#include "gdn_mma_sync.cuh"
#include "gdn_tc_workspace.h"

namespace gdn {
namespace {

using namespace msync;

constexpr int kC = 64;
constexpr int kThreads = 128;

// Shared memory (bytes).  The K tile becomes the fp32 T tile once K K^T and Q K^T are
// done; the Q tile becomes the hi/lo tiles of the intermediate products.
constexpr uint32_t OFF_K = 0;                       // bf16 [64][128], 256-byte swizzled rows
constexpr uint32_t OFF_TF = 0;                      // fp32 T [64][64] row-major (over K)
constexpr uint32_t OFF_Q = 16384;                   // bf16 [64][128], 256-byte swizzled rows
constexpr uint32_t OFF_SH = 16384;                  // bf16 [64][64] intermediate products hi/lo (over Q)
constexpr uint32_t OFF_SL = 24576;
constexpr uint32_t OFF_TH = 32768;                  // bf16 [64][64] T hi/lo, 128-byte swizzled rows
constexpr uint32_t OFF_TL = 40960;
constexpr uint32_t OFF_AD = 49152;                  // fp32 diagonal blocks of A: 4 x [16][17]
constexpr uint32_t OFF_GATE = OFF_AD + 4 * 16 * 17 * 4;   // per v-head: beta, gamma*log2(e), Gamma, decay-to-end
constexpr uint32_t kGateBytes = 4 * 64 * 4;
constexpr uint32_t smem_bytes(int nh) { return OFF_GATE + nh * kGateBytes; }

struct PrepParams {
    const __nv_bfloat16 *q, *k;
    const void *A_log, *a, *dt_bias, *b;
    const int32_t *cu_seqlens;
    int64_t T;
    int Hq, Hv, groups;
    int gate_dtype, param_dtype;
    uint8_t *ws_T;
    float *ws_g;
    __nv_bfloat16 *ws_P;
    int64_t group0;   // (sequence, v-head group) index of blockIdx.x = 0
    int sa, sb;       // elements between consecutive tokens' gate inputs in a, b
};

// [64][128] bf16 rows t0.. of head hh into 256-byte swizzled rows; rows past T read
// as zero (tokens past the sequence end only meet beta = 0 rows and j >= i columns).
__device__ __forceinline__ void load_tile(uint32_t dst, const __nv_bfloat16 *src, int64_t T, int H, int hh,
                                          int64_t t0, int tid) {
#pragma unroll
    for (int u = 0; u < (64 * 16) / kThreads; ++u) {
        const int idx = tid + u * kThreads;
        const int j = idx >> 4, ch = idx & 15;
        const int64_t t = t0 + j;
        const bool ok = t < T;
        cp_async16(dst + j * 256 + ((ch ^ (j & 7)) << 4), src + ((ok ? t : 0) * H + hh) * kHeadDim + ch * 8,
                   ok ? 16 : 0);
    }
}

// acc (16 x 8*NT) += X[16 rows][16 KS] . Y, X as per-k-step hi/lo A fragments in
// registers, Y (k rows, n columns) from bf16 hi/lo tiles [64][64] via ldmatrix.trans;
// hi*hi + hi*lo + lo*hi.
template <int KS, int NT>
__device__ __forceinline__ void prod_rf(float (&acc)[NT][4], const uint32_t (&xh)[KS][4],
                                        const uint32_t (&xl)[KS][4], uint32_t Yh, uint32_t Yl, int yr,
                                        int yc, int lane) {
#pragma unroll
    for (int s = 0; s < KS; ++s)
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t bh[4], bl[4];
            ldsm_x4_t(bh, b_addr_kn<128>(Yh, yc + 16 * np, yr + 16 * s, lane));
            ldsm_x4_t(bl, b_addr_kn<128>(Yl, yc + 16 * np, yr + 16 * s, lane));
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                mma16816(acc[2 * np + u], xh[s], bh[2 * u], bh[2 * u + 1]);
                mma16816(acc[2 * np + u], xh[s], bl[2 * u], bl[2 * u + 1]);
                mma16816(acc[2 * np + u], xl[s], bh[2 * u], bh[2 * u + 1]);
            }
        }
}

// X fragments (rows xr.., k columns xc.. xc + 16 KS) from bf16 hi/lo tiles [64][64].
template <int KS>
__device__ __forceinline__ void load_frags(uint32_t (&xh)[KS][4], uint32_t (&xl)[KS][4], uint32_t Xh,
                                           uint32_t Xl, int xr, int xc, int lane) {
#pragma unroll
    for (int s = 0; s < KS; ++s) {
        ldsm_x4(xh[s], a_addr<128>(Xh, xr, xc + 16 * s, lane));
        ldsm_x4(xl[s], a_addr<128>(Xl, xr, xc + 16 * s, lane));
    }
}

// Store a 16 x 8*NT accumulator block (rows r0.., cols c0..), times `sgn`, as bf16 hi/lo
// into tiles Hh/Hl (when Hh != nullptr) and as fp32 into the row-major [64][64] tile F
// (when F != nullptr).
template <int NT>
__device__ __forceinline__ void store_block(const float (&acc)[NT][4], float sgn, uint8_t *Hh, uint8_t *Hl,
                                            float *F, int r0, int c0, int lane) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int row = r0 + g + 8 * hf, col = c0 + nt * 8 + 2 * t4;
            const float v0 = sgn * acc[nt][2 * hf], v1 = sgn * acc[nt][2 * hf + 1];
            if (Hh) {
                float h0, l0, h1, l1;
                split_bf16(v0, h0, l0);
                split_bf16(v1, h1, l1);
                *reinterpret_cast<uint32_t *>(Hh + swz<128>(row, col)) = pack_bf16x2(h0, h1);
                *reinterpret_cast<uint32_t *>(Hl + swz<128>(row, col)) = pack_bf16x2(l0, l1);
            }
            if (F) *reinterpret_cast<float2 *>(F + row * 64 + col) = make_float2(v0, v1);
        }
}

// kStrided: a and b are read through their row strides (views into a wider projection
// output); the packed instantiation reads them at t * Hv + h, as before.
template <int NH, bool kStrided>
__global__ void __launch_bounds__(kThreads, 4) chunk_prep_kernel(const PrepParams p) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int64_t chain = blockIdx.x + p.group0;       // (sequence, group of NH v-heads)
    const int hgroups = p.Hv / NH;
    const int64_t n = chain / hgroups;
    const int h0 = static_cast<int>(chain % hgroups) * NH;
    const int hq = h0 / (p.Hv / p.Hq);
    int64_t s0 = p.cu_seqlens[n], s1 = p.cu_seqlens[n + 1];
    s0 = s0 < 0 ? 0 : (s0 > p.T ? p.T : s0);
    s1 = s1 < s0 ? s0 : (s1 > p.T ? p.T : s1);
    const int nch = static_cast<int>((s1 - s0 + kC - 1) / kC);
    if (static_cast<int>(blockIdx.y) >= nch) return;

    const uint32_t sbase = smem_addr(sm);
    float *A_d = reinterpret_cast<float *>(sm + OFF_AD);
    float *T_f = reinterpret_cast<float *>(sm + OFF_TF);
    // gate vectors of v-head h0 + hh: beta, gamma*log2(e), Gamma, decay-to-end
    auto gates = [&](int hh) { return reinterpret_cast<float *>(sm + OFF_GATE + hh * kGateBytes); };
    // warp hh < NH computes the gates of v-head h0 + hh
    const int hw = h0 + (warp < NH ? warp : 0);
    const float exp_A = expf(load_scalar(p.A_log, hw, p.param_dtype));
    const float dtb = load_scalar(p.dt_bias, hw, p.param_dtype);
    const uint32_t Th = sbase + OFF_TH, Tl = sbase + OFF_TL, Sh = sbase + OFF_SH, Sl = sbase + OFF_SL;
    const int r0 = 16 * warp;    // this warp's rows of the chunk

    // Warps 0..NH-1 keep the next chunk's gate inputs in registers (loaded a chunk ahead).
    float ga[2] = {0.f, 0.f}, gb[2] = {0.f, 0.f};
    auto fetch_gates = [&](int cc) {
        const int64_t tb = s0 + static_cast<int64_t>(cc) * kC;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int64_t t = tb + lane + 32 * u;
            if (t < s1) {
                ga[u] = load_scalar(p.a, t * (kStrided ? p.sa : p.Hv) + hw, p.gate_dtype);
                gb[u] = load_scalar(p.b, t * (kStrided ? p.sb : p.Hv) + hw, p.gate_dtype);
            }
        }
    };
    if (warp < NH) fetch_gates(blockIdx.y);

    for (int c = blockIdx.y; c < nch; c += p.groups) {
        const int64_t t0 = s0 + static_cast<int64_t>(c) * kC;
        const int nt = static_cast<int>(s1 - t0 < kC ? s1 - t0 : kC);
        load_tile(sbase + OFF_K, p.k, p.T, p.Hq, hq, t0, tid);
        load_tile(sbase + OFF_Q, p.q, p.T, p.Hq, hq, t0, tid);
        cp_async_commit();

        // Gates (warp hh for v-head h0 + hh), then the next chunk's inputs.
        if (warp < NH) {
            float lg[2], bt[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const bool live = lane + 32 * u < nt;
                lg[u] = live ? log_decay(exp_A, ga[u], dtb) : 0.0f;
                bt[u] = live ? sigmoid_f(gb[u]) : 0.0f;
            }
            if (c + p.groups < nch) fetch_gates(c + p.groups);
            float x0 = lg[0], x1 = lg[1];
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float y0 = __shfl_up_sync(0xffffffffu, x0, off);
                const float y1 = __shfl_up_sync(0xffffffffu, x1, off);
                if (lane >= off) { x0 += y0; x1 += y1; }
            }
            x1 += __shfl_sync(0xffffffffu, x0, 31);
            const float xC = __shfl_sync(0xffffffffu, x1, 31);
            constexpr float kLog2e = 1.4426950408889634f;
            float *g_beta = gates(warp), *g_gam2 = g_beta + 64, *g_Gam = g_beta + 128, *g_dec = g_beta + 192;
            g_beta[lane] = bt[0]; g_beta[lane + 32] = bt[1];
            g_gam2[lane] = x0 * kLog2e; g_gam2[lane + 32] = x1 * kLog2e;
            g_Gam[lane] = expf(x0); g_Gam[lane + 32] = expf(x1);
            g_dec[lane] = expf(xC - x0); g_dec[lane + 32] = expf(xC - x1);
        }
        cp_async_wait<0>();
        __syncthreads();

        // K K^T rows r0..r0+15 (columns right of the diagonal block are zero in A and
        // skipped), kept in these registers for the NH v-heads.
        float R[8][4];
        {
#pragma unroll
            for (int i = 0; i < 8; ++i) R[i][0] = R[i][1] = R[i][2] = R[i][3] = 0.0f;
            const uint32_t sK = sbase + OFF_K;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t af[4];
                ldsm_x4(af, a_addr<256>(sK, r0, kk * 16, lane));
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    if (16 * np > r0) continue;
                    uint32_t bf[4];
                    ldsm_x4(bf, b_addr_nk<256>(sK, np * 16, kk * 16, lane));
                    mma16816(R[2 * np], af, bf[0], bf[1]);
                    mma16816(R[2 * np + 1], af, bf[2], bf[3]);
                }
            }
        }
        // Q K^T rows r0.. -> P = exp(gamma_i - gamma_j) q_i.k_j for j <= i of each v-head, to
        // the workspace as bf16 in the swizzled layout the chain kernel's tensor core reads.
        const int64_t unit0 = tc_slot(s0, c, n) * p.Hv + h0;
        {
            float acc[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
            const uint32_t sK = sbase + OFF_K, sQ = sbase + OFF_Q;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t af[4];
                ldsm_x4(af, a_addr<256>(sQ, r0, kk * 16, lane));
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    if (16 * np > r0) continue;
                    uint32_t bf[4];
                    ldsm_x4(bf, b_addr_nk<256>(sK, np * 16, kk * 16, lane));
                    mma16816(acc[2 * np], af, bf[0], bf[1]);
                    mma16816(acc[2 * np + 1], af, bf[2], bf[3]);
                }
            }
#pragma unroll
            for (int hh = 0; hh < NH; ++hh) {
                const float *g_gam2 = gates(hh) + 64;
                uint8_t *dP = reinterpret_cast<uint8_t *>(p.ws_P) + (unit0 + hh) * kTcPBytes;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int i = r0 + g + 8 * hf;
                    const float gi = g_gam2[i];
#pragma unroll
                    for (int ntl = 0; ntl < 8; ++ntl) {
                        const int j = ntl * 8 + 2 * t4;
                        const float p0 = j <= i ? exp2f(gi - g_gam2[j]) * acc[ntl][2 * hf] : 0.0f;
                        const float p1 = j + 1 <= i ? exp2f(gi - g_gam2[j + 1]) * acc[ntl][2 * hf + 1] : 0.0f;
                        *reinterpret_cast<uint32_t *>(dP + swz<128>(i, j)) = pack_bf16x2(p0, p1);
                    }
                }
            }
        }

#pragma unroll 1
        for (int hh = 0; hh < NH; ++hh) {
        const float *g_beta = gates(hh), *g_gam2 = g_beta + 64, *g_Gam = g_beta + 128;
        const int64_t unit = unit0 + hh;
        // A = beta_i exp(gamma_i - gamma_j) k_i.k_j for j < i in registers (in place of
        // K K^T when this is its only v-head); its diagonal block also goes to A_d (fp32).
        float A2[8][4];
        float(&A)[8][4] = NH == 1 ? R : A2;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int i = r0 + g + 8 * hf;
            const float gi = g_gam2[i], bi = g_beta[i];
#pragma unroll
            for (int ntl = 0; ntl < 8; ++ntl) {
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int j = ntl * 8 + 2 * t4 + u;
                    const float a = j < i ? bi * exp2f(gi - g_gam2[j]) * R[ntl][2 * hf + u] : 0.0f;
                    A[ntl][2 * hf + u] = a;
                    if ((j >> 4) == warp) A_d[(16 * warp + (i & 15)) * 17 + (j & 15)] = a;
                }
            }
        }
        __syncthreads();   // A_d complete; the K and Q tiles are dead from here on

        // D_b = (I + A_bb)^-1 (threads 0-63: block ob, column cc, forward substitution with
        // two partial sums per row) -> T hi/lo tiles and T_f; threads 64-127 zero the upper
        // off-diagonal blocks of T_a and T_b in the T hi/lo tiles.
        if (tid < 64) {
            const int ob = tid >> 4, cc = tid & 15, o = ob * 16;
            const float *Ab = A_d + ob * 16 * 17;
            float x[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float a0 = (r == cc) ? 1.0f : 0.0f, a1 = 0.0f;
#pragma unroll
                for (int jj = 0; jj < r; ++jj) {
                    if (jj & 1) a1 = fmaf(-Ab[r * 17 + jj], x[jj], a1);
                    else a0 = fmaf(-Ab[r * 17 + jj], x[jj], a0);
                }
                x[r] = a0 + a1;
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float hi, lo;
                split_bf16(x[r], hi, lo);
                *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_TH + swz<128>(o + r, o + cc)) = __float2bfloat16_rn(hi);
                *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_TL + swz<128>(o + r, o + cc)) = __float2bfloat16_rn(lo);
                T_f[(o + r) * 64 + o + cc] = x[r];
            }
        } else {
            const int e = tid - 64, r = e >> 2, q = e & 3;     // 16 rows x 4 quads of 4 columns
#pragma unroll
            for (int blkz = 0; blkz < 2; ++blkz) {
                const int row = blkz * 32 + r, col = blkz * 32 + 16 + q * 4;
                *reinterpret_cast<uint2 *>(sm + OFF_TH + swz<128>(row, col)) = make_uint2(0u, 0u);
                *reinterpret_cast<uint2 *>(sm + OFF_TL + swz<128>(row, col)) = make_uint2(0u, 0u);
            }
        }
        __syncthreads();

        // M_10 = A_10 D_0 (warp 1), M_32 = A_32 D_2 (warp 3); A blocks from registers.
        if (warp & 1) {
            const int o = warp == 1 ? 0 : 32;       // column block of A_10 / A_32
            uint32_t xh[1][4], xl[1][4];
            if (warp == 1) acc_to_a_split(A[0], A[1], xh[0], xl[0]);   // static indices keep A in registers
            else acc_to_a_split(A[4], A[5], xh[0], xl[0]);
            float acc[2][4] = {};
            prod_rf<1, 2>(acc, xh, xl, Th, Tl, o, o, lane);
            store_block<2>(acc, 1.0f, sm + OFF_SH, sm + OFF_SL, nullptr, r0, o, lane);
        }
        __syncthreads();
        // T_10 = -D_1 M_10 (warp 1), T_32 = -D_3 M_32 (warp 3)
        if (warp & 1) {
            const int o = warp == 1 ? 0 : 32;
            uint32_t xh[1][4], xl[1][4];
            load_frags<1>(xh, xl, Th, Tl, r0, r0, lane);
            float acc[2][4] = {};
            prod_rf<1, 2>(acc, xh, xl, Sh, Sl, r0, o, lane);
            store_block<2>(acc, -1.0f, sm + OFF_TH, sm + OFF_TL, T_f, r0, o, lane);
        }
        __syncthreads();
        // M_ba = A[32..64)[0..32) T_a (warps 2, 3); A from registers.
        if (warp >= 2) {
            uint32_t xh[2][4], xl[2][4];
            acc_to_a_split(A[0], A[1], xh[0], xl[0]);
            acc_to_a_split(A[2], A[3], xh[1], xl[1]);
            float acc[4][4] = {};
            prod_rf<2, 4>(acc, xh, xl, Th, Tl, 0, 0, lane);
            store_block<4>(acc, 1.0f, sm + OFF_SH, sm + OFF_SL, nullptr, r0, 0, lane);
        }
        __syncthreads();
        // T_ba = -T_b M_ba (warps 2, 3)
        if (warp >= 2) {
            uint32_t xh[2][4], xl[2][4];
            load_frags<2>(xh, xl, Th, Tl, r0, 32, lane);
            float acc[4][4] = {};
            prod_rf<2, 4>(acc, xh, xl, Sh, Sl, 32, 0, lane);
            store_block<4>(acc, -1.0f, nullptr, nullptr, T_f, r0, 0, lane);
        }
        __syncthreads();

        // T' = T diag(beta) and T'' = T diag(beta Gamma) (zero above the diagonal) as bf16
        // hi/lo tiles, and the gate vectors, to the workspace.  Thread (i, ch) writes the
        // 16-byte chunk ch of row i of each tile.
        uint8_t *dT = p.ws_T + unit * kTcTBytes;
#pragma unroll
        for (int u = 0; u < (64 * 8) / kThreads; ++u) {
            const int idx = tid + u * kThreads, i = idx >> 3, ch = idx & 7;
            const float4 ta = *reinterpret_cast<const float4 *>(T_f + i * 64 + ch * 8);
            const float4 tb = *reinterpret_cast<const float4 *>(T_f + i * 64 + ch * 8 + 4);
            const float t[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
            uint32_t w1h[4], w1l[4], w2h[4], w2l[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = ch * 8 + 2 * e;
                const float a0 = (j <= i ? t[2 * e] : 0.0f) * g_beta[j];
                const float a1 = (j + 1 <= i ? t[2 * e + 1] : 0.0f) * g_beta[j + 1];
                split2_bf16(a0, a1, w1h[e], w1l[e]);
                split2_bf16(a0 * g_Gam[j], a1 * g_Gam[j + 1], w2h[e], w2l[e]);
            }
            uint8_t *d = dT + swz<128>(i, ch * 8);
            *reinterpret_cast<uint4 *>(d) = make_uint4(w1h[0], w1h[1], w1h[2], w1h[3]);
            *reinterpret_cast<uint4 *>(d + kTcTileBytes) = make_uint4(w1l[0], w1l[1], w1l[2], w1l[3]);
            *reinterpret_cast<uint4 *>(d + 2 * kTcTileBytes) = make_uint4(w2h[0], w2h[1], w2h[2], w2h[3]);
            *reinterpret_cast<uint4 *>(d + 3 * kTcTileBytes) = make_uint4(w2l[0], w2l[1], w2l[2], w2l[3]);
        }
        p.ws_g[unit * (kTcGateBytes / 4) + tid] = g_beta[tid];
        p.ws_g[unit * (kTcGateBytes / 4) + 128 + tid] = g_beta[128 + tid];
        __syncthreads();   // the next v-head, or the next chunk's copies, overwrite T_f and the tiles
        }
    }
}

}  // namespace

// Chunks of an average-length sequence one prep CTA walks at most.  A CTA walks every
// groups-th chunk of its sequence, so in a batch of uneven lengths the CTAs of the long
// sequences run longest; the block scheduler starts them in launch order, and one that
// starts late ends the launch alone.  Bounding the average keeps the long ones short
// (256 log-uniform sequences, 128-32768 tokens, in index order: 32.9 ms with 2 groups,
// 31.7 ms with 6 = 16 chunks per CTA, 31.7 ms with 8 chunks; 16 x 8192 unchanged).
constexpr int64_t kPrepAvgChunksPerCta = 16;

int prep_groups(int64_t chains, int64_t avg_chunks) {
    // Enough CTAs for several waves of 148 SMs x 4 resident CTAs, and CTAs that each
    // walk at most about kPrepAvgChunksPerCta chunks of an average sequence.
    const int64_t want = 8 * 148 * 4;
    int64_t gsz = (want + chains - 1) / chains;
    const int64_t by_len = (avg_chunks + kPrepAvgChunksPerCta - 1) / kPrepAvgChunksPerCta;
    if (by_len > gsz) gsz = by_len;
    return static_cast<int>(gsz < 1 ? 1 : (gsz > 64 ? 64 : gsz));
}

int prep_heads_per_cta(const PrefillArgs &p) {
    // Two v-heads per CTA when the v-heads of every q/k head pair up.
    return ((p.Hv / p.Hq) % 2 == 0) ? 2 : 1;
}

cudaError_t launch_chunk_prep(const PrefillArgs &p, uint8_t *ws_T, __nv_bfloat16 *ws_P, float *ws_g,
                              cudaStream_t stream, int64_t chain_begin, int64_t chain_end) {
    const int nh = prep_heads_per_cta(p);
    if (chain_end < 0) chain_end = p.num_seqs * p.Hv;
    if (chain_begin % nh != 0 || chain_end % nh != 0 || chain_begin > chain_end)
        return cudaErrorInvalidValue;
    const int64_t chains = (chain_end - chain_begin) / nh;
    if (chains == 0) return cudaSuccess;
    if (chains > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const int groups = prep_groups(chains, p.num_seqs > 0 ? (p.total_tokens + 63) / 64 / p.num_seqs : 0);
    const bool strided = (p.a_stride && p.a_stride != p.Hv) || (p.b_stride && p.b_stride != p.Hv);
    auto kernel = strided ? (nh == 2 ? chunk_prep_kernel<2, true> : chunk_prep_kernel<1, true>)
                          : (nh == 2 ? chunk_prep_kernel<2, false> : chunk_prep_kernel<1, false>);
    const uint32_t smem = smem_bytes(nh);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    PrepParams pp{static_cast<const __nv_bfloat16 *>(p.q), static_cast<const __nv_bfloat16 *>(p.k), p.A_log,
                  p.a, p.dt_bias, p.b, p.cu_seqlens, p.total_tokens, p.Hq, p.Hv, groups, p.gate_dtype,
                  p.param_dtype, ws_T, ws_g, ws_P, chain_begin / nh,
                  static_cast<int>(p.a_stride ? p.a_stride : p.Hv), static_cast<int>(p.b_stride ? p.b_stride : p.Hv)};
    kernel<<<dim3(static_cast<unsigned>(chains), groups), kThreads, smem, stream>>>(pp);
    return cudaGetLastError();
}

}  // namespace gdn
