// gdn_chunk_prep.cu -- the state-independent half of the chunked prefill, for every
// chunk of every sequence at once: the chunk's gates and T = (I + A)^-1, written to
// the workspace of gdn_tc_workspace.h that the tcgen05 chain kernel
// (gdn_prefill_tc.cu) streams in, together with the chunk's decayed Q K^T tile P.
//
// For a chunk of tokens i, j = 0..63 (solution/gdn_baseline_torch.py:42-44, 71-87):
//   log alpha_i = -exp(A_log) softplus(a_i + dt_bias),  beta_i = sigmoid(b_i)
//   gamma_i = sum_{j<=i} log alpha_j,   Gamma_i = exp(gamma_i)
//   A[i][j] = beta_i exp(gamma_i - gamma_j) k_i.k_j  (j < i),   T = (I + A)^-1
//   P[i][j] = exp(gamma_i - gamma_j) q_i.k_j            (j <= i)
// None of it depends on the recurrent state, so all chunks run in parallel here and
// the chain kernel keeps only the state path on its serial critical path.
//
// One CTA per (sequence, v-head, chunk group): the CTA handles chunks g, g + G,
// g + 2G, ... of its chain, the next chunk's K tile loading while the current one
// is processed.  K K^T runs on mma.sync (bf16 inputs are exact, fp32 accumulation).
// T is built block-recursively on mma.sync: the four 16x16 diagonal blocks
// D_b = (I + A_bb)^-1 by fp32 forward substitution, then
//   T_10 = -D_1 A_10 D_0,   T_32 = -D_3 A_32 D_2          (T_a, T_b: the 32x32 halves)
//   T_ba = -T_b A_ba T_a                                    (the 32x32 lower-left block)
// with every fp32 operand split into bf16 hi + lo (hi*hi + hi*lo + lo*hi).
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
constexpr int kThreads = 256;
constexpr int kLD = 65;                                // fp32 tile row stride (floats)

constexpr uint32_t OFF_K = 0;                          // 2 x bf16 [64][128], 256-byte swizzled rows
constexpr uint32_t OFF_AH = 2 * 64 * 256;              // bf16 [64][64] A hi/lo (128-byte swizzled rows)
constexpr uint32_t OFF_AL = OFF_AH + 8192;
constexpr uint32_t OFF_TH = OFF_AL + 8192;             // bf16 [64][64] T hi/lo
constexpr uint32_t OFF_TL = OFF_TH + 8192;
constexpr uint32_t OFF_SH = OFF_TL + 8192;             // bf16 [64][64] intermediate products hi/lo;
constexpr uint32_t OFF_SL = OFF_SH + 8192;             // before them, the Q tile [64][128] (16 KB)
constexpr uint32_t OFF_AD = OFF_SL + 8192;             // fp32 diagonal blocks of A: 4 x [16][17]
constexpr uint32_t OFF_T = OFF_AD + 4 * 16 * 17 * 4;   // fp32 T [64][65]
constexpr uint32_t OFF_GATE = OFF_T + 64 * kLD * 4;    // beta, gamma*log2(e), Gamma, decay-to-end
constexpr uint32_t SMEM_BYTES = OFF_GATE + 4 * 64 * 4;

// acc (16 x 16 as two m16n8 tiles) += X[xr.., xc..xc+16ks) * Y[yr..yr+16ks, yc..yc+16) with
// X and Y bf16 hi/lo tiles [64][64]; hi*hi + hi*lo + lo*hi carries ~fp32 accuracy.
__device__ __forceinline__ void prod16(float (&acc)[2][4], uint32_t Xh, uint32_t Xl, uint32_t Yh,
                                       uint32_t Yl, int xr, int xc, int yr, int yc, int ks, int lane) {
    for (int s = 0; s < ks; ++s) {
        uint32_t ah[4], al[4], bh[4], bl[4];
        ldsm_x4(ah, a_addr<128>(Xh, xr, xc + 16 * s, lane));
        ldsm_x4(al, a_addr<128>(Xl, xr, xc + 16 * s, lane));
        ldsm_x4_t(bh, b_addr_kn<128>(Yh, yc, yr + 16 * s, lane));
        ldsm_x4_t(bl, b_addr_kn<128>(Yl, yc, yr + 16 * s, lane));
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            mma16816(acc[nt], ah, bh[2 * nt], bh[2 * nt + 1]);
            mma16816(acc[nt], ah, bl[2 * nt], bl[2 * nt + 1]);
            mma16816(acc[nt], al, bh[2 * nt], bh[2 * nt + 1]);
        }
    }
}

// Store a 16x16 accumulator block (rows r0.., cols c0..), times `sgn`, as bf16 hi/lo
// into tiles Hh/Hl and, when F != nullptr, as fp32 into F (row stride kLD).
__device__ __forceinline__ void store16(const float (&acc)[2][4], float sgn, uint8_t *Hh, uint8_t *Hl,
                                        float *F, int r0, int c0, int lane) {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int row = r0 + g + 8 * hf, col = c0 + nt * 8 + 2 * t4;
            const float v0 = sgn * acc[nt][2 * hf], v1 = sgn * acc[nt][2 * hf + 1];
            float h0, l0, h1, l1;
            split_bf16(v0, h0, l0);
            split_bf16(v1, h1, l1);
            *reinterpret_cast<uint32_t *>(Hh + swz<128>(row, col)) = pack_bf16x2(h0, h1);
            *reinterpret_cast<uint32_t *>(Hl + swz<128>(row, col)) = pack_bf16x2(l0, l1);
            if (F) {
                F[row * kLD + col] = v0;
                F[row * kLD + col + 1] = v1;
            }
        }
}

// A [64][128] bf16 tile (rows t0.., head hq) into 256-byte swizzled rows; rows past T
// read as zero.  One cp.async group.
__device__ __forceinline__ void load_k_tile(uint32_t sK, const __nv_bfloat16 *k, int64_t T, int Hq, int hq,
                                            int64_t t0, int tid) {
#pragma unroll
    for (int u = 0; u < (64 * 16) / 256; ++u) {
        const int idx = tid + u * 256;
        const int j = idx >> 4, ch = idx & 15;
        const int64_t t = t0 + j;
        const bool ok = t < T;
        cp_async16(sK + j * 256 + ((ch ^ (j & 7)) << 4), k + ((ok ? t : 0) * Hq + hq) * kHeadDim + ch * 8,
                   ok ? 16 : 0);
    }
    cp_async_commit();
}

struct PrepParams {
    const __nv_bfloat16 *q, *k;
    const void *A_log, *a, *dt_bias, *b;
    const int32_t *cu_seqlens;
    int64_t T;
    int Hq, Hv, groups;
    int gate_dtype, param_dtype;
    float *ws_T, *ws_g;
    __nv_bfloat16 *ws_P;
};

__global__ void __launch_bounds__(kThreads, 2) chunk_prep_kernel(const PrepParams p) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int64_t chain = blockIdx.x;
    const int64_t n = chain / p.Hv;
    const int h = static_cast<int>(chain % p.Hv);
    const int hq = h / (p.Hv / p.Hq);
    int64_t s0 = p.cu_seqlens[n], s1 = p.cu_seqlens[n + 1];
    s0 = s0 < 0 ? 0 : (s0 > p.T ? p.T : s0);
    s1 = s1 < s0 ? s0 : (s1 > p.T ? p.T : s1);
    const int nch = static_cast<int>((s1 - s0 + kC - 1) / kC);

    const uint32_t sbase = smem_addr(sm);
    float *A_d = reinterpret_cast<float *>(sm + OFF_AD);
    float *T_f = reinterpret_cast<float *>(sm + OFF_T);
    float *g_beta = reinterpret_cast<float *>(sm + OFF_GATE);
    float *g_gam2 = g_beta + 64, *g_Gam = g_beta + 128, *g_dec = g_beta + 192;
    const float exp_A = expf(load_scalar(p.A_log, h, p.param_dtype));
    const float dtb = load_scalar(p.dt_bias, h, p.param_dtype);

    // Tokens past T read as zero; tokens past the sequence end only meet beta = 0
    // rows and j >= i columns of A.
    int c = blockIdx.y;
    if (c < nch) load_k_tile(sbase + OFF_K, p.k, p.T, p.Hq, hq, s0 + static_cast<int64_t>(c) * kC, tid);
    for (int it = 0; c < nch; c += p.groups, ++it) {
        const int64_t t0 = s0 + static_cast<int64_t>(c) * kC;
        const int nt = static_cast<int>(s1 - t0 < kC ? s1 - t0 : kC);
        const uint32_t sK = sbase + OFF_K + (it & 1) * (64 * 256);
        // This chunk's Q tile into the intermediate-product tiles (free until the products),
        // then the next chunk's K tile into the other K buffer.
        load_k_tile(sbase + OFF_SH, p.q, p.T, p.Hq, hq, t0, tid);
        const int cn = c + p.groups;
        if (cn < nch)
            load_k_tile(sbase + OFF_K + ((it + 1) & 1) * (64 * 256), p.k, p.T, p.Hq, hq,
                        s0 + static_cast<int64_t>(cn) * kC, tid);

        // Gates (warp 0) while the tiles are in flight.
        if (warp == 0) {
            float lg[2], bt[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int i = lane + 32 * u;
                lg[u] = 0.0f;
                bt[u] = 0.0f;
                if (i < nt) {
                    const int64_t gi = (t0 + i) * p.Hv + h;
                    lg[u] = log_decay(exp_A, load_scalar(p.a, gi, p.gate_dtype), dtb);
                    bt[u] = sigmoid_f(load_scalar(p.b, gi, p.gate_dtype));
                }
            }
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
            g_beta[lane] = bt[0]; g_beta[lane + 32] = bt[1];
            g_gam2[lane] = x0 * kLog2e; g_gam2[lane + 32] = x1 * kLog2e;
            g_Gam[lane] = expf(x0); g_Gam[lane + 32] = expf(x1);
            g_dec[lane] = expf(xC - x0); g_dec[lane + 32] = expf(xC - x1);
        }
        // cp.async groups, oldest first: this chunk's K, its Q, [the next chunk's K].
        if (cn < nch) cp_async_wait<2>(); else cp_async_wait<1>();
        __syncthreads();

        // K K^T: warp w computes rows 16*(w&3).. and columns 32*(w>>2).. on mma.sync;
        // A[i][j] = beta_i exp(gamma_i - gamma_j) k_i.k_j for j < i (zero elsewhere) goes
        // to the A hi/lo tiles, its diagonal 16x16 blocks also to A_d in fp32.
        {
            const int r0 = (warp & 3) * 16, c0 = (warp >> 2) * 32;
            float acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t af[4];
                ldsm_x4(af, a_addr<256>(sK, r0, kk * 16, lane));
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t bf[4];
                    ldsm_x4(bf, b_addr_nk<256>(sK, c0 + np * 16, kk * 16, lane));
                    mma16816(acc[2 * np], af, bf[0], bf[1]);
                    mma16816(acc[2 * np + 1], af, bf[2], bf[3]);
                }
            }
            const int blk = warp & 3;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int i = r0 + g + 8 * half;
                const float gi = g_gam2[i], bi = g_beta[i];
#pragma unroll
                for (int ntl = 0; ntl < 4; ++ntl) {
                    const int j = c0 + ntl * 8 + 2 * t4;
                    float v[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u)
                        v[u] = j + u < i ? bi * exp2f(gi - g_gam2[j + u]) * acc[ntl][2 * half + u] : 0.0f;
                    float h0, l0, h1, l1;
                    split_bf16(v[0], h0, l0);
                    split_bf16(v[1], h1, l1);
                    *reinterpret_cast<uint32_t *>(sm + OFF_AH + swz<128>(i, j)) = pack_bf16x2(h0, h1);
                    *reinterpret_cast<uint32_t *>(sm + OFF_AL + swz<128>(i, j)) = pack_bf16x2(l0, l1);
                    if ((j >> 4) == blk) {
                        A_d[(blk * 16 + (i & 15)) * 17 + (j & 15)] = v[0];
                        A_d[(blk * 16 + (i & 15)) * 17 + (j & 15) + 1] = v[1];
                    }
                }
            }
        }
        __syncthreads();

        // D_b = (I + A_bb)^-1: thread (block o, column cc) of threads 0-63 solves column
        // cc by forward substitution (two partial sums per row).  Threads 64-127 zero
        // the upper off-diagonal blocks of T_a and T_b in the T hi/lo tiles.
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
                reinterpret_cast<__nv_bfloat16 *>(sm + OFF_TH + swz<128>(o + r, o + cc))[0] = __float2bfloat16_rn(hi);
                reinterpret_cast<__nv_bfloat16 *>(sm + OFF_TL + swz<128>(o + r, o + cc))[0] = __float2bfloat16_rn(lo);
                T_f[(o + r) * kLD + o + cc] = x[r];
            }
        } else if (tid < 128) {
            const int e = tid - 64, r = e >> 2, q = e & 3;     // 16 rows x 4 quads of 4 columns
#pragma unroll
            for (int blkz = 0; blkz < 2; ++blkz) {
                const int row = blkz * 32 + r, col = blkz * 32 + 16 + q * 4;
                *reinterpret_cast<uint2 *>(sm + OFF_TH + swz<128>(row, col)) = make_uint2(0u, 0u);
                *reinterpret_cast<uint2 *>(sm + OFF_TL + swz<128>(row, col)) = make_uint2(0u, 0u);
            }
        }
        __syncthreads();

        // Q K^T on mma.sync, same warp tiling as K K^T; P (bf16, swizzled) straight to the workspace.
        const int64_t unit = tc_slot(s0, c, n) * p.Hv + h;
        if (cn < nch) cp_async_wait<1>(); else cp_async_wait<0>();
        __syncthreads();
        {
            const uint32_t sQ = sbase + OFF_SH;
            const int r0 = (warp & 3) * 16, c0 = (warp >> 2) * 32;
            float acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t af[4];
                ldsm_x4(af, a_addr<256>(sQ, r0, kk * 16, lane));
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t bf[4];
                    ldsm_x4(bf, b_addr_nk<256>(sK, c0 + np * 16, kk * 16, lane));
                    mma16816(acc[2 * np], af, bf[0], bf[1]);
                    mma16816(acc[2 * np + 1], af, bf[2], bf[3]);
                }
            }
            uint8_t *dP = reinterpret_cast<uint8_t *>(p.ws_P) + unit * kTcPBytes;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int i = r0 + g + 8 * half;
                const float gi = g_gam2[i];
#pragma unroll
                for (int ntl = 0; ntl < 4; ++ntl) {
                    const int j = c0 + ntl * 8 + 2 * t4;
                    const float p0 = j <= i ? exp2f(gi - g_gam2[j]) * acc[ntl][2 * half] : 0.0f;
                    const float p1 = j + 1 <= i ? exp2f(gi - g_gam2[j + 1]) * acc[ntl][2 * half + 1] : 0.0f;
                    *reinterpret_cast<uint32_t *>(dP + swz<128>(i, j)) = pack_bf16x2(p0, p1);
                }
            }
        }
        __syncthreads();   // the Q tile is dead; the products below reuse its space

        const uint32_t Ah = sbase + OFF_AH, Al = sbase + OFF_AL, Th = sbase + OFF_TH, Tl = sbase + OFF_TL;
        const uint32_t Sh = sbase + OFF_SH, Sl = sbase + OFF_SL;
        // M_10 = A_10 D_0 (warp 0), M_32 = A_32 D_2 (warp 1)
        if (warp < 2) {
            const int o = warp * 32;
            float acc[2][4] = {};
            prod16(acc, Ah, Al, Th, Tl, o + 16, o, o, o, 1, lane);
            store16(acc, 1.0f, sm + OFF_SH, sm + OFF_SL, nullptr, o + 16, o, lane);
        }
        __syncthreads();
        // T_10 = -D_1 M_10 (warp 0), T_32 = -D_3 M_32 (warp 1)
        if (warp < 2) {
            const int o = warp * 32;
            float acc[2][4] = {};
            prod16(acc, Th, Tl, Sh, Sl, o + 16, o + 16, o + 16, o, 1, lane);
            store16(acc, -1.0f, sm + OFF_TH, sm + OFF_TL, T_f, o + 16, o, lane);
        }
        __syncthreads();
        // M_ba = A[32..64)[0..32) T_a (warps 0-3, one 16x16 block each)
        if (warp < 4) {
            const int rb = warp >> 1, cb = warp & 1;
            float acc[2][4] = {};
            prod16(acc, Ah, Al, Th, Tl, 32 + 16 * rb, 0, 0, 16 * cb, 2, lane);
            store16(acc, 1.0f, sm + OFF_SH, sm + OFF_SL, nullptr, 32 + 16 * rb, 16 * cb, lane);
        }
        __syncthreads();
        // T_ba = -T_b M_ba
        if (warp < 4) {
            const int rb = warp >> 1, cb = warp & 1;
            float acc[2][4] = {};
            prod16(acc, Th, Tl, Sh, Sl, 32 + 16 * rb, 32, 32, 16 * cb, 2, lane);
            const int gg = lane >> 2, tt = lane & 3;
#pragma unroll
            for (int ntl = 0; ntl < 2; ++ntl)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int row = 32 + 16 * rb + gg + 8 * hf, col = 16 * cb + ntl * 8 + 2 * tt;
                    T_f[row * kLD + col] = -acc[ntl][2 * hf];
                    T_f[row * kLD + col + 1] = -acc[ntl][2 * hf + 1];
                }
        }
        __syncthreads();

        // T (row-major, zero above the diagonal) and the gate vectors to the workspace.
        float *dT = p.ws_T + unit * (kTcTileBytes / 4);
#pragma unroll
        for (int u = 0; u < (64 * 16) / kThreads; ++u) {
            const int idx = tid + u * kThreads;
            const int i = idx >> 4, j = (idx & 15) * 4;
            float4 val;
            val.x = j <= i ? T_f[i * kLD + j] : 0.0f;
            val.y = j + 1 <= i ? T_f[i * kLD + j + 1] : 0.0f;
            val.z = j + 2 <= i ? T_f[i * kLD + j + 2] : 0.0f;
            val.w = j + 3 <= i ? T_f[i * kLD + j + 3] : 0.0f;
            *reinterpret_cast<float4 *>(dT + i * 64 + j) = val;
        }
        p.ws_g[unit * (kTcGateBytes / 4) + tid] = g_beta[tid];
        __syncthreads();   // the next chunk reuses every shared buffer
    }
}

}  // namespace

int prep_groups(int64_t chains) {
    // Enough CTAs for a few waves of 148 SMs x 2 resident CTAs.
    const int64_t want = 4 * 148 * 2;
    int64_t gsz = (want + chains - 1) / chains;
    return static_cast<int>(gsz < 1 ? 1 : (gsz > 64 ? 64 : gsz));
}

cudaError_t launch_chunk_prep(const PrefillArgs &p, float *ws_T, __nv_bfloat16 *ws_P, float *ws_g,
                              cudaStream_t stream) {
    const int64_t chains = p.num_seqs * p.Hv;
    if (chains == 0) return cudaSuccess;
    if (chains > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const int groups = prep_groups(chains);
    cudaError_t e = cudaFuncSetAttribute(chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) return e;
    PrepParams pp{static_cast<const __nv_bfloat16 *>(p.q), static_cast<const __nv_bfloat16 *>(p.k), p.A_log,
                  p.a, p.dt_bias, p.b, p.cu_seqlens, p.total_tokens, p.Hq, p.Hv, groups, p.gate_dtype,
                  p.param_dtype, ws_T, ws_g, ws_P};
    chunk_prep_kernel<<<dim3(static_cast<unsigned>(chains), groups), kThreads, SMEM_BYTES, stream>>>(pp);
    return cudaGetLastError();
}

}  // namespace gdn
