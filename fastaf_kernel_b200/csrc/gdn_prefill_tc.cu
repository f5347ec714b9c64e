// gdn_prefill_tc.cu -- chunked (C = 64) Gated DeltaNet prefill on the 5th-generation
// tensor cores: tcgen05.mma with TMEM accumulators, TMA-fed q/k/v tiles.
//
// Same recurrence as gdn_prefill_chunked.cu (solution/gdn_baseline_torch.py:71-87),
// in the "UW" form that puts only two tensor-core round trips on the serial
// state path of each 64-token chunk (state S0 = S[v][k] at the chunk start):
//
//   gamma_i = sum_{j<=i} log alpha_j,  Gamma_i = exp(gamma_i)
//   A[i][j] = beta_i exp(gamma_i - gamma_j) k_i.k_j  (j < i),   T = (I + A)^-1
//   U = T diag(beta) V,   W = T diag(beta Gamma) K            (independent of S0)
//   delta = U - W S0^T                                         (innovations, [i][v])
//   O     = scale (diag(Gamma) Q S0^T + P delta),  P[i][j] = exp(gamma_i - gamma_j) q_i.k_j (j <= i)
//   S_end = Gamma_63 S0 + sum_i exp(gamma_63 - gamma_i) delta_i k_i^T
//
// Padding tokens of a partial chunk get beta = 0 and log alpha = 0, which makes
// their rows of T the identity and their innovations zero.  Every product with an
// fp32 operand (S0, T, W, the decayed delta) splits it into bf16 hi + lo.
//
// The state-independent part of every chunk -- its gates and T -- is computed for
// all chunks at once by gdn_chunk_prep.cu into a workspace (gdn_tc_workspace.h);
// this kernel streams T and the gate vectors in with the chunk's q/k/v tiles.
//
// One CTA per (sequence, v-head) chain.  Warp roles:
//   warp 0      allocates all 512 TMEM columns; lane 0 issues every TMA copy and MMA
//   warps 0-3   shared-memory work: diag(Gamma) Q, T', T''
//   warps 4-7   own TMEM lanes 0-127 (state row v / token row): every TMEM load/store
// The fp32 state lives in TMEM columns [0,128) for the whole sequence; the
// per-chunk inputs are double-buffered so the copy of chunk c+1 overlaps chunk c.
//
// Every mbarrier wait is bounded (about 2 s).  A wait that gives up records its
// site in g_tc_error; the CTA then stops at the next block barrier, waits
// (bounded) for its own copies and MMAs still in flight, frees TMEM and exits.
#include <cuda_bf16.h>

#include <cstring>

#include "gdn_chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_launch.h"
#include "sm100.cuh"
#include "gdn_tc_workspace.h"
#include "tma_host.h"

namespace gdn {

__device__ int g_tc_error = 0;

namespace {

using namespace sm100;

constexpr int kC = 64;
constexpr int kThreads = 256;

// Shared memory map (bytes from the 1024-aligned dynamic base).
constexpr uint32_t OFF_KQ = 0;              // 2 stages x 32 KB: [K_h0 | Q_h0 | K_h1 | Q_h1]
constexpr uint32_t KQ_STAGE = 32 * 1024;
constexpr uint32_t OFF_V = 64 * 1024;       // 2 stages x 16 KB: [V_h0 | V_h1]
constexpr uint32_t V_STAGE = 16 * 1024;
constexpr uint32_t OFF_QS = 96 * 1024;      // 16 KB: diag(Gamma) Q, K-major [i][k]
constexpr uint32_t OFF_P = 112 * 1024;      // 8 KB: P, K-major [i][j]
constexpr uint32_t OFF_T1H = 120 * 1024;    // 8 KB each: T diag(beta) hi/lo, T diag(beta Gamma) hi/lo
constexpr uint32_t OFF_T1L = 128 * 1024;
constexpr uint32_t OFF_T2H = 136 * 1024;
constexpr uint32_t OFF_T2L = 144 * 1024;
constexpr uint32_t OFF_WH = 152 * 1024;     // 16 KB each: -W hi/lo, MN-major [k][i]
constexpr uint32_t OFF_WL = 168 * 1024;
constexpr uint32_t OFF_TST = 184 * 1024;    // 2 stages x 16 KB: fp32 T [64][64] from the workspace
constexpr uint32_t OFF_GST = 216 * 1024;    // 2 stages x 1 KB: beta, gamma*log2(e), Gamma, exp(gamma_63 - gamma)
constexpr uint32_t OFF_O = OFF_QS;          // bf16 [64][128] output staging (over diag(Gamma) Q)
constexpr uint32_t SMEM_BYTES = 218 * 1024;
constexpr uint32_t kStageTx = 6 * 8192 + kTcTileBytes + kTcGateBytes;   // bytes per chunk copy
constexpr uint32_t SMEM_ALLOC = SMEM_BYTES + 1024;

// TMEM columns (all 512 allocated).
constexpr uint32_t TM_S = 0;      // [0,128)   fp32 state S[v][k]
constexpr uint32_t TM_SHI = 128;  // [128,192) bf16x2 S hi     | later delta bf16 [128,160)
constexpr uint32_t TM_SLO = 192;  // [192,256) bf16x2 S lo     | later delta' hi  [160,192), delta' lo [192,224)
constexpr uint32_t TM_DBF = 128;
constexpr uint32_t TM_DPH = 160;
constexpr uint32_t TM_DPL = 192;
constexpr uint32_t TM_D1A = 256;  // [256,320) U^T, then delta^T   (lanes v, columns i)
constexpr uint32_t TM_D1B = 320;  // [320,384) (Gamma Q S^T)^T, then O^T
constexpr uint32_t TM_KK = 384;   // [384,448) [K;Q] K^T: lanes 0-63 K K^T, lanes 64-127 Q K^T
constexpr uint32_t TM_W = 448;    // [448,512) W^T (lanes k, columns i)

enum WaitSite { kWaitTma = 1, kWaitKK = 2, kWaitWU = 3, kWaitD1 = 4, kWaitUpd = 5 };

struct TcParams {
    const float *state;
    const void *A_log, *a, *dt_bias, *b;
    const int32_t *cu_seqlens;
    int64_t T;
    int Hq, Hv;
    float scale;
    int gate_dtype, param_dtype;
    __nv_bfloat16 *out;
    float *new_state;
    const float *ws_T, *ws_g;
};

// The copies of one chunk: k and q halves into [K_h0|Q_h0|K_h1|Q_h1], v halves (TMA),
// and the chunk's T and gate vectors from the workspace (bulk copies).
__device__ __forceinline__ void issue_chunk(const CUtensorMap *qmap, const CUtensorMap *kmap,
                                            const CUtensorMap *vmap, uint32_t kq, uint32_t vv,
                                            uint32_t ts, uint32_t gs, const float *wT, const float *wg,
                                            uint32_t bar, int z, int hq, int h) {
    mbar_arrive_expect_tx(bar, kStageTx);
    bulk_load(ts, wT, kTcTileBytes, bar);
    bulk_load(gs, wg, kTcGateBytes, bar);
    tma_load_3d(kq, kmap, bar, 0, hq, z);
    tma_load_3d(kq + 8192, qmap, bar, 0, hq, z);
    tma_load_3d(kq + 16384, kmap, bar, 64, hq, z);
    tma_load_3d(kq + 24576, qmap, bar, 64, hq, z);
    tma_load_3d(vv, vmap, bar, 0, h, z);
    tma_load_3d(vv + 8192, vmap, bar, 64, h, z);
}

// Bounded wait on an mbarrier phase; records `site` in g_tc_error when it gives up.
// Ends with __syncwarp so the warp is converged for the next .aligned tcgen05 op.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, int site) {
    const bool ok = mbar_wait(bar, parity);
    if (!ok) atomicExch(&g_tc_error, site);
    __syncwarp();
    tc_fence_after();
    return ok;
}

__device__ __forceinline__ void block_sync_tc() {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

// Block barrier that also tells every thread whether all threads are still ok.
__device__ __forceinline__ bool block_sync_ok(bool ok) {
    tc_fence_before();
    const bool all = __syncthreads_and(ok) != 0;
    tc_fence_after();
    return all;
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = smem_raw;
    __shared__ uint64_t bar_tma[2];
    __shared__ uint64_t bar_mma;
    __shared__ uint32_t tmem_slot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool owner = warp >= 4;                      // TMEM lane owner
    const int v = tid - 128;                           // owner's lane (state row / token row)
    const uint32_t lane_base = static_cast<uint32_t>(warp & 3) * 32;
    const int64_t chain = blockIdx.x;
    const int64_t n = chain / p.Hv;
    const int h = static_cast<int>(chain % p.Hv);
    const int hq = h / (p.Hv / p.Hq);
    int64_t s0 = p.cu_seqlens[n], s1 = p.cu_seqlens[n + 1];
    s0 = s0 < 0 ? 0 : (s0 > p.T ? p.T : s0);
    s1 = s1 < s0 ? s0 : (s1 > p.T ? p.T : s1);
    const int nch = static_cast<int>((s1 - s0 + kC - 1) / kC);

    const uint32_t sbase = smem_u32(sm);
    const uint32_t b_tma0 = smem_u32(&bar_tma[0]), b_tma1 = smem_u32(&bar_tma[1]);
    const uint32_t b_mma = smem_u32(&bar_mma);

    if (warp == 0) {
        if (lane == 0) {
            mbar_init(b_tma0, 1);
            mbar_init(b_tma1, 1);
            mbar_init(b_mma, 1);
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(smem_u32(&tmem_slot), 512);
        tmem_relinquish();
    }
    block_sync_tc();
    const uint32_t tm = tmem_slot;
    float *dst_state = p.new_state + chain * kHeadDim * kHeadDim;

    // Thread 0's record of what it has in flight, for the drain after an abort.
    int tma_issued = 0, tma_done = 0;
    bool mma_inflight = false;
    uint32_t mma_phase = 0;
    bool ok = true;

    if (nch == 0) {
        // Empty sequence: zero new state (solution/gdn_baseline_torch.py:61-62).
        for (int i = tid; i < kHeadDim * kHeadDim / 4; i += kThreads)
            reinterpret_cast<float4 *>(dst_state)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
        if (owner) {   // initial state -> TMEM, lane v = state row v
            const float *src = p.state ? p.state + (chain * kHeadDim + v) * kHeadDim : nullptr;
            for (int q4 = 0; q4 < 4; ++q4) {
                uint32_t r[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 x = src ? *reinterpret_cast<const float4 *>(src + 32 * q4 + j)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                    r[j] = __float_as_uint(x.x); r[j + 1] = __float_as_uint(x.y);
                    r[j + 2] = __float_as_uint(x.z); r[j + 3] = __float_as_uint(x.w);
                }
                tmem_st32(tmem_addr(tm, lane_base, TM_S + 32 * q4), r);
                tmem_wait_st();
            }
        }
        if (tid == 0) {
            for (int c = 0; c < 2 && c < nch; ++c) {
                const int64_t unit = tc_slot(s0, c, n) * p.Hv + h;
                issue_chunk(&qmap, &kmap, &vmap, sbase + OFF_KQ + c * KQ_STAGE, sbase + OFF_V + c * V_STAGE,
                            sbase + OFF_TST + c * kTcTileBytes, sbase + OFF_GST + c * kTcGateBytes,
                            p.ws_T + unit * (kTcTileBytes / 4), p.ws_g + unit * (kTcGateBytes / 4),
                            c ? b_tma1 : b_tma0, static_cast<int>(s0 + c * kC), hq, h);
                ++tma_issued;
            }
        }
        for (int c = 0; c < nch; ++c) {
            const int st = c & 1;
            const int64_t t0 = s0 + static_cast<int64_t>(c) * kC;
            const int nt = static_cast<int>(s1 - t0 < kC ? s1 - t0 : kC);
            const uint32_t kq = sbase + OFF_KQ + st * KQ_STAGE;
            const uint32_t vv = sbase + OFF_V + st * V_STAGE;

            // (1) this chunk's tiles, T and gates (every thread reads the gate vectors)
            ok = wait_phase(st ? b_tma1 : b_tma0, (c >> 1) & 1, kWaitTma);
            if (tid == 0 && ok) ++tma_done;
            if (!block_sync_ok(ok)) break;
            const float *g_beta = reinterpret_cast<const float *>(sm + OFF_GST + st * kTcGateBytes);
            const float *g_gam2 = g_beta + 64, *g_Gam = g_beta + 128, *g_dec = g_beta + 192;
            const float *T_s = reinterpret_cast<const float *>(sm + OFF_TST + st * kTcTileBytes);

            if (owner) {
                // (2) S -> bf16 hi/lo (TMEM A operands); S <- Gamma_63 * S
                const float GamC = g_Gam[63];
                for (int q4 = 0; q4 < 4; ++q4) {
                    uint32_t r[32], hi[16], lo[16];
                    tmem_ld32(tmem_addr(tm, lane_base, TM_S + 32 * q4), r);
                    tmem_wait_ld_dep(r);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float h0, l0, h1, l1;
                        split_bf16(__uint_as_float(r[2 * j]), h0, l0);
                        split_bf16(__uint_as_float(r[2 * j + 1]), h1, l1);
                        hi[j] = pack_bf16x2(h0, h1);
                        lo[j] = pack_bf16x2(l0, l1);
                    }
                    tmem_st16(tmem_addr(tm, lane_base, TM_SHI + 16 * q4), hi);
                    tmem_st16(tmem_addr(tm, lane_base, TM_SLO + 16 * q4), lo);
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * GamC);
                    tmem_st32(tmem_addr(tm, lane_base, TM_S + 32 * q4), r);
                    tmem_wait_st();
                }
            } else {
                // (3) [K;Q] K^T on the tensor core (its Q K^T rows); diag(Gamma) Q
                if (tid == 0) {
                    const uint32_t id = idesc_bf16_f32(128, 64, false, false);
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint32_t off = (s >> 2) * 16384 + (s & 3) * 32;
                        mma_ss(tm + TM_KK, smem_desc_sw128(kq + off, 16, 1024),
                               smem_desc_sw128(kq + off, 16, 1024), id, s > 0);
                    }
                    mma_commit(b_mma);
                    mma_inflight = true;
                }
                __syncwarp();
                const int i = tid >> 1, half = tid & 1;
                const uint8_t *src = sm + OFF_KQ + st * KQ_STAGE + half * 16384 + 8192;
                uint8_t *dst = sm + OFF_QS + half * 8192;
                const float gi = g_Gam[i];
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    const uint32_t off = sw128(i, ch);
                    const uint4 x = *reinterpret_cast<const uint4 *>(src + off);
                    uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) w[e] = pack_bf16x2(bf16_lo(w[e]) * gi, bf16_hi(w[e]) * gi);
                    *reinterpret_cast<uint4 *>(dst + off) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                fence_proxy_async_smem();
            }
            if (!block_sync_ok(ok)) break;

            // (4) P = lower(exp(gamma_i - gamma_j) Q K^T) (owner lanes 64-127)
            ok = wait_phase(b_mma, mma_phase, kWaitKK);
            if (ok) { mma_phase ^= 1; mma_inflight = false; }
            if (owner && v >= 64) {
                const int i = v - 64;
                const float gi = g_gam2[i];
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t r[32];
                    tmem_ld32(tmem_addr(tm, lane_base, TM_KK + 32 * hf), r);
                    tmem_wait_ld_dep(r);
#pragma unroll
                    for (int cq = 0; cq < 4; ++cq) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int jj = cq * 8 + 2 * e, j0 = 32 * hf + jj, j1 = j0 + 1;
                            const float p0 = j0 <= i ? exp2f(gi - g_gam2[j0]) * __uint_as_float(r[jj]) : 0.0f;
                            const float p1 = j1 <= i ? exp2f(gi - g_gam2[j1]) * __uint_as_float(r[jj + 1]) : 0.0f;
                            w[e] = pack_bf16x2(p0, p1);
                        }
                        *reinterpret_cast<uint4 *>(sm + OFF_P + sw128(i, 4 * hf + cq)) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
                fence_proxy_async_smem();
            }

            // (5) T' = T diag(beta), T'' = T diag(beta Gamma) as bf16 hi/lo (T from the workspace)
            {
                const int i = tid >> 2, qd = tid & 3;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int ch = 2 * qd + cc;
                    uint32_t w1h[4], w1l[4], w2h[4], w2l[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float v1[2], v2[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int j = ch * 8 + 2 * e + u;
                            const float t = T_s[i * 64 + j];
                            v1[u] = t * g_beta[j];
                            v2[u] = v1[u] * g_Gam[j];
                        }
                        float h0, l0, h1, l1;
                        split_bf16(v1[0], h0, l0); split_bf16(v1[1], h1, l1);
                        w1h[e] = pack_bf16x2(h0, h1); w1l[e] = pack_bf16x2(l0, l1);
                        split_bf16(v2[0], h0, l0); split_bf16(v2[1], h1, l1);
                        w2h[e] = pack_bf16x2(h0, h1); w2l[e] = pack_bf16x2(l0, l1);
                    }
                    const uint32_t off = sw128(i, ch);
                    *reinterpret_cast<uint4 *>(sm + OFF_T1H + off) = make_uint4(w1h[0], w1h[1], w1h[2], w1h[3]);
                    *reinterpret_cast<uint4 *>(sm + OFF_T1L + off) = make_uint4(w1l[0], w1l[1], w1l[2], w1l[3]);
                    *reinterpret_cast<uint4 *>(sm + OFF_T2H + off) = make_uint4(w2h[0], w2h[1], w2h[2], w2h[3]);
                    *reinterpret_cast<uint4 *>(sm + OFF_T2L + off) = make_uint4(w2l[0], w2l[1], w2l[2], w2l[3]);
                }
            }
            fence_proxy_async_smem();
            if (!block_sync_ok(ok)) break;

            // (6) W^T = K^T T''^T (lanes k), U^T = V^T T'^T (lanes v)
            if (tid == 0) {
                const uint32_t id = idesc_bf16_f32(128, 64, true, false);
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    const uint32_t t2 = sbase + (part ? OFF_T2L : OFF_T2H);
                    const uint32_t t1 = sbase + (part ? OFF_T1L : OFF_T1H);
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        mma_ss(tm + TM_W, smem_desc_sw128(kq + s * 2048, 16384, 1024),
                               smem_desc_sw128(t2 + s * 32, 16, 1024), id, part | s);
                        mma_ss(tm + TM_D1A, smem_desc_sw128(vv + s * 2048, 8192, 1024),
                               smem_desc_sw128(t1 + s * 32, 16, 1024), id, part | s);
                    }
                }
                mma_commit(b_mma);
                mma_inflight = true;
            }
            ok = wait_phase(b_mma, mma_phase, kWaitWU);
            if (ok) { mma_phase ^= 1; mma_inflight = false; }

            // (7) -W as bf16 hi/lo, MN-major [k][i] (owner lane k holds row k of W^T)
            if (owner) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t r[32];
                    tmem_ld32(tmem_addr(tm, lane_base, TM_W + 32 * hf), r);
                    tmem_wait_ld_dep(r);
#pragma unroll
                    for (int cq = 0; cq < 4; ++cq) {
                        uint32_t wh[4], wl[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float h0, l0, h1, l1;
                            split_bf16(-__uint_as_float(r[cq * 8 + 2 * e]), h0, l0);
                            split_bf16(-__uint_as_float(r[cq * 8 + 2 * e + 1]), h1, l1);
                            wh[e] = pack_bf16x2(h0, h1);
                            wl[e] = pack_bf16x2(l0, l1);
                        }
                        const uint32_t off = sw128(v, 4 * hf + cq);
                        *reinterpret_cast<uint4 *>(sm + OFF_WH + off) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
                        *reinterpret_cast<uint4 *>(sm + OFF_WL + off) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
                    }
                }
                fence_proxy_async_smem();
            }
            if (!block_sync_ok(ok)) break;

            // (8) delta^T = U^T - S W^T (3 split products); (Gamma Q S^T)^T
            if (tid == 0) {
                const uint32_t idw = idesc_bf16_f32(128, 64, false, true);
#pragma unroll
                for (int part = 0; part < 3; ++part) {
                    const uint32_t src = part == 1 ? TM_SLO : TM_SHI;
                    const uint32_t wt = sbase + (part == 2 ? OFF_WL : OFF_WH);
#pragma unroll
                    for (int s = 0; s < 8; ++s)
                        mma_ts(tm + TM_D1A, tm + src + 8 * s, smem_desc_sw128(wt + s * 2048, 8192, 1024),
                               idw, 1);
                }
                const uint32_t idq = idesc_bf16_f32(128, 64, false, false);
#pragma unroll
                for (int s = 0; s < 8; ++s)
                    mma_ts(tm + TM_D1B, tm + TM_SHI + 8 * s,
                           smem_desc_sw128(sbase + OFF_QS + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024),
                           idq, s > 0);
                mma_commit(b_mma);
                mma_inflight = true;
            }
            ok = wait_phase(b_mma, mma_phase, kWaitD1);
            if (ok) { mma_phase ^= 1; mma_inflight = false; }

            // (9) delta -> bf16 (output path), exp(gamma_63 - gamma_i) delta -> hi/lo (state path)
            if (owner) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t r[32], db[16], dh[16], dl[16];
                    tmem_ld32(tmem_addr(tm, lane_base, TM_D1A + 32 * half), r);
                    tmem_wait_ld_dep(r);
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int i0 = half * 32 + 2 * e, i1 = i0 + 1;
                        const float d0 = __uint_as_float(r[2 * e]), d1 = __uint_as_float(r[2 * e + 1]);
                        db[e] = pack_bf16x2(d0, d1);
                        float h0, l0, h1, l1;
                        split_bf16(d0 * g_dec[i0], h0, l0);
                        split_bf16(d1 * g_dec[i1], h1, l1);
                        dh[e] = pack_bf16x2(h0, h1);
                        dl[e] = pack_bf16x2(l0, l1);
                    }
                    tmem_st16(tmem_addr(tm, lane_base, TM_DBF + 16 * half), db);
                    tmem_st16(tmem_addr(tm, lane_base, TM_DPH + 16 * half), dh);
                    tmem_st16(tmem_addr(tm, lane_base, TM_DPL + 16 * half), dl);
                }
                tmem_wait_st();
            }
            if (!block_sync_ok(ok)) break;

            // (10) S += delta'^T K (split), O^T += delta^T P^T
            if (tid == 0) {
                const uint32_t ids = idesc_bf16_f32(128, 128, false, true);
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int s = 0; s < 4; ++s)
                        mma_ts(tm + TM_S, tm + (part ? TM_DPL : TM_DPH) + 8 * s,
                               smem_desc_sw128(kq + s * 2048, 16384, 1024), ids, 1);
                const uint32_t ido = idesc_bf16_f32(128, 64, false, false);
#pragma unroll
                for (int s = 0; s < 4; ++s)
                    mma_ts(tm + TM_D1B, tm + TM_DBF + 8 * s,
                           smem_desc_sw128(sbase + OFF_P + s * 32, 16, 1024), ido, 1);
                mma_commit(b_mma);
                mma_inflight = true;
            }
            ok = wait_phase(b_mma, mma_phase, kWaitUpd);
            if (ok) { mma_phase ^= 1; mma_inflight = false; }

            // (11) this chunk's output: owner lane v -> column v of a bf16 [i][v] tile,
            //      then coalesced 16-byte row stores; refill this stage with chunk c+2
            if (owner) {
                __nv_bfloat16 *so = reinterpret_cast<__nv_bfloat16 *>(sm + OFF_O) + v;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t r[32];
                    tmem_ld32(tmem_addr(tm, lane_base, TM_D1B + 32 * hf), r);
                    tmem_wait_ld_dep(r);
#pragma unroll
                    for (int ii = 0; ii < 32; ++ii)
                        so[(32 * hf + ii) * kHeadDim] = __float2bfloat16_rn(p.scale * __uint_as_float(r[ii]));
                }
            }
            if (tid == 0 && ok && c + 2 < nch) {
                const int64_t unit = tc_slot(s0, c + 2, n) * p.Hv + h;
                issue_chunk(&qmap, &kmap, &vmap, kq, vv, sbase + OFF_TST + st * kTcTileBytes,
                            sbase + OFF_GST + st * kTcGateBytes, p.ws_T + unit * (kTcTileBytes / 4),
                            p.ws_g + unit * (kTcGateBytes / 4), st ? b_tma1 : b_tma0,
                            static_cast<int>(t0 + 2 * kC), hq, h);
                ++tma_issued;
            }
            if (!block_sync_ok(ok)) break;
            for (int idx = tid; idx < nt * 16; idx += kThreads) {
                const int i = idx >> 4, c16 = idx & 15;
                const uint4 val = *reinterpret_cast<const uint4 *>(sm + OFF_O + i * 256 + c16 * 16);
                *reinterpret_cast<uint4 *>(p.out + ((t0 + i) * p.Hv + h) * kHeadDim + c16 * 8) = val;
            }
        }

        if (ok && owner) {   // final state: TMEM -> new_state (owner lane v writes row v)
            float *dst = dst_state + v * kHeadDim;
            for (int q4 = 0; q4 < 4; ++q4) {
                uint32_t r[32];
                tmem_ld32(tmem_addr(tm, lane_base, TM_S + 32 * q4), r);
                tmem_wait_ld_dep(r);
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(dst + 32 * q4 + j) =
                        make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                    __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            }
        }
        // After an abort: wait (bounded) for thread 0's MMAs and copies still in flight.
        if (tid == 0) {
            if (mma_inflight) mbar_wait(b_mma, mma_phase);
            for (int cc = tma_done; cc < tma_issued; ++cc)
                mbar_wait((cc & 1) ? b_tma1 : b_tma0, (cc >> 1) & 1);
        }
    }
    block_sync_tc();
    if (warp == 0) tmem_dealloc(tm, 512);
}

int g_sm100 = -2;   // cached: device index known to be sm_100

bool is_sm100() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (g_sm100 == dev) return true;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major == 10 && minor == 0) {
        g_sm100 = dev;
        return true;
    }
    return false;
}

}  // namespace

// The TMA box is 64 tokens deep; the tensor must be at least that long.
bool prefill_tc_supported(const PrefillArgs &p) {
    return p.total_tokens >= kC && p.total_tokens < (int64_t(1) << 31) && is_sm100();
}

size_t prefill_tc_workspace_bytes(const PrefillArgs &p) {
    return static_cast<size_t>(tc_workspace_bytes(p.total_tokens, p.num_seqs, p.Hv));
}

// Two launches on `stream`: the per-chunk prep of every chunk, then the chains.
cudaError_t launch_prefill_tc(const PrefillArgs &p, void *workspace, cudaStream_t stream) {
    const int64_t ctas = p.num_seqs * p.Hv;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    float *ws_T = static_cast<float *>(workspace);
    float *ws_g = reinterpret_cast<float *>(static_cast<char *>(workspace) +
                                            tc_num_slots(p.total_tokens, p.num_seqs) * p.Hv * kTcTileBytes);
    CUtensorMap qm, km, vm;
    std::memset(&qm, 0, sizeof(qm));
    std::memset(&km, 0, sizeof(km));
    std::memset(&vm, 0, sizeof(vm));
    if (!make_tmap_thd_bf16(&qm, p.q, p.total_tokens, p.Hq) ||
        !make_tmap_thd_bf16(&km, p.k, p.total_tokens, p.Hq) ||
        !make_tmap_thd_bf16(&vm, p.v, p.total_tokens, p.Hv))
        return cudaErrorInvalidValue;
    cudaError_t e = launch_chunk_prep(p, ws_T, ws_g, stream);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e != cudaSuccess) return e;
    TcParams tp{p.state, p.A_log, p.a, p.dt_bias, p.b, p.cu_seqlens, p.total_tokens, p.Hq, p.Hv,
                p.scale, p.gate_dtype, p.param_dtype, static_cast<__nv_bfloat16 *>(p.out),
                p.new_state, ws_T, ws_g};
    prefill_tc_kernel<<<static_cast<unsigned>(ctas), kThreads, SMEM_ALLOC, stream>>>(qm, km, vm, tp);
    return cudaGetLastError();
}

cudaError_t read_tc_device_error(cudaStream_t stream, int *code, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(code, g_tc_error, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess || !clear || *code == 0) return e;
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

}  // namespace gdn
