// gdn_prefill_tc.cu -- chunked (C = 64) Gated DeltaNet prefill on the 5th-generation
// tensor cores: tcgen05.mma with TMEM accumulators, TMA-fed tiles, warp-specialised.
//
// Same recurrence as gdn_prefill_chunked.cu (solution/gdn_baseline_torch.py:71-87),
// in the "UW" form that puts only two tensor-core round trips on the serial state
// path of each 64-token chunk (state S0 = S[v][k] at the chunk start):
//
//   gamma_i = sum_{j<=i} log alpha_j,  Gamma_i = exp(gamma_i)
//   A[i][j] = beta_i exp(gamma_i - gamma_j) k_i.k_j  (j < i),   T = (I + A)^-1
//   U = T diag(beta) V,   W = T diag(beta Gamma) K            (independent of S0)
//   delta = U - W S0^T                                         (innovations, [i][v])
//   O     = scale (diag(Gamma) Q S0^T + P delta),  P[i][j] = exp(gamma_i - gamma_j) q_i.k_j (j <= i)
//   S_end = Gamma_63 S0 + sum_i exp(gamma_63 - gamma_i) delta_i k_i^T
//
// The state-independent inputs of every chunk -- its gates, the T' = T diag(beta) and
// T'' = T diag(beta Gamma) operand tiles and P -- come from gdn_chunk_prep.cu through
// a workspace (gdn_tc_workspace.h).  Padding tokens of a
// partial chunk have beta = 0 and log alpha = 0.  Every product with an fp32 operand
// (S0, T, W, the decayed delta) splits it into bf16 hi + lo.
//
// One CTA per (sequence, v-head) chain (the pooled entry points may rank the sequences
// longest first, TcParams::order), 16 warps in five roles that hand chunks to
// each other through mbarriers, so the next chunk's state-independent products run
// while the current chunk's state update is on the tensor core:
//   warp 0      allocates all 512 TMEM columns; lane 0 issues every MMA, each batch as
//               soon as its inputs are ready, state path first: per chunk c the order
//               on the tensor pipe is  W^T(c), [S update(c-1)], U^T(c), delta(c), ...
//               so W^T is computed while the previous innovation is being split
//   warp 13     lane 0 issues the copies of each chunk (TMA tiles, bulk T tiles, P and
//               gates) as soon as their previous readers are done
//   warps 1-4   prep (one per TMEM lane quadrant): the diag(Gamma) Q tile, -W from W^T
//               in TMEM, then the previous chunk's output rows from O^T in TMEM into a
//               bf16 staging tile
//   warps 14-17 output stores: the staging tile's rows to global memory, with the gated
//               RMSNorm of the output applied on the way when the call asks for it
//   warps 5-12  state path, two halves of four warps: S -> hi/lo split and decay, the
//               innovation split
// The fp32 state lives in TMEM columns [0,128) for the whole sequence.  The barrier
// protocol is modelled on the CPU under random schedules (tests/test_tc_chain_protocol.py).
//
// Every wait is bounded (2 s by default, TcParams::wait_ns).  A wait that gives up
// records its site in g_tc_error and raises a shared abort flag; every role then stops
// at its next wait (the staging-tile hand-off between the prep and store warps included),
// the issuing thread waits for the last commit of every MMA batch it issued and the copy
// thread for every copy it issued (both bounded by kDrainWaitNs), and the CTA frees TMEM
// and exits.
#include <cuda_bf16.h>
#include <atomic>
#include <cstring>
#include <mutex>

#include "gdn_chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_launch.h"
#include "gdn_mma_sync.cuh"
#include "gdn_tc_workspace.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace gdn {

__device__ int g_tc_error = 0;

// Limit of a role's wait when the caller sets none (gdn_set_wait_limit_ns(0)).
constexpr uint64_t kDefaultWaitNs = 2000000000ull;

namespace {

using namespace sm100;
using msync::cp_async16;
using msync::cp_async_commit;
using msync::cp_async_wait;

constexpr int kC = 64;
// warp 0: MMA issue; warps 1-4: prep; warps 5-12: state (two halves); warp 13: copies;
// warps 14-17: output stores (and the gated RMSNorm of the output, when asked for).
// 576 threads leave at most 112 registers a thread (65,536 per SM, one CTA).
constexpr int kThreads = 576;
constexpr int kStoreWarps = 4;

// Shared memory map (bytes from the 1024-aligned dynamic base).
constexpr uint32_t OFF_KQ = 0;              // 2 stages x 32 KB: [K_h0 | Q_h0 | K_h1 | Q_h1]
constexpr uint32_t KQ_STAGE = 32 * 1024;
constexpr uint32_t OFF_V = 64 * 1024;       // 2 stages x 16 KB: [V_h0 | V_h1]
constexpr uint32_t V_STAGE = 16 * 1024;
constexpr uint32_t OFF_O = 96 * 1024;       // 16 KB: bf16 [64][128] output staging
constexpr uint32_t OFF_P = 112 * 1024;      // 2 stages x 8 KB: P, K-major [i][j] (from the workspace)
constexpr uint32_t OFF_T1H = 128 * 1024;    // 8 KB each, K-major [i][j] (from the workspace):
constexpr uint32_t OFF_T1L = 136 * 1024;    //   T' = T diag(beta) hi/lo, T'' = T diag(beta Gamma) hi/lo
constexpr uint32_t OFF_T2H = 144 * 1024;
constexpr uint32_t OFF_T2L = 152 * 1024;
constexpr uint32_t OFF_WH = 160 * 1024;     // 16 KB each, MN-major [k][i]: -W hi, -W lo, (diag(Gamma) Q)^T;
constexpr uint32_t OFF_WL = 176 * 1024;     //   one N = 192 operand of the delta batch
constexpr uint32_t OFF_QS = 192 * 1024;
constexpr uint32_t OFF_GST = 208 * 1024;    // 2 stages x 1 KB: beta, gamma*log2(e), Gamma, decay-to-end
constexpr uint32_t SMEM_BYTES = 210 * 1024;
// With the gated output: the store warps' gate rows of one chunk, bf16 [64][128] (16 KB).
constexpr uint32_t OFF_Z = SMEM_BYTES;
constexpr uint32_t SMEM_BYTES_GATED = SMEM_BYTES + 16 * 1024;
constexpr int kStoreWarp0 = 14;
constexpr int kStoreRows = kC / kStoreWarps;     // rows of an output chunk per store warp
static_assert(OFF_T1L - OFF_T1H == kTcTileBytes && OFF_T2H - OFF_T1H == 2 * kTcTileBytes,
              "T tiles sit in shared memory in their workspace order (T'_hi rows 0-63 and T'_lo rows"
              " 64-127 of one K-major N = 128 operand)");
constexpr uint32_t kStageTx = 6 * 8192 + kTcPBytes + kTcGateBytes;

// TMEM columns (all 512 allocated).
constexpr uint32_t TM_S = 0;      // [0,128)   fp32 state S[v][k]
constexpr uint32_t TM_SHI = 128;  // [128,192) bf16x2 S hi | later delta bf16 [128,160)
constexpr uint32_t TM_SLO = 192;  // [192,256) bf16x2 S lo | later delta' hi [160,192), lo [192,224)
constexpr uint32_t TM_DBF = 128;
constexpr uint32_t TM_DPH = 160;
constexpr uint32_t TM_DPL = 192;
constexpr uint32_t TM_W = 256;    // [256,320) W^T (lanes k, columns i)
// The U batch writes [U | X] and the delta batch accumulates into [U | X | O] (lanes v,
// columns i); delta^T = U + X:
constexpr uint32_t TM_U = 320;    // [320,384) (T'_hi V)^T - S_hi W_hi^T - S_lo W_hi^T
constexpr uint32_t TM_X = 384;    // [384,448) (T'_lo V)^T - S_hi W_lo^T
constexpr uint32_t TM_O = 448;    // [448,512) (Gamma Q S_hi^T)^T, then O^T (zero before the batch)

enum WaitSite { kWaitTma = 1, kWaitWU = 3, kWaitD = 4, kWaitS = 5, kWaitTT = 6,
                kWaitW = 7, kWaitSS = 8, kWaitDS = 9, kWaitT = 10, kWaitIssue = 11, kWaitUD = 12,
                kWaitOFull = 13, kWaitOFree = 14 };
// Limit of the waits for the CTA's own MMAs and copies in flight once it stops (these
// complete on their own; the limit only keeps a broken device from holding the SM).
constexpr uint64_t kDrainWaitNs = 2000000000ull;
// (output reads O^T of chunk c before the delta batch of chunk c + 1 overwrites it)

struct TcParams {
    const float *state;
    const int32_t *cu_seqlens;
    int64_t num_seqs;
    int64_t T;
    int Hq, Hv;
    float scale;
    __nv_bfloat16 *out;
    float *new_state;
    const uint8_t *ws_T;
    const float *ws_g;
    const __nv_bfloat16 *ws_P;
    int64_t chain0;   // (sequence rank, v-head) chain of blockIdx.x = 0
    uint64_t wait_ns; // limit of every role's wait (ns)
    const int32_t *order;   // sequence of each rank (nullptr: rank = sequence index)
    // Gated RMSNorm of the output in the store (gate == nullptr: plain store):
    // o <- bf16(o / sqrt(mean(o^2) + eps) * w * silu(z)) per 128-element head vector.
    const __nv_bfloat16 *gate;   // z, [T, Hv, 128] bf16
    const void *norm_w;          // w, [128] (norm_w_dtype)
    int norm_w_dtype;
    float norm_eps;
};

struct Bars {
    uint64_t tma[2], wdone, udone, d, s, qs, w, ss, ds, tw, tu, free_[2], oread, ofull, ofree;
};

__device__ __forceinline__ void issue_chunk(const CUtensorMap *qmap, const CUtensorMap *kmap,
                                            const CUtensorMap *vmap, uint32_t sbase, int st,
                                            const __nv_bfloat16 *wP, const float *wg, uint32_t bar, int z,
                                            int hq, int h) {
    const uint32_t kq = sbase + OFF_KQ + st * KQ_STAGE, vv = sbase + OFF_V + st * V_STAGE;
    mbar_arrive_expect_tx(bar, kStageTx);
    bulk_load(sbase + OFF_P + st * kTcPBytes, wP, kTcPBytes, bar);
    bulk_load(sbase + OFF_GST + st * kTcGateBytes, wg, kTcGateBytes, bar);
    tma_load_3d(kq, kmap, bar, 0, hq, z);
    tma_load_3d(kq + 8192, qmap, bar, 0, hq, z);
    tma_load_3d(kq + 16384, kmap, bar, 64, hq, z);
    tma_load_3d(kq + 24576, qmap, bar, 64, hq, z);
    tma_load_3d(vv, vmap, bar, 0, h, z);
    tma_load_3d(vv + 8192, vmap, bar, 64, h, z);
}

// Longest a waiting thread sleeps between looks at the abort flag and the clock.
constexpr uint32_t kMaxSuspendNs = 1000000;

// Bounded wait that gives up at once when another role has already given up.  Each
// probe sleeps until the phase completes or min(limit, 1 ms) has passed, so the limit
// holds to within one probe however short it is, and a thread whose barrier will never
// complete (because another role gave up) notices the flag within 1 ms.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, int site, volatile int *abort,
                                             uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    const uint32_t hint = limit_ns < kMaxSuspendNs ? static_cast<uint32_t>(limit_ns) : kMaxSuspendNs;
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, hint)) return true;
        if (*abort) return false;
        if (global_timer_ns() - t0 > limit_ns) {
            atomicExch(&g_tc_error, site);
            *abort = 1;
            return false;
        }
    }
}
// Wait for this CTA's own asynchronous work (an MMA commit or a copy it issued), also
// after a give-up: it completes on its own.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int site) {
    volatile int never = 0;
    wait_bounded(bar, parity, site, &never, kDrainWaitNs);
}
// Whole-warp wait: reconverges the warp for the next .aligned tcgen05 op.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, int site, volatile int *abort,
                                          uint64_t limit_ns) {
    const bool ok = wait_bounded(bar, parity, site, abort, limit_ns);
    __syncwarp();
    tc_fence_after();
    return __all_sync(0xffffffffu, ok);
}
// One arrive per warp on a barrier counting the 4 warps of a role.
__device__ __forceinline__ void warp_arrive(uint32_t bar, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = smem_raw;
    __shared__ Bars bars;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    volatile int *abort = &abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t lane_base = static_cast<uint32_t>(warp & 3) * 32;
    const int row = static_cast<int>(lane_base) + lane;    // this thread's TMEM lane (warps 1-8)
    const int64_t chain = blockIdx.x + p.chain0;           // (sequence rank, v-head)
    const int64_t rank = chain / p.Hv;
    const int64_t n = p.order ? p.order[rank] : rank;
    const int h = static_cast<int>(chain % p.Hv);
    const int64_t nh = n * p.Hv + h;                         // (sequence, v-head) of the state
    const int hq = h / (p.Hv / p.Hq);
    if (tid == 0 && h == 0) check_seq_bounds(p.cu_seqlens, n, p.num_seqs, p.T, &g_tc_error);
    int64_t s0 = p.cu_seqlens[n], s1 = p.cu_seqlens[n + 1];
    s0 = s0 < 0 ? 0 : (s0 > p.T ? p.T : s0);
    s1 = s1 < s0 ? s0 : (s1 > p.T ? p.T : s1);
    const int nch = static_cast<int>((s1 - s0 + kC - 1) / kC);
    const uint32_t sbase = smem_u32(sm);
    const uint32_t b_tma0 = smem_u32(&bars.tma[0]), b_tma1 = smem_u32(&bars.tma[1]);
    // wdone / udone: the W^T / U^T batch of a chunk is done; tw / tu: its T'' / T' tiles arrived
    const uint32_t b_wdone = smem_u32(&bars.wdone), b_udone = smem_u32(&bars.udone), b_d = smem_u32(&bars.d);
    const uint32_t b_s = smem_u32(&bars.s), b_qs = smem_u32(&bars.qs), b_w = smem_u32(&bars.w);
    const uint32_t b_ss = smem_u32(&bars.ss), b_ds = smem_u32(&bars.ds);
    const uint32_t b_tw = smem_u32(&bars.tw), b_tu = smem_u32(&bars.tu);
    // free[b]: chunk c's S-update batch (the last reader of stage c & 1 and P buffer c & 1) is done
    const uint32_t b_free0 = smem_u32(&bars.free_[0]), b_free1 = smem_u32(&bars.free_[1]);
    const uint32_t b_oread = smem_u32(&bars.oread);   // the prep warps have read O^T of a chunk
    // output staging tile: ofull = the four prep warps have put output chunk j in it,
    // ofree = the four store warps have read chunk j out of it
    const uint32_t b_ofull = smem_u32(&bars.ofull), b_ofree = smem_u32(&bars.ofree);
    const uint64_t wl = p.wait_ns;
    float *dst_state = p.new_state + nh * kHeadDim * kHeadDim;

    if (warp == 0) {
        if (lane == 0) {
            mbar_init(b_tma0, 1);
            mbar_init(b_tma1, 1);
            mbar_init(b_wdone, 1);
            mbar_init(b_udone, 1);
            mbar_init(b_d, 1);
            mbar_init(b_s, 1);
            mbar_init(b_qs, 4);
            mbar_init(b_w, 4);
            mbar_init(b_ss, 8);
            mbar_init(b_ds, 8);
            mbar_init(b_tw, 1);
            mbar_init(b_tu, 1);
            mbar_init(b_free0, 1);
            mbar_init(b_free1, 1);
            mbar_init(b_oread, 4);
            mbar_init(b_ofull, 4);
            mbar_init(b_ofree, kStoreWarps);
            abort_flag = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(smem_u32(&tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_slot;

    if (nch == 0) {
        // Empty sequence: zero new state (solution/gdn_baseline_torch.py:61-62).
        for (int i = tid; i < kHeadDim * kHeadDim / 4; i += kThreads)
            reinterpret_cast<float4 *>(dst_state)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (warp == 0) {
        // ------------------------------------------------------------ MMA issue
        if (lane == 0) {
            // Shared-memory matrix descriptors, built once: every operand tile's base
            // descriptor plus, per MMA, its byte offset / 16 in the start-address field.
            const uint64_t dK0 = smem_desc_sw128(sbase + OFF_KQ, 16384, 1024);
            const uint64_t dV0 = smem_desc_sw128(sbase + OFF_V, 8192, 1024);
            const uint64_t dT1h = smem_desc_sw128(sbase + OFF_T1H, 16, 1024);
            const uint64_t dT2h = smem_desc_sw128(sbase + OFF_T2H, 16, 1024);
            // [-W hi | -W lo | (Gamma Q)^T]: three MN-major 64-column atoms 16 KB apart
            static_assert(OFF_WL - OFF_WH == 16384 && OFF_QS - OFF_WL == 16384, "N = 192 operand layout");
            const uint64_t dWh = smem_desc_sw128(sbase + OFF_WH, 16384, 1024);
            const uint64_t dP0 = smem_desc_sw128(sbase + OFF_P, 16, 1024);
            // (the lo tiles sit 8 or 16 KB above the hi tiles; stage 1 one stage above stage 0)
            constexpr uint64_t kLoT = (OFF_T1L - OFF_T1H) >> 4;
            static_assert(OFF_T2L - OFF_T2H == OFF_T1L - OFF_T1H, "T' / T'' hi-lo spacing");
            constexpr uint32_t id6 = idesc_bf16_f32(128, 64, true, false);
            auto mma6w = [&](int c) {   // W^T = K^T T''^T -> TM_W
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int s = 0; s < 4; ++s)
                        mma_ss(tm + TM_W, dK0 + (c & 1) * (KQ_STAGE >> 4) + 128 * s, dT2h + part * kLoT + 2 * s,
                               id6, part | s);
                mma_commit(b_wdone);
            };
            auto mma6u = [&](int c) {   // [U | X] = V^T [T'_hi | T'_lo]^T (the two tiles as one N = 128 operand)
                constexpr uint32_t id128 = idesc_bf16_f32(128, 128, true, false);
#pragma unroll
                for (int s = 0; s < 4; ++s)
                    mma_ss(tm + TM_U, dV0 + (c & 1) * (V_STAGE >> 4) + 128 * s, dT1h + 2 * s, id128, s);
                mma_commit(b_udone);
            };
            auto mma8 = [&](int) {      // [U | X | O] += S_hi [-W_hi | -W_lo | Gamma Q]^T;  U += S_lo (-W_hi)^T
                constexpr uint32_t id192 = idesc_bf16_f32(128, 192, false, true);
                constexpr uint32_t id64 = idesc_bf16_f32(128, 64, false, true);
#pragma unroll
                for (int s = 0; s < 8; ++s) mma_ts(tm + TM_U, tm + TM_SHI + 8 * s, dWh + 128 * s, id192, 1);
#pragma unroll
                for (int s = 0; s < 8; ++s) mma_ts(tm + TM_U, tm + TM_SLO + 8 * s, dWh + 128 * s, id64, 1);
                mma_commit(b_d);
            };
            auto mma10 = [&](int c) {   // S += delta'^T K, O^T += delta^T P^T
                const int st = c & 1;
                constexpr uint32_t ids = idesc_bf16_f32(128, 128, false, true);
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int s = 0; s < 4; ++s)
                        mma_ts(tm + TM_S, tm + (part ? TM_DPL : TM_DPH) + 8 * s, dK0 + st * (KQ_STAGE >> 4) + 128 * s,
                               ids, 1);
                constexpr uint32_t ido = idesc_bf16_f32(128, 64, false, false);
#pragma unroll
                for (int s = 0; s < 4; ++s)
                    mma_ts(tm + TM_O, tm + TM_DBF + 8 * s, dP0 + st * (kTcPBytes >> 4) + 2 * s, ido, 1);
                mma_commit(b_s);
                mma_commit(st ? b_free1 : b_free0);
            };
            // Event-driven issue: each MMA batch goes out as soon as its inputs are
            // ready, state-path batches first.  The loop probes with test_wait, which
            // never suspends (try_wait may, for a system-defined time, per probe).
            // n6w / n6u / n8 / n10 = next chunk of each batch kind.
            int n6w = 0, n6u = 0, n8 = 0, n10 = 0;
            bool ok = true;
            uint64_t t_idle = 0;
            uint32_t idle = 0;
            while (ok && n10 < nch) {
                bool progress = false;
                if (n10 < n8 && mbar_test_wait(b_ds, n10 & 1)) {
                    tc_fence_after();
                    mma10(n10++);
                    progress = true;
                }
                // delta goes behind its U^T batch; TM_O must have been read out
                if (n8 < n6u && mbar_test_wait(b_ss, n8 & 1) && mbar_test_wait(b_w, n8 & 1) &&
                    mbar_test_wait(b_qs, n8 & 1) && (n8 == 0 || mbar_test_wait(b_oread, (n8 - 1) & 1))) {
                    tc_fence_after();
                    mma8(n8++);
                    progress = true;
                }
                // W^T overwrites the previous chunk's, which the prep warps turned into -W
                // before the previous delta batch went out
                if (n6w < nch && n6w <= n8 && mbar_test_wait(b_tw, n6w & 1) &&
                    mbar_test_wait((n6w & 1) ? b_tma1 : b_tma0, (n6w >> 1) & 1)) {
                    tc_fence_after();
                    mma6w(n6w++);
                    progress = true;
                }
                // U^T reuses the buffer of chunk n6u - 2 and goes behind the previous
                // chunk's S update, never ahead of it
                if (n6u < n6w && n6u <= n10 && mbar_test_wait(b_tu, n6u & 1)) {
                    tc_fence_after();
                    mma6u(n6u++);
                    progress = true;
                }
                // Idle bookkeeping every 256 empty rounds (the timer read is slow).
                if (progress) {
                    idle = 0;
                } else if ((++idle & 255u) == 0) {
                    if (t_idle == 0 || idle == 256) {
                        t_idle = global_timer_ns();
                    } else if (*abort) {
                        ok = false;
                    } else if (global_timer_ns() - t_idle > wl) {
                        atomicExch(&g_tc_error, kWaitIssue);
                        *abort = 1;
                        ok = false;
                    }
                }
            }
            // Wait (bounded, also after a give-up) for the last commit of every kind, so
            // no MMA or barrier arrive is still in flight when the CTA leaves.
            if (n6w) drain_wait(b_wdone, (n6w - 1) & 1, kWaitWU);
            if (n6u) drain_wait(b_udone, (n6u - 1) & 1, kWaitUD);
            if (n8) drain_wait(b_d, (n8 - 1) & 1, kWaitD);
            if (n10) drain_wait(b_s, (n10 - 1) & 1, kWaitS);
            for (int c = n10 > 2 ? n10 - 2 : 0; c < n10; ++c)
                drain_wait((c & 1) ? b_free1 : b_free0, (c >> 1) & 1, kWaitS);
        }
        __syncwarp();
    } else if (warp == 13) {
        // ------------------------------------------------------------ copies
        // Per chunk c, in the order the previous readers finish: the T'' tiles once the
        // W^T batch of c - 1 is done, the stage (K, Q, V, P, gates) once the S update of
        // c - 2 is done, the T' tiles once the U^T batch of c - 1 is done.
        if (lane == 0) {
            int issued = 0, n_tw = 0, n_tu = 0;
            auto unit_of = [&](int c) { return tc_slot(s0, c, n) * p.Hv + h; };
            for (int c = 0; c < nch; ++c) {
                const int64_t unit = unit_of(c);
                if (c >= 1 && !wait_bounded(b_wdone, (c - 1) & 1, kWaitWU, abort, wl)) break;
                mbar_arrive_expect_tx(b_tw, 2 * kTcTileBytes);
                bulk_load(sbase + OFF_T2H, p.ws_T + unit * kTcTBytes + 2 * kTcTileBytes, 2 * kTcTileBytes, b_tw);
                ++n_tw;
                if (c >= 2 && !wait_bounded((c & 1) ? b_free1 : b_free0, ((c - 2) >> 1) & 1, kWaitS, abort, wl))
                    break;
                issue_chunk(&qmap, &kmap, &vmap, sbase, c & 1, p.ws_P + unit * (kTcPBytes / 2),
                            p.ws_g + unit * (kTcGateBytes / 4), (c & 1) ? b_tma1 : b_tma0,
                            static_cast<int>(s0 + c * kC), hq, h);
                ++issued;
                if (c >= 1 && !wait_bounded(b_udone, (c - 1) & 1, kWaitUD, abort, wl)) break;
                mbar_arrive_expect_tx(b_tu, 2 * kTcTileBytes);
                bulk_load(sbase + OFF_T1H, p.ws_T + unit * kTcTBytes, 2 * kTcTileBytes, b_tu);
                ++n_tu;
            }
            // Wait for the copies still in flight (none after a normal run, where their
            // readers have waited for them; after a give-up of any role, possibly some).
            for (int cc = issued > 2 ? issued - 2 : 0; cc < issued; ++cc)
                drain_wait((cc & 1) ? b_tma1 : b_tma0, (cc >> 1) & 1, kWaitTma);
            if (n_tw) drain_wait(b_tw, (n_tw - 1) & 1, kWaitT);
            if (n_tu) drain_wait(b_tu, (n_tu - 1) & 1, kWaitT);
        }
        __syncwarp();
    } else if (warp <= 4) {
        // ------------------------------------------------------------ prep (chunk c + 1 while c runs)
        const int pt = tid - 32;    // 0..127
        // The previous chunk's output: O^T out of TMEM (TM_O then zeroed for the next delta
        // batch), bf16 rows into the staging tile once the store warps have read the chunk
        // before out of it, then handed to the store warps.  False: another role gave up.
        auto write_out = [&](int c) -> bool {
            uint32_t o[64];
            tmem_ld32(tmem_addr(tm, lane_base, TM_O), *reinterpret_cast<uint32_t(*)[32]>(o));
            tmem_ld32(tmem_addr(tm, lane_base, TM_O + 32), *reinterpret_cast<uint32_t(*)[32]>(o + 32));
            tmem_wait_ld_dep(o);
            {
                const uint32_t z[32] = {};   // the next delta batch accumulates into O^T
                tmem_st32(tmem_addr(tm, lane_base, TM_O), z);
                tmem_st32(tmem_addr(tm, lane_base, TM_O + 32), z);
                tmem_wait_st();
            }
            tc_fence_before();
            warp_arrive(b_oread, lane);
            if (c > 0 && !wait_warp(b_ofree, (c - 1) & 1, kWaitOFree, abort, wl)) return false;
            // two tokens per packed conversion (the single-value one runs at a quarter of the
            // rate and these warps share their SMSPs with the state split)
            uint16_t *so16 = reinterpret_cast<uint16_t *>(sm + OFF_O);
#pragma unroll
            for (int ii = 0; ii < 64; ii += 2) {
                float o0, o1;
                unf2(mul_f2(f2(__uint_as_float(o[ii]), __uint_as_float(o[ii + 1])), f2(p.scale, p.scale)), o0, o1);
                const uint32_t pk = pack_bf16x2(o0, o1);
                so16[ii * kHeadDim + row] = static_cast<uint16_t>(pk);
                so16[(ii + 1) * kHeadDim + row] = static_cast<uint16_t>(pk >> 16);
            }
            warp_arrive(b_ofull, lane);
            return true;
        };
        for (int c = 0; c < nch; ++c) {
            const int st = c & 1;
            if (!wait_warp(st ? b_tma1 : b_tma0, (c >> 1) & 1, kWaitTma, abort, wl)) break;
            const float *g_Gam = reinterpret_cast<const float *>(sm + OFF_GST + st * kTcGateBytes) + 128;
            // diag(Gamma) Q once the previous chunk's Q S^T product has read the tile
            if (c > 0 && !wait_warp(b_d, (c - 1) & 1, kWaitD, abort, wl)) break;
            {
                // (diag(Gamma) Q)^T, MN-major [k][i]: thread pt = k reads column k of the Q
                // tile (two threads per 4-byte word, conflict-free) and writes row k.
                const uint8_t *src = sm + OFF_KQ + st * KQ_STAGE + 8192 + (pt >> 6) * 16384 + (pt & 7) * 2;
                const int kc = (pt & 63) >> 3;
                // (rolled: these warps' code shares the instruction caches with the other
                // roles, and keeping it small measurably shortens the whole chain)
#pragma unroll 1
                for (int ch = 0; ch < 8; ++ch) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = ch * 8 + 2 * e;
                        const float q0 = __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(src + sw128(i, kc)));
                        const float q1 =
                            __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(src + sw128(i + 1, kc)));
                        float s0, s1;
                        unf2(mul_f2(f2(q0, q1), f2(g_Gam[i], g_Gam[i + 1])), s0, s1);
                        w[e] = pack_bf16x2(s0, s1);
                    }
                    *reinterpret_cast<uint4 *>(sm + OFF_QS + sw128(pt, ch)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            if (c == 0) {
                // The delta batch accumulates into O^T: start from zero.
                const uint32_t z[32] = {};
                tmem_st32(tmem_addr(tm, lane_base, TM_O), z);
                tmem_st32(tmem_addr(tm, lane_base, TM_O + 32), z);
                tmem_wait_st();
            }
            fence_proxy_async_smem();
            tc_fence_before();
            warp_arrive(b_qs, lane);
            // -W as bf16 hi/lo, MN-major [k][i] (TMEM lane k holds row k of W^T)
            if (!wait_warp(b_wdone, c & 1, kWaitWU, abort, wl)) break;
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t r[32];
                tmem_ld32(tmem_addr(tm, lane_base, TM_W + 32 * hf), r);
                tmem_wait_ld_dep(r);
#pragma unroll
                for (int cq = 0; cq < 4; ++cq) {
                    uint32_t wh[4], wl[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // hi/lo of -W = hi/lo of W with both packed signs flipped (the
                        // rounding is symmetric)
                        split2_bf16_f2(__uint_as_float(r[cq * 8 + 2 * e]), __uint_as_float(r[cq * 8 + 2 * e + 1]),
                                       wh[e], wl[e]);
                        wh[e] ^= 0x80008000u;
                        wl[e] ^= 0x80008000u;
                    }
                    const uint32_t off = sw128(row, 4 * hf + cq);
                    *reinterpret_cast<uint4 *>(sm + OFF_WH + off) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
                    *reinterpret_cast<uint4 *>(sm + OFF_WL + off) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            warp_arrive(b_w, lane);
            // the previous chunk's output: O^T (TMEM lane v = column v of O) into registers,
            // release TM_O, then bf16 staging -> coalesced row stores
            if (c > 0 && (!wait_warp(b_s, (c - 1) & 1, kWaitS, abort, wl) || !write_out(c - 1))) break;
        }
        // (a warp leaves the loop early only after a give-up, which has raised the flag)
        if (!*abort && nch > 0 && wait_warp(b_s, (nch - 1) & 1, kWaitS, abort, wl)) write_out(nch - 1);
    } else if (warp >= kStoreWarp0) {
        // ------------------------------------------------------------ output stores
        // Store warp sw owns rows [16 sw, 16 sw + 16) of each output chunk, two rows per
        // step (16 lanes, 16 bytes each: one coalesced 256-byte row).  With a gate, each
        // row gets the gated RMSNorm of gdn_output_gate.cu (gated_rmsnorm16, the same
        // arithmetic, so the result equals prefill followed by that pass bit for bit); the
        // warp's gate rows of the next chunk are copied into shared memory (cp.async) as
        // soon as it is done with the current one.  Rows past the sequence end are read
        // from stale tile rows and never stored; the RMS shuffles of a row stay inside its
        // own 16 lanes.  (Short loops, unrolled at most twice: these warps share the
        // instruction caches with the chain's critical path; fully unrolled, the step took
        // 20 % longer.)
        const int sw = warp - kStoreWarp0;
        const int l16 = lane & 15, half = lane >> 4;
        const uint32_t zbase = sbase + OFF_Z + sw * (kStoreRows * 256);
        float wv[8] = {};
        if (p.gate) {
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[i] = load_scalar(p.norm_w, l16 * 8 + i, p.norm_w_dtype);
        }
        auto fetch_gate = [&](int c) {
            const int64_t t0 = s0 + static_cast<int64_t>(c) * kC;
            const int nt = static_cast<int>(s1 - t0 < kC ? s1 - t0 : kC);
#pragma unroll 1
            for (int u = 0; u < kStoreRows / 2; ++u) {
                const int r = 2 * u + half, i = kStoreRows * sw + r;
                if (i < nt)
                    cp_async16(zbase + r * 256 + l16 * 16, p.gate + ((t0 + i) * p.Hv + h) * kHeadDim + l16 * 8, 16);
            }
            cp_async_commit();
        };
        if (p.gate && nch > 0) fetch_gate(0);
        for (int c = 0; c < nch; ++c) {
            const int64_t t0 = s0 + static_cast<int64_t>(c) * kC;
            const int nt = static_cast<int>(s1 - t0 < kC ? s1 - t0 : kC);
            const bool ok = wait_warp(b_ofull, c & 1, kWaitOFull, abort, wl);
            if (p.gate) {
                cp_async_wait<0>();      // (also after a give-up: nothing left in flight)
                __syncwarp();
            }
            if (!ok) break;
#pragma unroll 2
            for (int u = 0; u < kStoreRows / 2; ++u) {
                const int r = 2 * u + half, i = kStoreRows * sw + r;
                uint4 y = *reinterpret_cast<const uint4 *>(sm + OFF_O + i * 256 + l16 * 16);
                if (p.gate) {            // (every lane: the RMS shuffles span the 16-lane group)
                    const uint4 zv = *reinterpret_cast<const uint4 *>(sm + OFF_Z + sw * (kStoreRows * 256) +
                                                                      r * 256 + l16 * 16);
                    y = gated_rmsnorm16(y, zv, wv, p.norm_eps);
                }
                if (i < nt) *reinterpret_cast<uint4 *>(p.out + ((t0 + i) * p.Hv + h) * kHeadDim + l16 * 8) = y;
            }
            warp_arrive(b_ofree, lane);
            if (p.gate && c + 1 < nch) fetch_gate(c + 1);
        }
    } else {
        // ------------------------------------------------------------ state path (chunk c)
        // Two halves of four warps (one per TMEM lane quadrant): half hs owns state
        // columns [64 hs, 64 hs + 64) and chunk tokens [32 hs, 32 hs + 32).
        const int v = row;    // state row / token row of this thread's TMEM lane
        const int hs = (warp - 5) >> 2;
        {
            const float *src = p.state ? p.state + (nh * kHeadDim + v) * kHeadDim : nullptr;
#pragma unroll 1
            for (int q4 = 2 * hs; q4 < 2 * hs + 2; ++q4) {
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
        bool ok = true;
        for (int c = 0; c < nch; ++c) {
            const int st = c & 1;
            // the previous chunk's S update is done
            if (c > 0 && !(ok = wait_warp(b_s, (c - 1) & 1, kWaitS, abort, wl))) break;
            if (!(ok = wait_warp(st ? b_tma1 : b_tma0, (c >> 1) & 1, kWaitTma, abort, wl))) break;
            const float *g_beta = reinterpret_cast<const float *>(sm + OFF_GST + st * kTcGateBytes);
            const float *g_Gam = g_beta + 128, *g_dec = g_beta + 192;
            // S -> bf16 hi/lo (TMEM A operands of the delta and output products); S <- Gamma_63 S
            {
                const float GamC = g_Gam[63];
#pragma unroll 1
                for (int q4 = 2 * hs; q4 < 2 * hs + 2; ++q4) {
                    uint32_t r[32], hi[16], lo[16];
                    tmem_ld32(tmem_addr(tm, lane_base, TM_S + 32 * q4), r);
                    tmem_wait_ld_dep(r);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        split2_bf16_f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]), hi[j], lo[j]);
                    tmem_st16(tmem_addr(tm, lane_base, TM_SHI + 16 * q4), hi);
                    tmem_st16(tmem_addr(tm, lane_base, TM_SLO + 16 * q4), lo);
                    const uint64_t g2 = f2(GamC, GamC);
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float s0, s1;
                        unf2(mul_f2(f2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), g2), s0, s1);
                        r[j] = __float_as_uint(s0);
                        r[j + 1] = __float_as_uint(s1);
                    }
                    tmem_st32(tmem_addr(tm, lane_base, TM_S + 32 * q4), r);
                    tmem_wait_st();
                }
            }
            tc_fence_before();
            warp_arrive(b_ss, lane);
            // delta (fp32, TMEM) -> bf16 (output path) and exp(gamma_63 - gamma_i) delta -> hi/lo
            if (!(ok = wait_warp(b_d, c & 1, kWaitD, abort, wl))) break;
            {
                uint32_t r[32], x[32], db[16], dh[16], dl[16];
                tmem_ld32(tmem_addr(tm, lane_base, TM_U + 32 * hs), r);
                tmem_ld32(tmem_addr(tm, lane_base, TM_X + 32 * hs), x);
                tmem_wait_ld_dep(r);
                tmem_wait_ld_dep(x);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int i0 = hs * 32 + 2 * e, i1 = i0 + 1;
                    const uint64_t d2 = add_f2(f2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1])),
                                               f2(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1])));
                    float d0, d1, e0, e1;
                    unf2(d2, d0, d1);
                    db[e] = pack_bf16x2(d0, d1);
                    unf2(mul_f2(d2, f2(g_dec[i0], g_dec[i1])), e0, e1);
                    split2_bf16_f2(e0, e1, dh[e], dl[e]);
                }
                tmem_st16(tmem_addr(tm, lane_base, TM_DBF + 16 * hs), db);
                tmem_st16(tmem_addr(tm, lane_base, TM_DPH + 16 * hs), dh);
                tmem_st16(tmem_addr(tm, lane_base, TM_DPL + 16 * hs), dl);
                tmem_wait_st();
            }
            tc_fence_before();
            warp_arrive(b_ds, lane);
        }
        if (ok && wait_warp(b_s, (nch - 1) & 1, kWaitS, abort, wl)) {
            float *dst = dst_state + v * kHeadDim;
#pragma unroll 1
            for (int q4 = 2 * hs; q4 < 2 * hs + 2; ++q4) {
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
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, 512);
    }
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

namespace {

// order[r] = the sequence of rank r among sequences [0, R) (longest first, ties by
// index), order[r] = r for R <= r < N.  One thread per sequence i, 32 per CTA; the CTA's
// eight warps split the sequences j it is compared with, 32 at a time (one load per
// lane, then a broadcast per j), and add their counts.  The rank of i is the number of
// j that come before it, so ranks are distinct.
constexpr int kOrderWarps = 8;

__device__ __forceinline__ int clamped_length(const int32_t *cu, int64_t j, int64_t T) {
    int64_t s0 = cu[j], s1 = cu[j + 1];
    s0 = s0 < 0 ? 0 : (s0 > T ? T : s0);
    s1 = s1 < s0 ? s0 : (s1 > T ? T : s1);
    return static_cast<int>(s1 - s0);
}

__global__ void __launch_bounds__(32 * kOrderWarps)
chain_order_kernel(const int32_t *cu, int64_t N, int64_t R, int64_t T, int32_t *order) {
    __shared__ int counts[kOrderWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 32 + lane;
    // Every lane runs the whole loop (full-warp shuffles, one block barrier); a lane
    // past R counts against length -2, which no sequence has, and its count is unused.
    const int li = i < R ? clamped_length(cu, i, T) : -2;
    int before = 0;
    for (int64_t jb = static_cast<int64_t>(warp) * 32; jb < R; jb += 32 * kOrderWarps) {
        const int lj_own = jb + lane < R ? clamped_length(cu, jb + lane, T) : -1;   // -1: no sequence
#pragma unroll 8
        for (int jj = 0; jj < 32; ++jj) {
            const int lj = __shfl_sync(0xffffffffu, lj_own, jj);
            before += (lj > li) || (lj == li && jb + jj < i);
        }
    }
    counts[warp][lane] = before;
    __syncthreads();
    if (warp == 0 && i < R) {
        int r = 0;
#pragma unroll
        for (int w = 0; w < kOrderWarps; ++w) r += counts[w][lane];
        order[r] = static_cast<int32_t>(i);
    } else if (warp == 0 && i < N) {
        order[i] = static_cast<int32_t>(i);
    }
}

}  // namespace

cudaError_t launch_chain_order(const int32_t *cu_seqlens, int64_t num_seqs, int64_t ranked,
                               int64_t total_tokens, int32_t *order, cudaStream_t stream) {
    if (num_seqs <= 0) return cudaSuccess;
    if (ranked < 0 || ranked > num_seqs) return cudaErrorInvalidValue;
    const int64_t ctas = (num_seqs + 31) / 32;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    chain_order_kernel<<<static_cast<unsigned>(ctas), 32 * kOrderWarps, 0, stream>>>(
        cu_seqlens, num_seqs, ranked, total_tokens, order);
    return cudaGetLastError();
}

// The ranking compares every pair of sequences (a few microseconds for thousands of
// sequences); beyond kMaxRankedSeqs the batch keeps sequence order.
constexpr int64_t kMaxRankedSeqs = 65536;

bool prefill_tc_orders_chains(int64_t num_seqs, int Hv, int sms) {
    return num_seqs >= 2 && num_seqs <= kMaxRankedSeqs && sms > 0 && num_seqs * Hv > sms;
}

int64_t prefill_tc_overlap_tail(int64_t chains, int sms, int heads_per_prep_cta) {
    if (sms <= 0 || chains <= sms) return 0;
    const int64_t tail = chains % sms;
    return (tail > 0 && tail % heads_per_prep_cta == 0) ? tail : 0;
}

namespace {

// The library's second stream of a device (highest priority) and its fork / join events,
// created on first use and kept until exit; `mu` serialises the fork-join enqueue.
// Limit of the chains' bounded waits set by gdn_set_wait_limit_ns (0: kDefaultWaitNs).
std::atomic<uint64_t> g_wait_limit_ns{0};

struct OverlapStream {
    cudaStream_t aux = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    int sms = 0;
    bool tried = false;
};
constexpr int kMaxDevices = 64;
OverlapStream g_overlap[kMaxDevices];
std::mutex g_overlap_mu;

// (with g_overlap_mu held) the device's overlap stream, or nullptr when it cannot be had.
OverlapStream *overlap_stream(cudaStream_t stream) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    OverlapStream &o = g_overlap[dev];
    if (!o.tried) {
        // Not created inside a stream capture (creation is then left to a later call).
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
            cudaGetLastError();   // (not left pending for the launch's own error check)
            return nullptr;
        }
        if (cs != cudaStreamCaptureStatusNone) return nullptr;
        o.tried = true;
        int lo = 0, hi = 0;
        if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
            cudaDeviceGetAttribute(&o.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaStreamCreateWithPriority(&o.aux, cudaStreamNonBlocking, hi) != cudaSuccess ||
            cudaEventCreateWithFlags(&o.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&o.join, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            o.aux = nullptr;
            return nullptr;
        }
    }
    return o.aux ? &o : nullptr;
}

// Whether this call may fork onto the shared overlap stream `aux`: either neither stream
// is being captured, or `stream` is being captured (the fork then pulls `aux` into that
// capture until it ends) and `aux` is free or already in that same capture.  While `aux`
// belongs to one capture, calls on other streams -- eager ones, or ones captured into
// another graph -- must not touch it: they run unsplit on their own stream.
bool aux_usable(cudaStream_t stream, cudaStream_t aux) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone, ca = cudaStreamCaptureStatusNone;
    unsigned long long id_s = 0, id_a = 0;
    if (cudaStreamGetCaptureInfo(stream, &cs, &id_s) != cudaSuccess ||
        cudaStreamGetCaptureInfo(aux, &ca, &id_a) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (cs == cudaStreamCaptureStatusInvalidated || ca == cudaStreamCaptureStatusInvalidated) return false;
    if (ca == cudaStreamCaptureStatusNone) return true;
    return cs == cudaStreamCaptureStatusActive && id_s == id_a;
}

}  // namespace

// The prep and chain kernels of every chain on `stream`, or -- with `overlap`, more
// chains than SMs and a partial last wave -- the last (chains mod SMs) chains on the
// high-priority overlap stream and the rest on `stream`: the block scheduler then runs
// the short group's chains on part of the GPU while the other group is being prepped,
// and the long group's chains fill whole waves.  The chain kernel takes one SM per chain
// (all 512 TMEM columns), so without the split the last wave of a batch of equal-length
// chains leaves (SMs - chains mod SMs) SMs idle for a whole chain length.
cudaError_t launch_prefill_tc(const PrefillArgs &p, void *workspace, cudaStream_t stream, bool overlap,
                              int32_t *order) {
    const int64_t ctas = p.num_seqs * p.Hv;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const int64_t units = tc_num_slots(p.total_tokens, p.num_seqs) * p.Hv;
    char *ws = static_cast<char *>(workspace);
    uint8_t *ws_T = reinterpret_cast<uint8_t *>(ws);
    __nv_bfloat16 *ws_P = reinterpret_cast<__nv_bfloat16 *>(ws + units * kTcTBytes);
    float *ws_g = reinterpret_cast<float *>(ws + units * (kTcTBytes + kTcPBytes));
    CUtensorMap qm, km, vm;
    std::memset(&qm, 0, sizeof(qm));
    std::memset(&km, 0, sizeof(km));
    std::memset(&vm, 0, sizeof(vm));
    if (!make_tmap_thd_bf16(&qm, p.q, p.total_tokens, p.Hq) ||
        !make_tmap_thd_bf16(&km, p.k, p.total_tokens, p.Hq) ||
        !make_tmap_thd_bf16(&vm, p.v, p.total_tokens, p.Hv))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES_GATED);
    const uint32_t smem = p.out_gate ? SMEM_BYTES_GATED : SMEM_BYTES;
    if (e != cudaSuccess) return e;
    const uint64_t limit = g_wait_limit_ns.load(std::memory_order_relaxed);
    const uint64_t wait_ns = limit ? limit : kDefaultWaitNs;
    // The split: the last `tail` chains (0: none) on the overlap stream.
    std::unique_lock<std::mutex> lock(g_overlap_mu, std::defer_lock);
    OverlapStream *o = nullptr;
    int64_t tail = 0;
    if (overlap) {
        lock.lock();
        o = overlap_stream(stream);
        if (o && aux_usable(stream, o->aux)) tail = prefill_tc_overlap_tail(ctas, o->sms, prep_heads_per_cta(p));
    }
    if (order) {
        // Chains run in launch order as SMs free up (list scheduling); longest first keeps
        // a long sequence late in the batch from starting its chains last.  Ranked: the
        // sequences whose chains all run on `stream` (the chunk prep there covers the same
        // sequences, in index order, before those chains start); the others keep their place.
        int sms = o ? o->sms : 0;
        if (!o) {
            int dev = 0;
            if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
            if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        }
        if (prefill_tc_orders_chains(p.num_seqs, p.Hv, sms)) {
            const int64_t ranked = (ctas - tail) / p.Hv;
            if ((e = launch_chain_order(p.cu_seqlens, p.num_seqs, ranked, p.total_tokens, order, stream)) !=
                cudaSuccess)
                return e;
        } else {
            order = nullptr;
        }
    }
    // prep + chains of [c0, c1) on stream st
    auto launch_range = [&](int64_t c0, int64_t c1, cudaStream_t st) -> cudaError_t {
        cudaError_t er = launch_chunk_prep(p, ws_T, ws_P, ws_g, st, c0, c1);
        if (er != cudaSuccess) return er;
        TcParams tp{p.state, p.cu_seqlens, p.num_seqs, p.total_tokens, p.Hq, p.Hv, p.scale,
                    static_cast<__nv_bfloat16 *>(p.out), p.new_state, ws_T, ws_g, ws_P, c0, wait_ns, order,
                    static_cast<const __nv_bfloat16 *>(p.out_gate), p.norm_w, p.norm_w_dtype, p.norm_eps};
        prefill_tc_kernel<<<static_cast<unsigned>(c1 - c0), kThreads, smem, st>>>(qm, km, vm, tp);
        return cudaGetLastError();
    };
    if (tail > 0) {
        // (the order kernel above is on `stream` before the fork)
        if ((e = cudaEventRecord(o->fork, stream)) != cudaSuccess) return e;
        if ((e = cudaStreamWaitEvent(o->aux, o->fork, 0)) != cudaSuccess) return e;
        if ((e = launch_range(ctas - tail, ctas, o->aux)) != cudaSuccess) return e;
        if ((e = cudaEventRecord(o->join, o->aux)) != cudaSuccess) return e;
        if ((e = launch_range(0, ctas - tail, stream)) != cudaSuccess) return e;
        return cudaStreamWaitEvent(stream, o->join, 0);
    }
    return launch_range(0, ctas, stream);
}

uint64_t set_wait_limit_ns(uint64_t ns) { return g_wait_limit_ns.exchange(ns); }

int *device_status_word() {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_tc_error) != cudaSuccess) {
        cudaGetLastError();   // (not left pending for the caller's launch check)
        return nullptr;
    }
    return static_cast<int *>(ptr);
}

cudaError_t read_device_status(cudaStream_t stream, int *code, bool clear) {
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
