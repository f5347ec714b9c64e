// gdn_selftest.cu -- known-answer checks of the tcgen05 / TMA building blocks in
// sm100.cuh, built as a separate test library (libgdn_b200_selftest.so).
//
// One CTA computes D[128][N] = A[128][K] * B[N][K]^T with one operand layout
// combination per mode, exactly as the chunked prefill kernel issues them:
//   0: A K-major smem,          B K-major smem
//   1: A MN-major smem,         B K-major smem
//   2: A K-major smem,          B MN-major smem
//   3: A in TMEM,               B K-major smem
//   4: A in TMEM,               B MN-major smem
//   5: A K-major via TMA (128 token rows of X[:, h, :]),      B K-major smem   (K = 128)
//   6: A MN-major via TMA (A[d][t] = X[64+t][h][d], M = 128), B K-major smem   (K = 64)
//   7: A in TMEM,  B MN-major via TMA (B[d][t] = X[64+t][h][d], N = 128)       (K = 64)
// A and B are given row-major in global memory (bf16) for the smem/TMEM modes;
// the TMA modes read X [T][H][128] bf16 instead.  The host compares D with a
// float64 product.  Shared memory is over-allocated so that every descriptor
// stays inside the CTA's allocation whatever the stride interpretation.
#include <cuda_bf16.h>

#include <cstring>

#include "gdn_common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace gdn {
namespace {

using namespace sm100;

constexpr uint32_t kSmemA = 0;
constexpr uint32_t kSmemB = 64 * 1024;
constexpr uint32_t kSmemBytes = 200 * 1024;

__device__ void fill_kmajor(uint8_t *base, const __nv_bfloat16 *g, int rows, int K) {
    const int chunks = K / 8;
    for (int idx = threadIdx.x; idx < rows * chunks; idx += blockDim.x) {
        const int r = idx / chunks, c8 = idx % chunks;
        const uint4 v = *reinterpret_cast<const uint4 *>(g + r * K + c8 * 8);
        *reinterpret_cast<uint4 *>(base + (c8 / 8) * (rows * 128) + sw128(r, c8 % 8)) = v;
    }
}

__device__ void fill_mnmajor(uint8_t *base, const __nv_bfloat16 *g, int rows, int K) {
    const int mchunks = rows / 8;
    const uint16_t *gs = reinterpret_cast<const uint16_t *>(g);
    for (int idx = threadIdx.x; idx < K * mchunks; idx += blockDim.x) {
        const int k = idx / mchunks, mc = idx % mchunks;
        uint32_t w[4];
        for (int e = 0; e < 4; ++e)
            w[e] = uint32_t(gs[(mc * 8 + 2 * e) * K + k]) |
                   (uint32_t(gs[(mc * 8 + 2 * e + 1) * K + k]) << 16);
        *reinterpret_cast<uint4 *>(base + (mc / 8) * (K * 128) + sw128(k, mc % 8)) =
            make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void __launch_bounds__(128, 1)
selftest_kernel(const __grid_constant__ CUtensorMap xmap, int mode, const __nv_bfloat16 *A,
                const __nv_bfloat16 *B, int h, int N, int K, float *D, int *status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t bars[2];
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t bar_tma = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);

    if (threadIdx.x == 0) {
        mbar_init(bar_tma, 1);
        mbar_init(bar_mma, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&tmem_slot), 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t d_col = 0, a_col = 128;   // D in columns [0,128), TMEM-A in [128,192)
    uint8_t *sA = smem + kSmemA, *sB = smem + kSmemB;
    bool ok = true;

    // ---- operand staging
    const bool a_tmem = (mode == 3 || mode == 4 || mode == 7);
    if (mode == 0 || mode == 2) fill_kmajor(sA, A, 128, K);
    if (mode == 1) fill_mnmajor(sA, A, 128, K);
    if (mode == 0 || mode == 1 || mode == 3 || mode == 5 || mode == 6) fill_kmajor(sB, B, N, K);
    if (mode == 2 || mode == 4) fill_mnmajor(sB, B, N, K);
    if (a_tmem) {
        const int m = warp * 32 + lane;
        for (int c0 = 0; c0 < K / 2; c0 += 16) {
            uint32_t r[16];
            const uint32_t *row = reinterpret_cast<const uint32_t *>(A + m * K);
            for (int j = 0; j < 16; ++j) r[j] = row[c0 + j];
            tmem_st16(tmem_addr(tmem, warp * 32, a_col + c0), r);
        }
        tmem_wait_st();
    }
    if (mode >= 5 && threadIdx.x == 0) {
        tma_prefetch_desc(&xmap);
        const uint32_t dst = smem_u32(mode == 7 ? sB : sA);
        if (mode == 5) {
            mbar_arrive_expect_tx(bar_tma, 4 * 8192);
            for (int hk = 0; hk < 2; ++hk) {
                tma_load_3d(dst + hk * 16384, &xmap, bar_tma, 64 * hk, h, 0);
                tma_load_3d(dst + hk * 16384 + 8192, &xmap, bar_tma, 64 * hk, h, 64);
            }
        } else {
            mbar_arrive_expect_tx(bar_tma, 2 * 8192);
            tma_load_3d(dst, &xmap, bar_tma, 0, h, 64);
            tma_load_3d(dst + 8192, &xmap, bar_tma, 64, h, 64);
        }
    }
    if (mode >= 5) ok = mbar_wait(bar_tma, 0);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMA issue
    if (ok && threadIdx.x == 0) {
        const bool a_mn = (mode == 1 || mode == 6);
        const bool b_mn = (mode == 2 || mode == 4 || mode == 7);
        const uint32_t idesc = idesc_bf16_f32(128, N, a_mn, b_mn);
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
        for (int s = 0; s < K / 16; ++s) {
            uint64_t bd;
            if (b_mn) bd = smem_desc_sw128(b0 + s * 2048, (mode == 7 ? 64 : K) * 128, 1024);
            else bd = smem_desc_sw128(b0 + (s / 4) * (N * 128) + (s % 4) * 32, 16, 1024);
            if (a_tmem) {
                mma_ts(tmem + d_col, tmem + a_col + s * 8, bd, idesc, s > 0);
            } else {
                uint64_t ad;
                if (a_mn) ad = smem_desc_sw128(a0 + s * 2048, (mode == 6 ? 64 : K) * 128, 1024);
                else ad = smem_desc_sw128(a0 + (s / 4) * (128 * 128) + (s % 4) * 32, 16, 1024);
                mma_ss(tmem + d_col, ad, bd, idesc, s > 0);
            }
        }
        mma_commit(bar_mma);
    }
    bool mma_done = true;
    if (ok) ok = mma_done = mbar_wait(bar_mma, 0);
    tc_fence_after();

    // ---- readback: thread m holds row m of D
    if (ok) {
        const int m = warp * 32 + lane;
        for (int c0 = 0; c0 < N; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem_addr(tmem, warp * 32, d_col + c0), r);
            tmem_wait_ld();
            for (int j = 0; j < 16; ++j) D[m * N + c0 + j] = __uint_as_float(r[j]);
        }
    } else if (threadIdx.x == 0) {
        atomicExch(status, 1);
    }
    // Never free TMEM under an MMA that may still be running: one more bounded wait.
    if (!mma_done) mbar_wait(bar_mma, 0);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}


// Warp-role layout check (256 threads): warp 0 allocates all 512 TMEM columns and
// its lane 0 issues the MMAs (the allocating warp is the issuing warp); warps 4-7
// write the A operand into TMEM with 32-column stores and read the accumulator
// back with 32-column loads.  D = A[128][K] * B[N][K]^T with A in TMEM at column
// a_col and D at column d_col; B K-major in shared memory.
__global__ void __launch_bounds__(256, 1)
selftest_roles_kernel(const __nv_bfloat16 *A, const __nv_bfloat16 *B, int N, int K, int a_col,
                      int d_col, float *D, int *status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t b_mma = smem_u32(&bar);
    if (warp == 0) {
        if (lane == 0) {
            mbar_init(b_mma, 1);
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(smem_u32(&tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    uint8_t *sB = smem + kSmemB;
    // B by all threads; A into TMEM by warps 4-7 (thread m = row m).
    for (int idx = threadIdx.x; idx < N * (K / 8); idx += blockDim.x) {
        const int r = idx / (K / 8), c8 = idx % (K / 8);
        *reinterpret_cast<uint4 *>(sB + (c8 / 8) * (N * 128) + sw128(r, c8 % 8)) =
            *reinterpret_cast<const uint4 *>(B + r * K + c8 * 8);
    }
    if (warp >= 4) {
        const int m = (warp - 4) * 32 + lane;
        const uint32_t *row = reinterpret_cast<const uint32_t *>(A + m * K);
        for (int c0 = 0; c0 < K / 2; c0 += 32) {
            uint32_t r[32];
            for (int j = 0; j < 32; ++j) r[j] = row[c0 + j];
            tmem_st32(tmem_addr(tmem, (warp & 3) * 32, a_col + c0), r);
        }
        tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, N, false, false);
            const uint32_t b0 = smem_u32(sB);
            for (int s = 0; s < K / 16; ++s)
                mma_ts(tmem + d_col, tmem + a_col + s * 8,
                       smem_desc_sw128(b0 + (s / 4) * (N * 128) + (s % 4) * 32, 16, 1024), idesc,
                       s > 0);
            mma_commit(b_mma);
        }
        __syncwarp();
    }
    ok = mbar_wait(b_mma, 0);
    tc_fence_after();
    if (ok && warp >= 4) {
        const int m = (warp - 4) * 32 + lane;
        for (int c0 = 0; c0 < N; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tmem_addr(tmem, (warp & 3) * 32, d_col + c0), r);
            tmem_wait_ld_dep(r);
            for (int j = 0; j < 32; ++j) D[m * N + c0 + j] = __uint_as_float(r[j]);
        }
    }
    if (!ok && threadIdx.x == 0) atomicExch(status, 1);
    if (!ok) mbar_wait(b_mma, 0);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Bounded wait on an mbarrier that nothing ever arrives on: the wait must give up after
// `limit_ns` and return.  out[0] = 1 if the wait reported completion (a failure of the
// check), out[1] = elapsed ns of the wait, out[2] = 1 when the kernel reached its end.
__global__ void __launch_bounds__(32, 1) selftest_wait_timeout_kernel(uint64_t limit_ns,
                                                                      unsigned long long *out) {
    __shared__ uint64_t bar;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        const uint64_t t0 = global_timer_ns();
        const bool completed = mbar_wait(b, 0, limit_ns);
        const uint64_t t1 = global_timer_ns();
        out[0] = completed ? 1ull : 0ull;
        out[1] = t1 - t0;
        out[2] = 1ull;
    }
}

}  // namespace
}  // namespace gdn

// Bounded-wait check: one warp waits on an mbarrier nobody arrives on, with a limit of
// `limit_ns` (at most 0.1 s), and writes three counters to `out` (device, 3 x uint64).
extern "C" __attribute__((visibility("default"))) int gdn_selftest_wait_timeout(uint64_t limit_ns, void *out,
                                                                                void *stream) {
    if (limit_ns == 0 || limit_ns > 100000000ull || out == nullptr) return -1;
    gdn::selftest_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        limit_ns, static_cast<unsigned long long *>(out));
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

extern "C" __attribute__((visibility("default"))) int gdn_selftest_umma(
    int mode, const void *A, const void *B, const void *X, int T, int H, int h, int N, int K,
    float *D, int *status, void *stream) {
    using namespace gdn;
    if (mode < 0 || mode > 7 || (N != 64 && N != 128) || (K != 64 && K != 128)) return -1;
    if (mode >= 5 && (X == nullptr || T < 128 || h < 0 || h >= H)) return -1;
    if (mode == 5 && K != 128) return -1;
    if ((mode == 6 || mode == 7) && K != 64) return -1;
    if (mode == 7 && N != 128) return -1;
    CUtensorMap map;
    memset(&map, 0, sizeof(map));
    if (mode >= 5 && !make_tmap_thd_bf16(&map, X, T, H)) return -2;
    const auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaFuncSetAttribute(selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes + 1024);
    if (e != cudaSuccess) return -3;
    selftest_kernel<<<1, 128, kSmemBytes + 1024, s>>>(
        map, mode, static_cast<const __nv_bfloat16 *>(A), static_cast<const __nv_bfloat16 *>(B), h,
        N, K, D, status);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Warp-role layout check; a_col, d_col are TMEM column offsets (A needs K/2 columns,
// D needs N columns, both inside the 512 allocated).
extern "C" __attribute__((visibility("default"))) int gdn_selftest_roles(
    const void *A, const void *B, int N, int K, int a_col, int d_col, float *D, int *status,
    void *stream) {
    using namespace gdn;
    if ((N != 64 && N != 128) || (K != 64 && K != 128)) return -1;
    if (a_col < 0 || a_col % 32 || a_col + K / 2 > 512) return -1;
    if (d_col < 0 || d_col % 32 || d_col + N > 512) return -1;
    if ((a_col < d_col + N) && (d_col < a_col + K / 2)) return -1;   // must not overlap
    cudaError_t e = cudaFuncSetAttribute(selftest_roles_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes + 1024);
    if (e != cudaSuccess) return -3;
    selftest_roles_kernel<<<1, 256, kSmemBytes + 1024, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16 *>(A), static_cast<const __nv_bfloat16 *>(B), N, K, a_col,
        d_col, D, status);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
