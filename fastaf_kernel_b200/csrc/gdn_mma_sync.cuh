// gdn_mma_sync.cuh -- warp-level tensor-core helpers (mma.sync m16n8k16 bf16,
// ldmatrix, cp.async) over the XOR-swizzled shared-memory tiles of
// gdn_chunk_common.cuh, shared by the chunked prefill kernels.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "gdn_chunk_common.cuh"
#include "gdn_common.cuh"

namespace gdn {
namespace msync {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// 16-byte async copy global -> shared; src_bytes = 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ldmatrix address of a 16x16 A block (rows r0.., cols c0..) of a swizzled tile.
template <int kRowBytes>
__device__ __forceinline__ uint32_t a_addr(uint32_t base, int r0, int c0, int lane) {
    return base + swz<kRowBytes>(r0 + (lane & 15), c0 + ((lane >> 4) << 3));
}
// ldmatrix (non-trans) address for B fragments of two n-tiles (n0, n0+8) at k-step k0,
// from a tile stored [n][k].
template <int kRowBytes>
__device__ __forceinline__ uint32_t b_addr_nk(uint32_t base, int n0, int k0, int lane) {
    const int q = lane >> 3;
    return base + swz<kRowBytes>(n0 + (lane & 7) + ((q >> 1) << 3), k0 + ((q & 1) << 3));
}
// ldmatrix.trans address for B fragments of two n-tiles at k-step k0, from a tile
// stored [k][n].
template <int kRowBytes>
__device__ __forceinline__ uint32_t b_addr_kn(uint32_t base, int n0, int k0, int lane) {
    const int q = lane >> 3;
    return base + swz<kRowBytes>(k0 + (lane & 7) + ((q & 1) << 3), n0 + ((q >> 1) << 3));
}

// A fragment for k-step kk built from fp32 accumulators of n-tiles 2kk, 2kk+1
// (the accumulator's columns become the next product's K dimension).
__device__ __forceinline__ void acc_to_a_bf16(const float (&c0)[4], const float (&c1)[4],
                                              uint32_t (&a)[4]) {
    a[0] = pack_bf16x2(c0[0], c0[1]);
    a[1] = pack_bf16x2(c0[2], c0[3]);
    a[2] = pack_bf16x2(c1[0], c1[1]);
    a[3] = pack_bf16x2(c1[2], c1[3]);
}
__device__ __forceinline__ void acc_to_a_split(const float (&c0)[4], const float (&c1)[4],
                                               uint32_t (&hi)[4], uint32_t (&lo)[4]) {
    float h[8], l[8];
    const float v[8] = {c0[0], c0[1], c0[2], c0[3], c1[0], c1[1], c1[2], c1[3]};
#pragma unroll
    for (int e = 0; e < 8; ++e) split_bf16(v[e], h[e], l[e]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        hi[e] = pack_bf16x2(h[2 * e], h[2 * e + 1]);
        lo[e] = pack_bf16x2(l[2 * e], l[2 * e + 1]);
    }
}

}  // namespace msync
}  // namespace gdn
