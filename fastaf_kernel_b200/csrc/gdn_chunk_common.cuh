// gdn_chunk_common.cuh -- pieces of the chunked (C = 64) prefill shared by its kernels:
// bf16 hi/lo splitting, swizzled shared-memory tile addressing, and the blocked
// 64x64 unit-lower-triangular inverse.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace gdn {

// x = hi + lo with hi = bf16(x) and lo = bf16(x - hi): ~16 significant bits in two bf16.
__device__ __forceinline__ void split_bf16(float x, float &hi, float &lo) {
    hi = __bfloat162float(__float2bfloat16_rn(x));
    lo = x - hi;
}

// The same split for two values at once, packed (a in bits 0-15): hi = bf16(a, b)
// rounded to nearest even, lo = bf16 of the exact fp32 remainders.
// Two fp32 lanes in one 64-bit register for sm_100's packed f32x2 arithmetic: one
// instruction does two IEEE round-to-nearest operations, with the results of two scalar ones.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unf2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t sub_f2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul_f2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ void split2_bf16(float a, float b, uint32_t &hi, uint32_t &lo) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    hi = *reinterpret_cast<uint32_t *>(&h);
    __nv_bfloat162 l = __floats2bfloat162_rn(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
    lo = *reinterpret_cast<uint32_t *>(&l);
}
// The same split with the two remainders in one packed subtraction (identical results).
__device__ __forceinline__ void split2_bf16_f2(float a, float b, uint32_t &hi, uint32_t &lo) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    hi = *reinterpret_cast<uint32_t *>(&h);
    float la, lb;
    unf2(sub_f2(f2(a, b), f2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u))), la, lb);
    __nv_bfloat162 l = __floats2bfloat162_rn(la, lb);
    lo = *reinterpret_cast<uint32_t *>(&l);
}

// Byte offset of element (row, col) of a bf16 tile whose rows are `kRowBytes`
// long (128 or 256), with the 16-byte chunk index XOR-ed by (row & 7): eight
// consecutive rows at the same logical chunk land in eight different banks, so
// ldmatrix reads of 8x8 blocks are conflict-free.
template <int kRowBytes>
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t col) {
    return row * kRowBytes + ((((col >> 3) ^ (row & 7u))) << 4) + (col & 7u) * 2u;
}

// (I + A)^-1 for a 64x64 strictly-lower A (fp32, row-major, row stride LD): the
// 16x16 diagonal blocks by forward substitution, then the off-diagonal blocks
// block-diagonal by block-diagonal as T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj.
// Only the lower triangle (j <= i) of Tm (same stride) is written.  An odd LD
// (65) keeps row-per-thread accesses free of bank conflicts.  All `nthreads`
// threads of the block must call it; it synchronizes the block internally.
template <int nthreads, int LD>
__device__ __forceinline__ void solve_unit_lower(const float *A, float *Tm, float *scr) {
    const int tid = threadIdx.x;
    if (tid < 64) {
        // Thread (block o, column c) solves column c of the diagonal block's inverse;
        // two partial sums halve the dependent FMA chain of each row.
        const int o = (tid >> 4) * 16, c = tid & 15;
        const float *Ab = A + o * LD + o;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float a0 = (r == c) ? 1.0f : 0.0f, a1 = 0.0f;
#pragma unroll
            for (int j = 0; j < r; ++j) {
                if (j & 1) a1 = fmaf(-Ab[r * LD + j], x[j], a1);
                else a0 = fmaf(-Ab[r * LD + j], x[j], a0);
            }
            x[r] = a0 + a1;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) Tm[(o + r) * LD + o + c] = x[r];
    }
    __syncthreads();
    for (int d = 1; d < 4; ++d) {
        const int nblk = 4 - d;
        for (int e = tid; e < nblk * 256; e += nthreads) {
            const int bi = d + (e >> 8), bj = bi - d, r = (e & 255) >> 4, cc = e & 15;
            float acc = 0.0f;
            for (int bk = bj; bk < bi; ++bk) {
                const float *ar = A + (16 * bi + r) * LD + 16 * bk;
                const float *tc = Tm + (16 * bk) * LD + 16 * bj + cc;
#pragma unroll
                for (int kk = 0; kk < 16; ++kk) acc = fmaf(ar[kk], tc[kk * LD], acc);
            }
            scr[e] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nblk * 256; e += nthreads) {
            const int bi = d + (e >> 8), bj = bi - d, r = (e & 255) >> 4, cc = e & 15;
            const float *tr = Tm + (16 * bi + r) * LD + 16 * bi;
            const float *m = scr + (e & ~255) + cc;
            float acc = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) acc = fmaf(tr[kk], m[kk * 16], acc);
            Tm[(16 * bi + r) * LD + 16 * bj + cc] = -acc;
        }
        __syncthreads();
    }
}

}  // namespace gdn
