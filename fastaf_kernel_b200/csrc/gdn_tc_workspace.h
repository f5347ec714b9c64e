// gdn_tc_workspace.h -- layout of the per-chunk workspace the tcgen05 prefill
// shares between its two kernels (gdn_chunk_prep.cu writes, gdn_prefill_tc.cu reads).
//
// Chunk c of sequence n (tokens [s0 + 64c, s0 + 64c + 64) with s0 = cu_seqlens[n])
// owns the slot  floor(s0 / 64) + c + n.  Slots of consecutive chunks and of
// consecutive sequences never collide (a sequence of L tokens starting at s0 ends
// at or after slot floor(s0/64) + ceil(L/64) - 1 + n, and the next one starts at
// floor((s0 + L)/64) + n + 1 or later), and every slot is below ceil(T/64) + N,
// so the workspace is sized from T and N alone, without reading cu_seqlens.
//
// Three arrays, each indexed by unit = slot * Hv + v-head:
//   T tiles: T' = T diag(beta) and T'' = T diag(beta Gamma), T = (I + A)^-1 (zero above
//      the diagonal), each split into bf16 hi + lo: four bf16 [64][64] tiles in the
//      order T'hi, T'lo, T''hi, T''lo (32 KB);
//   P  bf16 [64][64], P[i][j] = exp(gamma_i - gamma_j) q_i.k_j for j <= i, zero above (8 KB);
//   gates: four fp32 [64] rows: beta, gamma * log2(e), Gamma = exp(gamma),
//      exp(gamma_63 - gamma) (1 KB).
// Every bf16 tile is stored exactly as the tensor core reads it from shared memory
// (K-major [i][j]): 128-byte rows with the 16-byte chunk index XOR-ed by (i & 7), so
// one bulk copy moves it into place.
// Padding tokens of a partial chunk have beta = 0 and log alpha = 0.
#pragma once

#include <stdint.h>

namespace gdn {

constexpr int64_t kTcTileBytes = 64 * 64 * 2;          // one bf16 [64][64] tile
constexpr int64_t kTcTBytes = 4 * kTcTileBytes;          // T'hi, T'lo, T''hi, T''lo
constexpr int64_t kTcPBytes = 64 * 64 * 2;
constexpr int64_t kTcGateBytes = 4 * 64 * 4;
constexpr int64_t kTcUnitBytes = kTcTBytes + kTcPBytes + kTcGateBytes;

__host__ __device__ inline int64_t tc_num_slots(int64_t total_tokens, int64_t num_seqs) {
    return (total_tokens + 63) / 64 + num_seqs;
}

__host__ __device__ inline int64_t tc_workspace_bytes(int64_t total_tokens, int64_t num_seqs, int Hv) {
    return tc_num_slots(total_tokens, num_seqs) * Hv * kTcUnitBytes;
}

__host__ __device__ inline int64_t tc_slot(int64_t s0, int c, int64_t n) {
    return s0 / 64 + c + n;
}

}  // namespace gdn
