// gdn_launch.h -- internal launch interface between the C ABI (gdn_api.cu) and
// the kernels.  Arguments are already validated when these are called.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

struct DecodeArgs {
    const void *q, *k, *v;       // bf16 [B, Hq|Hv, D]
    const float *state;          // fp32 [B, Hv, D, D] or nullptr
    const void *A_log, *a, *dt_bias, *b;
    int64_t batch;
    int Hq, Hv;
    float scale;
    int gate_dtype, param_dtype;
    void *out;                   // bf16 [B, Hv, D]
    float *new_state;            // may equal state
    int qk_l2norm;               // 1: q, k <- bf16(x / sqrt(sum x^2 + 1e-6)) inside the kernel
    // Elements between the gate inputs of consecutive sequences in a and b (Hv when packed;
    // larger for views into a wider projection output).  0: Hv.
    int64_t a_stride = 0, b_stride = 0;
};

struct PrefillArgs {
    const void *q, *k, *v;       // bf16 [T, Hq|Hv, D]
    const float *state;          // fp32 [N, Hv, D, D] or nullptr
    const void *A_log, *a, *dt_bias, *b;
    const int32_t *cu_seqlens;   // [N+1], device
    int64_t num_seqs, total_tokens;
    int Hq, Hv;
    float scale;
    int gate_dtype, param_dtype;
    void *out;                   // bf16 [T, Hv, D]
    float *new_state;            // fp32 [N, Hv, D, D]
    // Optional gated RMSNorm of the output (gate == nullptr: none): bf16 [T, Hv, D] gate,
    // [D] weight (dtype code), eps; applied by a pass after the prefill kernels.
    const void *out_gate = nullptr;
    const void *norm_w = nullptr;
    int norm_w_dtype = 0;
    float norm_eps = 0.0f;
    // The device status word on this device (device_status_word()), where the kernels
    // record a malformed cu_seqlens; nullptr: no check.
    int *status = nullptr;
    // Elements between the gate inputs of consecutive tokens in a and b (Hv when packed;
    // larger for views into a wider projection output).  0: Hv.
    int64_t a_stride = 0, b_stride = 0;
};

// Set the message gdn_last_error() returns on this thread.
void set_last_error(const char *msg);

cudaError_t launch_decode(const DecodeArgs &p, cudaStream_t stream);
// o <- bf16(o / sqrt(mean(o^2) + eps) * w * silu(z)) per 128-element vector, in place.
cudaError_t launch_output_gate(void *o, const void *z, const void *w, int w_dtype, int64_t vectors, float eps,
                               cudaStream_t stream);
// qn, kn <- bf16(x / sqrt(sum x^2 + 1e-6)) for every 128-element head vector of q, k
// ([rows][128] bf16, rows = tokens * heads); the same arithmetic as the decode kernel's.
cudaError_t launch_qk_l2norm(const void *q, const void *k, int64_t rows, void *qn, void *kn,
                             cudaStream_t stream);
cudaError_t launch_prefill_recurrent(const PrefillArgs &p, cudaStream_t stream);
cudaError_t launch_prefill_chunked(const PrefillArgs &p, cudaStream_t stream);
bool prefill_chunked_supported(const PrefillArgs &p);
// tcgen05 prefill: per-chunk prep (gdn_chunk_prep.cu) into `workspace` of
// prefill_tc_workspace_bytes() bytes (256-byte aligned), then the chain kernel.
// With `overlap`, a call of more chains than the device has SMs whose last partial wave
// would leave SMs idle is split in two: the last (chains mod SMs) chains -- prep and
// chain kernels -- on a library-owned high-priority stream, the rest on `stream`, so the
// short group's chains run while the rest is being prepped (fork and join through
// events; same kernels, same results).
// With p.out_gate set, the chains' output stores apply the gated RMSNorm themselves (the
// result equals the prefill followed by launch_output_gate bit for bit).
// With `order` (room for num_seqs int32), a call of more chains than SMs first ranks its
// sequences longest first on the device (launch_chain_order) and the chain kernel takes
// them in that order, so the block scheduler starts the longest chains first.  Only the
// sequences whose chains all stay on `stream` are ranked; the chunk prep, which finishes
// before the chains on its stream start, covers the same sequences in index order.
cudaError_t launch_prefill_tc(const PrefillArgs &p, void *workspace, cudaStream_t stream, bool overlap = false,
                              int32_t *order = nullptr);
// order[r] for r < ranked = the sequence of rank r among sequences [0, ranked), ranked by
// clamped length, longest first, ties by index; order[r] = r for ranked <= r < num_seqs.
// A permutation of [0, num_seqs) whatever cu_seqlens holds.
cudaError_t launch_chain_order(const int32_t *cu_seqlens, int64_t num_seqs, int64_t ranked,
                               int64_t total_tokens, int32_t *order, cudaStream_t stream);
// Whether launch_prefill_tc ranks the sequences of a call (more than one sequence and
// more chains than the device's SMs).
bool prefill_tc_orders_chains(int64_t num_seqs, int Hv, int sms);
// Chains launch_prefill_tc puts on the overlap stream for `chains` chains on `sms` SMs
// (0: no split): chains mod sms when there are more chains than SMs and that tail is a
// whole number of prep CTAs (heads_per_prep_cta v-heads each).
int64_t prefill_tc_overlap_tail(int64_t chains, int sms, int heads_per_prep_cta);
bool prefill_tc_supported(const PrefillArgs &p);
size_t prefill_tc_workspace_bytes(const PrefillArgs &p);
// Prep of the chains (sequence-major (sequence, v-head) indices) [chain_begin, chain_end)
// (chain_end < 0: to the last chain); both multiples of prep_heads_per_cta(p).
cudaError_t launch_chunk_prep(const PrefillArgs &p, uint8_t *ws_T, __nv_bfloat16 *ws_P, float *ws_g,
                              cudaStream_t stream, int64_t chain_begin = 0, int64_t chain_end = -1);
int prep_heads_per_cta(const PrefillArgs &p);
// The device status word: 0, the site (1..99) of a bounded device wait of the tcgen05
// prefill that gave up, or kErrCuSeqlens.  read_device_status synchronizes `stream`.
cudaError_t read_device_status(cudaStream_t stream, int *code, bool clear);
// Its device address on the current device (looked up on every call, so it follows a
// new primary context), or nullptr when the lookup fails.
int *device_status_word();
// Limit of every bounded device wait of the tcgen05 chains, in ns (0: the default 2 s);
// returns the previous setting.
uint64_t set_wait_limit_ns(uint64_t ns);

}  // namespace gdn
