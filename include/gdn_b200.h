/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet prefill/decode library.
 *
 * The library (libgdn_b200.so) exposes the two hot paths of the gated delta
 * rule with a k-last fp32 recurrent state:
 *
 *   S_t = alpha_t * S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T,
 *   o_t = scale * S_t q_t,
 *   alpha = exp(-exp(A_log) * softplus(a + dt_bias)),  beta = sigmoid(b),
 *
 * with q/k heads shared by Hv/Hq consecutive v-heads (GVA).
 *
 * All tensor arguments are raw DEVICE pointers to contiguous row-major
 * buffers; no framework types cross this boundary.  Every entry point is
 * asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream) and
 * returns GDN_OK or a negative status; gdn_last_error() gives the message of
 * the calling thread's last failure.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define GDN_OK 0
#define GDN_ERR_INVALID_ARGUMENT (-1) /* shape, dtype, pointer or alignment error */
#define GDN_ERR_UNSUPPORTED (-2)      /* valid but not implemented (e.g. head size) */
#define GDN_ERR_CUDA (-3)             /* a CUDA runtime/driver call failed */
#define GDN_ERR_DEVICE_TIMEOUT (-4)   /* a kernel gave up on a bounded barrier wait */

/* Element type codes for the gate inputs (a, b) and parameters (A_log, dt_bias). */
#define GDN_DTYPE_F32 0
#define GDN_DTYPE_BF16 1

/* Option bits for gdn_prefill_flags() / gdn_decode_flags(). */
#define GDN_FLAG_QK_L2NORM 1   /* L2-normalise every q and k head vector first (see below) */

/* Prefill kernel choice for gdn_prefill_ex(). */
#define GDN_PREFILL_AUTO 0      /* see gdn_prefill_resolve() */
#define GDN_PREFILL_CHUNKED 1   /* chunked (C=64) WY/UT kernel on the tensor cores (mma.sync) */
#define GDN_PREFILL_RECURRENT 2 /* token-serial CUDA-core kernel */
#define GDN_PREFILL_TCGEN05 3   /* chunked (C=64) kernel on tcgen05 + TMEM + TMA; T >= 64 */

/*
 * Varlen chunked prefill.
 *
 * Replaces the reference entry point
 *   kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
 *   -> (output, new_state)                     solution/triton/kernel.py:416-489
 * whose outputs the caller now passes in (destination-passing style, the
 * convention of scripts/replay_first_workload.py:113-116).
 *
 *   q, k        bf16 [T, Hq, D]          (Hk == Hq)
 *   v           bf16 [T, Hv, D]
 *   state       fp32 [N, Hv, D, D] k-last ([.., V, K]) or NULL for a zero state
 *   A_log       [Hv]      (param_dtype)
 *   a, b        [T, Hv]   (gate_dtype)
 *   dt_bias     [Hv]      (param_dtype)
 *   cu_seqlens  int32 [N+1], non-decreasing, cu_seqlens[0] = 0, cu_seqlens[N] = T
 *   scale       0 selects 1/sqrt(D) (solution/triton/kernel.py:438-439)
 *   output      bf16 [T, Hv, D]
 *   new_state   fp32 [N, Hv, D, D]; must not overlap `state`.  A sequence of
 *               length 0 gets a zero new state (solution/gdn_baseline_torch.py:61-62).
 *
 * Requirements: D == 128, Hv % Hq == 0, 16-byte aligned q/k/v/output/state
 * pointers.  cu_seqlens is read on the device; entries outside [0, T] or
 * decreasing are a caller error, checked by the kernels themselves (no host
 * synchronization): they clamp such entries so they never read or write out of
 * bounds, and record the error for gdn_device_status().
 */
GDN_API int gdn_prefill(const void *q, const void *k, const void *v, const float *state,
                const void *A_log, const void *a, const void *dt_bias, const void *b,
                const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                int num_qk_heads, int num_v_heads, int head_size, float scale,
                int gate_dtype, int param_dtype, void *output, float *new_state,
                void *stream);

/* gdn_prefill with an explicit kernel choice (GDN_PREFILL_*).  Same contract. */
GDN_API int gdn_prefill_ex(const void *q, const void *k, const void *v, const float *state,
                   const void *A_log, const void *a, const void *dt_bias, const void *b,
                   const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                   int num_qk_heads, int num_v_heads, int head_size, float scale,
                   int gate_dtype, int param_dtype, void *output, float *new_state,
                   int method, void *stream);

/*
 * gdn_prefill_ex with option bits.  GDN_FLAG_QK_L2NORM replaces every 128-element head
 * vector x of q and k by bf16(x / sqrt(sum(x^2) + 1e-6)), computed in fp32 from the
 * bf16 inputs -- the L2 normalisation Gated DeltaNet layers apply before the
 * recurrence, rounded to bf16 as a normalisation layer would emit it -- before the
 * prefill runs (a pre-pass into scratch from the library's memory pool, since the
 * tensor-core kernels read q and k straight into their operand tiles).  The reference
 * never normalises (its benchmark inputs arrive normalised), so gdn_prefill and
 * gdn_prefill_ex run with no flags.  No counterpart in the reference.
 */
GDN_API int gdn_prefill_flags(const void *q, const void *k, const void *v, const float *state,
                      const void *A_log, const void *a, const void *dt_bias, const void *b,
                      const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                      int num_qk_heads, int num_v_heads, int head_size, float scale,
                      int gate_dtype, int param_dtype, void *output, float *new_state,
                      int method, int flags, void *stream);

/*
 * gdn_prefill_flags with the gate inputs a and b read straight from a wider tensor, such
 * as the output of the projection GEMM that produces them (a Gated DeltaNet layer's fused
 * projection emits [T, ...] rows holding a and b side by side): token t's gate inputs for
 * v-head h are a[t * a_row_stride + h] and b[t * b_row_stride + h].  Row strides are in
 * elements; 0 means num_v_heads (packed [T, Hv]), otherwise they must be >= num_v_heads.
 * No copy of a or b is made.  No counterpart in the reference (its entry points take
 * packed tensors and make them contiguous, solution/triton/kernel.py:452-453).
 */
GDN_API int gdn_prefill_strided(const void *q, const void *k, const void *v, const float *state,
                        const void *A_log, const void *a, const void *dt_bias, const void *b,
                        const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                        int num_qk_heads, int num_v_heads, int head_size, float scale,
                        int gate_dtype, int param_dtype, void *output, float *new_state,
                        int64_t a_row_stride, int64_t b_row_stride, int method, int flags,
                        void *stream);

/*
 * gdn_prefill_ex with a caller-provided workspace (no allocation inside the call).
 *
 * The GDN_PREFILL_TCGEN05 kernel computes each chunk's gates and T = (I + A)^-1 for
 * all chunks at once into a workspace before it runs the chains; gdn_prefill and
 * gdn_prefill_ex take that workspace from a library-owned stream-ordered memory pool,
 * this entry point takes it from the caller.  `workspace` must be 256-byte aligned
 * and hold gdn_prefill_workspace_size() bytes; other methods ignore it.  The
 * workspace must not be reused by other work until the call's stream reaches it.
 * The chains run on the caller's stream alone and in sequence order (the pooled entry
 * points may split off the last partial wave onto a second stream and rank the
 * sequences longest first; the results are the same bits).
 * No counterpart in the reference (its Triton kernel keeps no workspace).
 */
GDN_API int gdn_prefill_ws(const void *q, const void *k, const void *v, const float *state,
                   const void *A_log, const void *a, const void *dt_bias, const void *b,
                   const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                   int num_qk_heads, int num_v_heads, int head_size, float scale,
                   int gate_dtype, int param_dtype, void *output, float *new_state,
                   int method, void *workspace, size_t workspace_bytes, void *stream);

/*
 * gdn_prefill on the GDN_PREFILL_TCGEN05 kernel without any device allocation: its
 * per-chunk workspace is a fixed 64 MiB device array inside this library.  For callers
 * that must not allocate while serving (all device memory reserved by their own pools,
 * no driver allocation allowed on a latency-critical path, or memory accounting that
 * forbids allocations outside their allocator).  Same arguments and contract as
 * gdn_prefill; additionally requires
 *   (ceil(total_tokens / 64) + num_seqs) * num_v_heads * 41984 <= 64 MiB
 * (e.g. 2560 tokens in up to 9 sequences with 32 v-heads) and total_tokens >= 64;
 * larger calls return GDN_ERR_INVALID_ARGUMENT before any launch.  The first call on
 * each device resolves the array's address (cudaGetSymbolAddress with that device
 * current); make that first call before any stream capture that would include it.
 * There is one array per device: calls whose executions overlap on the device (other
 * streams, other host threads) race on it.
 * No counterpart in the reference (its Triton kernel keeps no workspace).
 */
GDN_API int gdn_prefill_noalloc(const void *q, const void *k, const void *v, const float *state,
                        const void *A_log, const void *a, const void *dt_bias, const void *b,
                        const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                        int num_qk_heads, int num_v_heads, int head_size, float scale,
                        int gate_dtype, int param_dtype, void *output, float *new_state,
                        void *stream);

/*
 * Gated RMSNorm of the recurrence output, in place:
 *   output <- bf16(output / sqrt(mean(output^2) + eps) * weight * silu(gate))
 * over every 128-element head vector (num_vectors = tokens * v-heads), in fp32 from
 * the bf16 output and gate (the reciprocal square root and the sigmoid of silu use the
 * hardware approximations: a few units of 2^-11 relative, below the bf16 rounding of the
 * result).  Gated DeltaNet layers apply it between the recurrence
 * and the output projection; call it on the output of gdn_prefill* / gdn_decode* on
 * the same stream.
 *   output   bf16 [num_vectors, head_size], 16-byte aligned (read and written)
 *   gate     bf16 [num_vectors, head_size], 16-byte aligned
 *   weight   [head_size] (weight_dtype: GDN_DTYPE_F32 or GDN_DTYPE_BF16)
 * Requirements: head_size == 128.  No counterpart in the reference (its entry points
 * return the ungated output).
 */
GDN_API int gdn_output_gate(void *output, const void *gate, const void *weight, int weight_dtype,
                    int64_t num_vectors, int head_size, float eps, void *stream);

/* gdn_prefill_flags followed by gdn_output_gate on the output, in one call (gate:
 * bf16 [T, Hv, D], 16-byte aligned; norm_weight [D] in norm_weight_dtype).
 * Bit-identical to the two calls.  On GDN_PREFILL_TCGEN05 the gating is applied in the
 * chains' output stores (the output is written once); the other methods run the
 * gdn_output_gate pass after the prefill.  No counterpart in the reference. */
GDN_API int gdn_prefill_gated(const void *q, const void *k, const void *v, const float *state,
                      const void *A_log, const void *a, const void *dt_bias, const void *b,
                      const int32_t *cu_seqlens, int64_t num_seqs, int64_t total_tokens,
                      int num_qk_heads, int num_v_heads, int head_size, float scale,
                      int gate_dtype, int param_dtype, void *output, float *new_state,
                      const void *out_gate, const void *norm_weight, int norm_weight_dtype, float eps,
                      int method, int flags, void *stream);

/* The prefill kernel (GDN_PREFILL_*) a call with `method` runs for `total_tokens` packed
 * tokens in `num_seqs` sequences on the current device: AUTO resolves to RECURRENT for
 * at most 32 tokens or fewer than 4 tokens per sequence, else to TCGEN05 from 256
 * tokens, else CHUNKED; other values are returned unchanged.  No counterpart in the
 * reference. */
GDN_API int gdn_prefill_resolve(int64_t total_tokens, int64_t num_seqs, int method);

/* Kernel launches of one tcgen05 prefill through the pooled-workspace entry points
 * (gdn_prefill, gdn_prefill_ex, gdn_prefill_flags, gdn_prefill_strided, gdn_prefill_gated)
 * on a device with `num_sms` SMs: 2 (chunk prep, chains), or 4
 * when the last partial wave of (sequence, v-head) chains is split onto the library's
 * second stream (more chains than SMs, chains mod SMs > 0 and a whole number of prep
 * CTAs); plus 1 when there are 2 to 65,536 sequences and more chains than SMs: a kernel
 * that ranks the sequences longest first on the device, so the chains of the longest
 * sequences start first (the results do not depend on the order).  0 for invalid
 * shapes.  Host arithmetic only.  No counterpart in the reference. */
GDN_API int gdn_prefill_tc_launches(int64_t num_seqs, int num_qk_heads, int num_v_heads, int num_sms);

/* Workspace bytes gdn_prefill_ws needs for GDN_PREFILL_TCGEN05:
 * (ceil(total_tokens / 64) + num_seqs) * num_v_heads * 41984.  No counterpart in the reference. */
GDN_API size_t gdn_prefill_workspace_size(int64_t num_seqs, int64_t total_tokens, int num_v_heads);

/*
 * Single-token decode.
 *
 * Replaces the reference entry point
 *   kernel_decode(q, k, v, state, A_log, a, dt_bias, b, scale)
 *   -> (output, new_state)                     solution/triton/kernel.py:492-556
 *
 *   q, k        bf16 [B, 1, Hq, D]
 *   v           bf16 [B, 1, Hv, D]
 *   state       fp32 [B, Hv, D, D] k-last, or NULL for a zero state
 *   a, b        [B, 1, Hv] (gate_dtype);  A_log, dt_bias [Hv] (param_dtype)
 *   output      bf16 [B, 1, Hv, D]
 *   new_state   fp32 [B, Hv, D, D]; may be the same pointer as `state` (in-place
 *               update: every element is read before it is written, by the same
 *               thread), but must not partially overlap it.
 *
 * Requirements: D == 128, Hv % Hq == 0, 16-byte aligned q/k/v/state/new_state.
 */
GDN_API int gdn_decode(const void *q, const void *k, const void *v, const float *state,
               const void *A_log, const void *a, const void *dt_bias, const void *b,
               int64_t batch, int num_qk_heads, int num_v_heads, int head_size,
               float scale, int gate_dtype, int param_dtype, void *output,
               float *new_state, void *stream);

/* gdn_decode with option bits.  GDN_FLAG_QK_L2NORM: q and k are L2-normalised inside
 * the decode kernel, with the same arithmetic as gdn_prefill_flags (so a normalised
 * prefill followed by normalised decode steps continues the same recurrence).  No
 * counterpart in the reference. */
GDN_API int gdn_decode_flags(const void *q, const void *k, const void *v, const float *state,
                     const void *A_log, const void *a, const void *dt_bias, const void *b,
                     int64_t batch, int num_qk_heads, int num_v_heads, int head_size,
                     float scale, int gate_dtype, int param_dtype, void *output,
                     float *new_state, int flags, void *stream);

/* gdn_decode_flags with the gate inputs read as a[s * a_row_stride + h], b[s * b_row_stride
 * + h] for sequence s (elements; 0 = num_v_heads; otherwise >= num_v_heads), straight from a
 * wider projection output, without a copy.  No counterpart in the reference. */
GDN_API int gdn_decode_strided(const void *q, const void *k, const void *v, const float *state,
                       const void *A_log, const void *a, const void *dt_bias, const void *b,
                       int64_t batch, int num_qk_heads, int num_v_heads, int head_size,
                       float scale, int gate_dtype, int param_dtype, void *output,
                       float *new_state, int64_t a_row_stride, int64_t b_row_stride, int flags,
                       void *stream);

/*
 * Synchronizes `stream` and reports the library's device status word since the last
 * call (the word is then cleared):
 *   GDN_ERR_DEVICE_TIMEOUT    a tcgen05 prefill CTA gave up on a bounded barrier wait
 *                             (the kernels never spin unboundedly: a wait that runs out
 *                             records its site, the CTA waits for its own copies and MMAs
 *                             in flight, frees its tensor memory and exits);
 *   GDN_ERR_INVALID_ARGUMENT  a prefill read a cu_seqlens that is not an offsets array over
 *                             [0, total_tokens] (checked on the device, where cu_seqlens
 *                             lives, so a call never synchronizes to check it on the host;
 *                             the kernels clamp such entries and never access memory out of
 *                             bounds, but the affected sequences' results are meaningless).
 * No counterpart in the reference (its Triton kernels have no device-side waits and
 * its entry points do no validation).
 */
GDN_API int gdn_device_status(void *stream);

/*
 * Limit, in nanoseconds, of every bounded device-side wait of the tcgen05 prefill
 * chains launched after this call (process-wide; 0 restores the default of 2 s).
 * Returns the previous setting (0 = default).  A serving process can lower it to
 * detect a stalled kernel sooner; a limit below a chunk's normal latency makes
 * healthy calls give up (gdn_device_status then reports GDN_ERR_DEVICE_TIMEOUT).
 * No counterpart in the reference.
 */
GDN_API uint64_t gdn_set_wait_limit_ns(uint64_t ns);

/* Message describing the calling thread's most recent failed call ("" if none). */
GDN_API const char *gdn_last_error(void);

/* Library version string, e.g. "gdn_b200 0.1.0 sm_100a". */
GDN_API const char *gdn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
