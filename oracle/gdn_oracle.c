/*
 * CPU oracle for the Gated DeltaNet prefill/decode path -- TEST INFRASTRUCTURE.
 *
 * It is what the GPU results are compared against and the timed CPU baseline, never
 * the product: only the tests, the smoke check and bench.py's CPU legs load it.
 *
 * A plain-C, fp32, token-serial restatement of the reference's torch
 * implementation (solution/gdn_baseline_torch.py:12-91) with the head-count
 * asserts lifted.  Per (sequence, v-head) chain and per token t, for every
 * state row v of the k-last state S[v][k]:
 *
 *   g     = exp(-exp(A_log[h]) * softplus(a[t,h] + dt_bias[h]))   (:42-43)
 *   beta  = sigmoid(b[t,h])                                          (:44)
 *   S'    = g * S                                                    (:79)
 *   u[v]  = sum_k k[k] * S'[v][k]                                    (:80)
 *   vn[v] = beta * v[v] + (1 - beta) * u[v]                          (:81)
 *   S[v][k] = S'[v][k] - k[k]*u[v] + k[k]*vn[v]                      (:82-84)
 *   o[v]  = scale * sum_k q[k] * S[v][k]                             (:86-87)
 *
 * The v-head h reads q/k head h / (Hv/Hq) (repeat_interleave, :46-47).  A
 * sequence of length <= 0 leaves its new state at zero (:61-62).  Reductions
 * use 8 fixed partial sums, so results are deterministic but differ from
 * torch's BLAS summation order in the last bits.
 *
 * Chains are independent, so they run in parallel under OpenMP.
 *
 * qk_l2norm != 0 first replaces every q and k head vector x by
 * bf16(x / sqrt(sum x^2 + 1e-6)) (fp32 arithmetic) -- the library's optional L2
 * normalisation, which the reference does not have; with qk_l2norm == 0 the
 * functions follow the reference exactly.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                                           /* RNE */
    return (uint16_t)(u >> 16);
}

/* dtype codes shared with the product's C-ABI: 0 = fp32, 1 = bf16 */
static inline float load_scalar(const void *p, int64_t i, int dtype) {
    return dtype == 1 ? bf16_to_f32(((const uint16_t *)p)[i]) : ((const float *)p)[i];
}

/* torch.nn.functional.softplus with beta=1, threshold=20 */
static inline float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

static inline float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

static inline float dot8(const float *x, const float *y, int n) {
    float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; ++j) p[j] += x[i + j] * y[i + j];
    for (; i < n; ++i) p[i & 7] += x[i] * y[i];
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}

static void l2norm_bf16(float *x, int n) {
    const float inv = 1.0f / sqrtf(dot8(x, x, n) + 1e-6f);
    for (int i = 0; i < n; ++i) x[i] = bf16_to_f32(f32_to_bf16(x[i] * inv));
}

/*
 * q, k: bf16 [T, Hq, D]; v: bf16 [T, Hv, D]; a, b: [T, Hv] (gate_dtype);
 * A_log, dt_bias: [Hv] (param_dtype); state: fp32 [N, Hv, D, D] or NULL;
 * cu_seqlens: int32 [N+1]; out: bf16 [T, Hv, D]; new_state: fp32 [N, Hv, D, D].
 * Returns 0, or a negative code for bad arguments.
 */
int gdn_oracle_prefill(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                       const float *state, const void *A_log, const void *a,
                       const void *dt_bias, const void *b, const int32_t *cu_seqlens,
                       int64_t N, int64_t T, int Hq, int Hv, int D, float scale,
                       int gate_dtype, int param_dtype, uint16_t *out,
                       float *new_state, int num_threads, int qk_l2norm) {
    if (Hq <= 0 || Hv <= 0 || D <= 0 || D > 1024 || Hv % Hq != 0 || N < 0 || T < 0) return -1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)D);
    const int ratio = Hv / Hq;
    const int64_t chains = N * (int64_t)Hv;
    memset(new_state, 0, sizeof(float) * (size_t)N * Hv * D * D);
#pragma omp parallel num_threads(num_threads > 0 ? num_threads : 1)
    {
        float kf[1024], qf[1024];
#pragma omp for schedule(dynamic, 1)
            for (int64_t c = 0; c < chains; ++c) {
                const int64_t n = c / Hv;
                const int h = (int)(c % Hv);
                const int hq = h / ratio;
                const int64_t s0 = cu_seqlens[n], s1 = cu_seqlens[n + 1];
                if (s1 - s0 <= 0 || s0 < 0 || s1 > T) continue;
                float *S = new_state + ((size_t)n * Hv + h) * (size_t)D * D;
                if (state) memcpy(S, state + ((size_t)n * Hv + h) * (size_t)D * D,
                                  sizeof(float) * (size_t)D * D);
                const float expA = expf(load_scalar(A_log, h, param_dtype));
                const float dtb = load_scalar(dt_bias, h, param_dtype);
                for (int64_t t = s0; t < s1; ++t) {
                    const float g = expf(-expA * softplus_f(load_scalar(a, t * Hv + h, gate_dtype) + dtb));
                    const float beta = sigmoid_f(load_scalar(b, t * Hv + h, gate_dtype));
                    const uint16_t *kp = k + ((size_t)t * Hq + hq) * D;
                    const uint16_t *qp = q + ((size_t)t * Hq + hq) * D;
                    const uint16_t *vp = v + ((size_t)t * Hv + h) * D;
                    uint16_t *op = out + ((size_t)t * Hv + h) * D;
                    for (int i = 0; i < D; ++i) { kf[i] = bf16_to_f32(kp[i]); qf[i] = bf16_to_f32(qp[i]); }
                    if (qk_l2norm) { l2norm_bf16(kf, D); l2norm_bf16(qf, D); }
                    for (int r = 0; r < D; ++r) {
                        float *row = S + (size_t)r * D;
                        for (int i = 0; i < D; ++i) row[i] *= g;
                        const float u = dot8(kf, row, D);
                        const float vn = beta * bf16_to_f32(vp[r]) + (1.0f - beta) * u;
                        for (int i = 0; i < D; ++i) row[i] = (row[i] - kf[i] * u) + kf[i] * vn;
                        op[r] = f32_to_bf16(scale * dot8(qf, row, D));
                    }
                }
            }
    }
    return 0;
}

/* Decode: the same recurrence with one token per sequence.  Shapes
 * q, k [B, Hq, D], v [B, Hv, D], a, b [B, Hv]; state may equal new_state. */
int gdn_oracle_decode(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                      const float *state, const void *A_log, const void *a,
                      const void *dt_bias, const void *b, int64_t B, int Hq, int Hv,
                      int D, float scale, int gate_dtype, int param_dtype,
                      uint16_t *out, float *new_state, int num_threads, int qk_l2norm) {
    if (Hq <= 0 || Hv <= 0 || D <= 0 || D > 1024 || Hv % Hq != 0 || B < 0) return -1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)D);
    const int ratio = Hv / Hq;
    const int64_t chains = B * (int64_t)Hv;
#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1) schedule(static)
    for (int64_t c = 0; c < chains; ++c) {
        float kf[1024], qf[1024];
        const int64_t n = c / Hv;
        const int h = (int)(c % Hv);
        const int hq = h / ratio;
        float *S = new_state + ((size_t)n * Hv + h) * (size_t)D * D;
        if (state) {
            if (state != new_state)
                memcpy(S, state + ((size_t)n * Hv + h) * (size_t)D * D, sizeof(float) * (size_t)D * D);
        } else {
            memset(S, 0, sizeof(float) * (size_t)D * D);
        }
        const float expA = expf(load_scalar(A_log, h, param_dtype));
        const float dtb = load_scalar(dt_bias, h, param_dtype);
        const float g = expf(-expA * softplus_f(load_scalar(a, c, gate_dtype) + dtb));
        const float beta = sigmoid_f(load_scalar(b, c, gate_dtype));
        const uint16_t *kp = k + ((size_t)n * Hq + hq) * D;
        const uint16_t *qp = q + ((size_t)n * Hq + hq) * D;
        const uint16_t *vp = v + ((size_t)n * Hv + h) * D;
        uint16_t *op = out + ((size_t)n * Hv + h) * D;
        for (int i = 0; i < D; ++i) { kf[i] = bf16_to_f32(kp[i]); qf[i] = bf16_to_f32(qp[i]); }
        if (qk_l2norm) { l2norm_bf16(kf, D); l2norm_bf16(qf, D); }
        for (int r = 0; r < D; ++r) {
            float *row = S + (size_t)r * D;
            for (int i = 0; i < D; ++i) row[i] *= g;
            const float u = dot8(kf, row, D);
            const float vn = beta * bf16_to_f32(vp[r]) + (1.0f - beta) * u;
            for (int i = 0; i < D; ++i) row[i] = (row[i] - kf[i] * u) + kf[i] * vn;
            op[r] = f32_to_bf16(scale * dot8(qf, row, D));
        }
    }
    return 0;
}
