/*
 * CPU oracle for Affon's affine group-quantized matmul.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA library in
 * affon_b200/ is compared against; nothing in the product path links, loads or
 * calls it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may use the shared object built from it (oracle/_build/libaffon_oracle.so).
 *
 * It restates the reference's scalar CPU kernel, which is not vendored in the
 * reference tree (compute/src/backend/cpu/quantized_matmul.zig lives in the
 * separate `compute` checkout).  Its documented behaviour is followed:
 *
 *   docs/core/quantized-inference.md:59-67   packing and affine decode:
 *       word = packed[n, k / P], P = 32 / bits,
 *       q = (word >> ((k % P) * bits)) & ((1 << bits) - 1)   (low bits first),
 *       w = scales[n, k / group] * q + biases[n, k / group]
 *   docs/core/quantized-inference.md:114-128 numerics: scalar, single thread,
 *       bf16 widened to f32 before arithmetic, weight decoded inside the dot
 *       product, ordered f32 accumulation, no bf16 rounding of weights, no
 *       dequantised matrix.
 *   src/js/compute/program.ts:481-495 shape / dtype validation.
 *   src/support/compute_core_cyna.zig:29-45,1000-1032 C-ABI status codes
 *       (0 ok, 1 invalid shape; output untouched on error).
 *   test/parity/reference/check-cuda-quantized-general.py:71-78 float64
 *       reference (explicit unpack, repeat-interleaved parameters, x @ W^T).
 *
 * Build with -ffp-contract=off so that `s * q + b` and `acc + x * w` round
 * after every operation, as the reference's strict-float Zig does.
 *
 * Parity pin: the restatement is checked against every known-answer test the
 * reference holds for this path (test/e2e/program/operations/
 * quantized-matmul.test.ts, src/support/compute_core_cyna_smoke.zig:970-977),
 * the deterministic fixture of test/parity/fixtures/quantized_fixture.py over
 * all 268 CUDA catalog cells, and the 192 seeded general cases of
 * check-cuda-quantized-general.py (seed 20261105).  The fixtures and the
 * script that produced them from the reference's Python live in tests/golden/.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORACLE_F32 = 0, ORACLE_BF16 = 1 };

/* A logical rank-two view: element strides for rows / columns plus a byte
 * offset from the base pointer (docs/core/quantized-inference.md:51-52:
 * "logical indices are mapped through their element strides and byte
 * offsets"). */
typedef struct oracle_view {
    const void *base;
    int64_t row_stride;
    int64_t col_stride;
    int64_t byte_offset;
    int dtype; /* ORACLE_F32 / ORACLE_BF16; ignored for the u32 weights */
} oracle_view;

static inline float bf16_bits_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u); /* NaN stays NaN */
    uint32_t rounding = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + rounding) >> 16);
}

static inline float load_float(const oracle_view *v, int64_t r, int64_t c) {
    const char *p = (const char *)v->base + v->byte_offset;
    int64_t e = r * v->row_stride + c * v->col_stride;
    if (v->dtype == ORACLE_BF16) return bf16_bits_to_f32(((const uint16_t *)p)[e]);
    return ((const float *)p)[e];
}

static inline uint32_t load_word(const oracle_view *v, int64_t r, int64_t c) {
    const char *p = (const char *)v->base + v->byte_offset;
    return ((const uint32_t *)p)[r * v->row_stride + c * v->col_stride];
}

/* Shape rules of src/js/compute/program.ts:484-493 (returns 0 when valid). */
int affon_oracle_validate(int64_t M, int64_t N, int64_t K, int bits, int64_t group_size) {
    if (bits != 2 && bits != 4 && bits != 8) return 1;
    if (group_size <= 0) return 1;
    if (M <= 0 || N <= 0 || K <= 0) return 1;
    int64_t per_word = 32 / bits;
    if (K % per_word || K % group_size) return 1;
    return 0;
}

/* Decoded integer code q[n,k] (quantized-inference.md:59-61). */
static inline uint32_t code_at(const oracle_view *w, int64_t n, int64_t k, int bits) {
    int64_t per_word = 32 / bits;
    uint32_t word = load_word(w, n, k / per_word);
    uint32_t mask = (bits == 32) ? 0xffffffffu : ((1u << bits) - 1u);
    return (word >> ((k % per_word) * bits)) & mask;
}

/* Unpack every code of a logical [N, K] packed view into bytes; used by the
 * bit-exact code parity check. */
int affon_oracle_unpack(const uint32_t *packed, int64_t N, int64_t K, int bits, uint8_t *codes) {
    if (bits != 2 && bits != 4 && bits != 8) return 1;
    int64_t per_word = 32 / bits;
    if (N <= 0 || K <= 0 || K % per_word) return 1;
    oracle_view w = {packed, K / per_word, 1, 0, 0};
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) codes[n * K + k] = (uint8_t)code_at(&w, n, k, bits);
    return 0;
}

/* One output row range [n0, n1) of y = x . decode(W)^T with the reference's
 * scalar order: decode w = s*q + b in f32, then acc = acc + x*w in ascending k. */
static void qmm_rows_f32(const oracle_view *x, const oracle_view *w, const oracle_view *s,
                         const oracle_view *b, float *y, int64_t y_row_stride, int64_t M,
                         int64_t n0, int64_t n1, int64_t K, int bits, int64_t group) {
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = n0; n < n1; ++n) {
            float acc = 0.0f;
            for (int64_t k = 0; k < K; ++k) {
                int64_t g = k / group;
                float q = (float)code_at(w, n, k, bits);
                float scaled = load_float(s, n, g) * q;
                float weight = scaled + load_float(b, n, g);
                float product = load_float(x, m, k) * weight;
                acc = acc + product;
            }
            y[m * y_row_stride + n] = acc;
        }
    }
}

/* Generic strided entry (all four operands are views).  y is dense f32 [M,N].
 * Returns 0 on success, 1 on an invalid shape (y untouched). */
int affon_oracle_qmm_view_f32(const void *x, int64_t x_rs, int64_t x_cs, int64_t x_off, int x_dtype,
                              const uint32_t *w, int64_t w_rs, int64_t w_cs, int64_t w_off,
                              const void *s, int64_t s_rs, int64_t s_cs, int64_t s_off,
                              const void *b, int64_t b_rs, int64_t b_cs, int64_t b_off, int p_dtype,
                              float *y, int64_t M, int64_t N, int64_t K, int bits, int64_t group) {
    if (affon_oracle_validate(M, N, K, bits, group)) return 1;
    if ((x_dtype != ORACLE_F32 && x_dtype != ORACLE_BF16) || (p_dtype != ORACLE_F32 && p_dtype != ORACLE_BF16)) return 1;
    oracle_view xv = {x, x_rs, x_cs, x_off, x_dtype};
    oracle_view wv = {w, w_rs, w_cs, w_off, 0};
    oracle_view sv = {s, s_rs, s_cs, s_off, p_dtype};
    oracle_view bv = {b, b_rs, b_cs, b_off, p_dtype};
    qmm_rows_f32(&xv, &wv, &sv, &bv, y, N, M, 0, N, K, bits, group);
    return 0;
}

/* Float64 variant of the same contraction (error-bound reference, following
 * check-cuda-quantized-general.py:71-78). */
int affon_oracle_qmm_view_f64(const void *x, int64_t x_rs, int64_t x_cs, int64_t x_off, int x_dtype,
                              const uint32_t *w, int64_t w_rs, int64_t w_cs, int64_t w_off,
                              const void *s, int64_t s_rs, int64_t s_cs, int64_t s_off,
                              const void *b, int64_t b_rs, int64_t b_cs, int64_t b_off, int p_dtype,
                              double *y, int64_t M, int64_t N, int64_t K, int bits, int64_t group) {
    if (affon_oracle_validate(M, N, K, bits, group)) return 1;
    oracle_view xv = {x, x_rs, x_cs, x_off, x_dtype};
    oracle_view wv = {w, w_rs, w_cs, w_off, 0};
    oracle_view sv = {s, s_rs, s_cs, s_off, p_dtype};
    oracle_view bv = {b, b_rs, b_cs, b_off, p_dtype};
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                int64_t g = k / group;
                double wt = (double)load_float(&sv, n, g) * (double)code_at(&wv, n, k, bits) + (double)load_float(&bv, n, g);
                acc += (double)load_float(&xv, m, k) * wt;
            }
            y[m * N + n] = acc;
        }
    return 0;
}

/* Dense entry: x [M,K], w [N,K/P], s/b [N,K/group], y [M,N] f32 (the
 * reference result dtype, program.ts:494). */
int affon_oracle_qmm_dense_f32(const void *x, int x_dtype, const uint32_t *w, const void *s, const void *b,
                               int p_dtype, float *y, int64_t M, int64_t N, int64_t K, int bits, int64_t group) {
    if (affon_oracle_validate(M, N, K, bits, group)) return 1;
    int64_t per_word = 32 / bits;
    return affon_oracle_qmm_view_f32(x, K, 1, 0, x_dtype, w, K / per_word, 1, 0, s, K / group, 1, 0, b, K / group, 1, 0,
                                     p_dtype, y, M, N, K, bits, group);
}

typedef struct {
    oracle_view x, w, s, b;
    float *y;
    int64_t M, N, K, n0, n1, group;
    int bits;
} oracle_job;

static void *oracle_worker(void *arg) {
    oracle_job *j = (oracle_job *)arg;
    qmm_rows_f32(&j->x, &j->w, &j->s, &j->b, j->y, j->N, j->M, j->n0, j->n1, j->K, j->bits, j->group);
    return NULL;
}

/* Same arithmetic split over output columns on `threads` POSIX threads.  Each
 * output element keeps the single-thread order, so results are identical to
 * affon_oracle_qmm_dense_f32.  This is the all-core CPU baseline (a
 * restatement, not the reference's own threading, which defaults to one). */
int affon_oracle_qmm_dense_f32_mt(const void *x, int x_dtype, const uint32_t *w, const void *s, const void *b,
                                  int p_dtype, float *y, int64_t M, int64_t N, int64_t K, int bits, int64_t group,
                                  int threads) {
    if (affon_oracle_validate(M, N, K, bits, group)) return 1;
    if (threads < 1) threads = 1;
    if (threads > N) threads = (int)N;
    int64_t per_word = 32 / bits;
    oracle_job *jobs = (oracle_job *)calloc((size_t)threads, sizeof(oracle_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    if (!jobs || !tids) { free(jobs); free(tids); return 2; }
    int64_t chunk = (N + threads - 1) / threads;
    int launched = 0;
    for (int t = 0; t < threads; ++t) {
        oracle_job *j = &jobs[t];
        j->x = (oracle_view){x, K, 1, 0, x_dtype};
        j->w = (oracle_view){w, K / per_word, 1, 0, 0};
        j->s = (oracle_view){s, K / group, 1, 0, p_dtype};
        j->b = (oracle_view){b, K / group, 1, 0, p_dtype};
        j->y = y; j->M = M; j->N = N; j->K = K; j->bits = bits; j->group = group;
        j->n0 = t * chunk; j->n1 = (t + 1) * chunk < N ? (t + 1) * chunk : N;
        if (j->n0 >= j->n1) continue;
        if (pthread_create(&tids[t], NULL, oracle_worker, j) == 0) { ++launched; }
        else { oracle_worker(j); tids[t] = 0; }
    }
    for (int t = 0; t < threads; ++t)
        if (jobs[t].n0 < jobs[t].n1 && tids[t]) pthread_join(tids[t], NULL);
    free(jobs); free(tids);
    (void)launched;
    return 0;
}

/* The reference's C-ABI shape (src/support/compute_core_cyna.zig:29-45):
 * f32 activations and parameters, dense buffers with explicit element counts,
 * status 0 ok / 1 invalid shape, output untouched on error
 * (compute_core_cyna_smoke.zig:978-983). */
int affon_oracle_compute_core_run_quantized_matmul_f32(
    const float *activation, size_t activation_count, const uint32_t *weights, size_t weight_count,
    const float *scales, size_t scale_count, const float *biases, size_t bias_count, float *output,
    size_t output_count, size_t rows, size_t depth, size_t columns, size_t bits, size_t group_size) {
    if (rows == 0 || depth == 0 || columns == 0 || group_size == 0 || (bits != 2 && bits != 4 && bits != 8)) return 1;
    size_t per_word = 32 / bits;
    if (depth % per_word || depth % group_size) return 1;
    if (rows > (size_t)INT64_MAX / depth || columns > (size_t)INT64_MAX / depth || rows > (size_t)INT64_MAX / columns) return 1;
    if (activation_count != rows * depth || weight_count != columns * (depth / per_word) ||
        scale_count != columns * (depth / group_size) || bias_count != columns * (depth / group_size) ||
        output_count != rows * columns)
        return 1;
    return affon_oracle_qmm_dense_f32(activation, ORACLE_F32, weights, scales, biases, ORACLE_F32, output,
                                      (int64_t)rows, (int64_t)columns, (int64_t)depth, (int)bits, (int64_t)group_size);
}

/* Round an f32 array to bf16 bit patterns (RNE), for bf16-output parity. */
void affon_oracle_f32_to_bf16(const float *in, uint16_t *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rne(in[i]);
}
