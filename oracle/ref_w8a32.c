/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of czxichen/rust-ppocrv6's quantised recognition-head path, used
 * by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs as
 * the CHECKER and the CPU baseline. Nothing in the shipped library links, loads or calls
 * this file; the product path (rust_ppocrv6_b200/csrc) fails loudly without its CUDA build.
 *
 * The reference is Rust (edition 2024) and cannot be compiled in this image (no cargo or
 * rustc), so this file restates it function by function. Every AVX2 function uses the
 * same intrinsics in the same order as the Rust source, so with -ffp-contract=off (Rust
 * never contracts a*b+c into an FMA) and without -ffast-math the results are bitwise what
 * the reference's own x86_64 build computes. The one libm call on the path (f32::exp in
 * the softmax tail, glibc expf on Linux) is the same libm call here.
 *
 * Parity pin: tests/test_oracle_pins.py re-runs the reference's own unit tests for this
 * path (matmul.rs, softmax.rs, ctc.rs test modules) against this file, with the same
 * generators and tolerances, plus a pack check against an independent numpy restatement
 * on a slice of the real PP-OCRv6 small-rec head weights (tests/golden/).
 *
 * Reference file:line citations are paths inside the rust-ppocrv6 project.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_OK 0
#define OR_ERR_ARG 1

/* ---------------------------------------------------------------- helpers */

/* f32::max (IEEE maxNum): a NaN operand yields the other operand. */
static inline float rust_fmax(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* f32::clamp(self, min, max): NaN stays NaN. */
static inline float rust_clamp(float v, float lo, float hi) {
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}

/* `v as i8`: saturating, NaN -> 0, truncation toward zero. */
static inline int8_t rust_as_i8(float v) {
    if (isnan(v)) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}

/* hsum256: src/ops/matmul.rs:899-910 (identical copy in src/ops/softmax.rs:302-312). */
__attribute__((target("avx2,fma"))) static inline float hsum256(__m256 v) {
    __m128 hi128 = _mm256_extractf128_ps(v, 1);
    __m128 lo128 = _mm256_castps256_ps128(v);
    __m128 sum128 = _mm_add_ps(lo128, hi128);
    __m128 hi64 = _mm_movehl_ps(sum128, sum128);
    __m128 sum64 = _mm_add_ps(sum128, hi64);
    __m128 hi32 = _mm_shuffle_ps(sum64, sum64, 1);
    return _mm_cvtss_f32(_mm_add_ss(sum64, hi32));
}

/* hmax256: src/ops/softmax.rs:289-300. */
__attribute__((target("avx2,fma"))) static inline float hmax256(__m256 v) {
    __m128 hi128 = _mm256_extractf128_ps(v, 1);
    __m128 lo128 = _mm256_castps256_ps128(v);
    __m128 max128 = _mm_max_ps(lo128, hi128);
    __m128 hi64 = _mm_movehl_ps(max128, max128);
    __m128 max64 = _mm_max_ps(max128, hi64);
    __m128 hi32 = _mm_shuffle_ps(max64, max64, 1);
    return _mm_cvtss_f32(_mm_max_ss(max64, hi32));
}

int oracle_cpu_has_avx2_fma(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
}

/* ------------------------------------------------------------------- pack */

/*
 * QuantizedWeight::from_f32_transposed — src/ops/matmul.rs:1173-1202.
 * w_t is the transposed head weight [n][k] (graph weight [k][n] transposed at load time,
 * src/engine/model.rs:565-605). Per row: max|w| folded from 0, scale = max/127 (or 1 when
 * max <= 1e-8), q = round(w * (1/scale)) clamped to [-127, 127].
 */
void oracle_pack(const float *w_t, int64_t n, int64_t k, int8_t *data, float *scales) {
    for (int64_t j = 0; j < n; j++) {
        const float *row = w_t + j * k;
        float max_abs = 0.0f;
        for (int64_t i = 0; i < k; i++) max_abs = rust_fmax(max_abs, fabsf(row[i]));
        float scale = max_abs > 1e-8f ? max_abs / 127.0f : 1.0f;
        float inv_scale = 1.0f / scale;
        scales[j] = scale;
        for (int64_t i = 0; i < k; i++) {
            float q = rust_clamp(roundf(row[i] * inv_scale), -127.0f, 127.0f);
            data[j * k + i] = rust_as_i8(q);
        }
    }
}

/* ------------------------------------------------------- projection (rows) */

/* avx2_dot_product_w8 — src/ops/matmul.rs:1473-1514. */
__attribute__((target("avx2,fma"))) static float avx2_dot_product_w8(const float *a, const int8_t *w8,
                                                                        int64_t n) {
    int64_t i = 0;
    __m256 v0 = _mm256_setzero_ps();
    __m256 v1 = _mm256_setzero_ps();
    while (i + 16 <= n) {
        __m256 va0 = _mm256_loadu_ps(a + i);
        __m256 va1 = _mm256_loadu_ps(a + i + 8);
        __m128i b_i8_0 = _mm_loadl_epi64((const __m128i *)(w8 + i));
        __m256 b_f32_0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b_i8_0));
        v0 = _mm256_fmadd_ps(va0, b_f32_0, v0);
        __m128i b_i8_1 = _mm_loadl_epi64((const __m128i *)(w8 + i + 8));
        __m256 b_f32_1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b_i8_1));
        v1 = _mm256_fmadd_ps(va1, b_f32_1, v1);
        i += 16;
    }
    v0 = _mm256_add_ps(v0, v1);
    while (i + 8 <= n) {
        __m256 va = _mm256_loadu_ps(a + i);
        __m128i b_i8 = _mm_loadl_epi64((const __m128i *)(w8 + i));
        __m256 b_f32 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b_i8));
        v0 = _mm256_fmadd_ps(va, b_f32, v0);
        i += 8;
    }
    float sum = hsum256(v0);
    while (i < n) {
        sum += a[i] * (float)w8[i];
        i++;
    }
    return sum;
}

/*
 * compute_quantized_b_cols_avx2 — src/ops/matmul.rs:1338-1443. Four columns at a time,
 * 8-wide K steps (cvtepi8_epi32 -> cvtepi32_ps -> FMA), hsum256, *scale, +bias; the
 * col_count % 4 tail columns go through avx2_dot_product_w8.
 */
__attribute__((target("avx2,fma"))) void oracle_cols_avx2(const float *a_row, const int8_t *w, const float *s,
                                                             const float *bias, float *out_chunk,
                                                             int64_t col_start, int64_t col_count, int64_t k) {
    int64_t c = 0;
    while (c + 4 <= col_count) {
        int64_t j0 = col_start + c, j1 = j0 + 1, j2 = j0 + 2, j3 = j0 + 3;
        const int8_t *w0 = w + j0 * k, *w1 = w + j1 * k, *w2 = w + j2 * k, *w3 = w + j3 * k;
        __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
        __m256 acc2 = _mm256_setzero_ps(), acc3 = _mm256_setzero_ps();
        int64_t i = 0;
        while (i + 8 <= k) {
            __m256 va = _mm256_loadu_ps(a_row + i);
            __m256 bf_0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(w0 + i))));
            acc0 = _mm256_fmadd_ps(va, bf_0, acc0);
            __m256 bf_1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(w1 + i))));
            acc1 = _mm256_fmadd_ps(va, bf_1, acc1);
            __m256 bf_2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(w2 + i))));
            acc2 = _mm256_fmadd_ps(va, bf_2, acc2);
            __m256 bf_3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(w3 + i))));
            acc3 = _mm256_fmadd_ps(va, bf_3, acc3);
            i += 8;
        }
        float sum0 = hsum256(acc0), sum1 = hsum256(acc1), sum2 = hsum256(acc2), sum3 = hsum256(acc3);
        while (i < k) {
            float a_val = a_row[i];
            sum0 += a_val * (float)w0[i];
            sum1 += a_val * (float)w1[i];
            sum2 += a_val * (float)w2[i];
            sum3 += a_val * (float)w3[i];
            i++;
        }
        float dot0 = sum0 * s[j0], dot1 = sum1 * s[j1], dot2 = sum2 * s[j2], dot3 = sum3 * s[j3];
        if (bias) {
            out_chunk[c] = dot0 + bias[j0];
            out_chunk[c + 1] = dot1 + bias[j1];
            out_chunk[c + 2] = dot2 + bias[j2];
            out_chunk[c + 3] = dot3 + bias[j3];
        } else {
            out_chunk[c] = dot0;
            out_chunk[c + 1] = dot1;
            out_chunk[c + 2] = dot2;
            out_chunk[c + 3] = dot3;
        }
        c += 4;
    }
    while (c < col_count) {
        int64_t j = col_start + c;
        float dot = avx2_dot_product_w8(a_row, w + j * k, k) * s[j];
        out_chunk[c] = bias ? dot + bias[j] : dot;
        c++;
    }
}

/* compute_quantized_b_cols_scalar — src/ops/matmul.rs:1445-1471 (sequential sum). */
void oracle_cols_scalar(const float *a_row, const int8_t *w, const float *s, const float *bias,
                        float *out_chunk, int64_t col_start, int64_t col_count, int64_t k) {
    for (int64_t c = 0; c < col_count; c++) {
        int64_t j = col_start + c;
        const int8_t *w_col = w + j * k;
        float acc = -0.0f;
        for (int64_t i = 0; i < k; i++) acc = acc + a_row[i] * (float)w_col[i];
        float dot = acc * s[j];
        out_chunk[c] = bias ? dot + bias[j] : dot;
    }
}

/*
 * matmul_quantized_b — src/ops/matmul.rs:1204-1336, restricted to the serial per-row
 * schedule (`run_row`, :1274-1286 and :1331-1333) that recognition workers use under
 * ScopedDisableParallel (src/pipeline.rs:417-427), so results do not depend on a thread
 * count. Validation mirrors :1227-1232 (K) and :1288-1295 (bias length).
 * a is [rows][k]; out is [rows][n].
 */
int oracle_matmul_quantized_b(const float *a, int64_t rows, int64_t k_a, const int8_t *w, const float *s,
                              int64_t n, int64_t k, const float *bias, int64_t bias_len, float *out,
                              int use_avx2) {
    if (k_a != k) return OR_ERR_ARG;
    if (bias && bias_len != n) return OR_ERR_ARG;
    for (int64_t r = 0; r < rows; r++) {
        if (use_avx2)
            oracle_cols_avx2(a + r * k, w, s, bias, out + r * n, 0, n, k);
        else
            oracle_cols_scalar(a + r * k, w, s, bias, out + r * n, 0, n, k);
    }
    return OR_OK;
}

/*
 * The column-split schedule of matmul_quantized_b (src/ops/matmul.rs:1297-1328) used when
 * the single-line path leaves the global Rayon pool enabled: chunk = max(ceil(n/threads),
 * 64) capped at n; chunk c covers [c*chunk, ...) for every row. Which columns fall in the
 * 4-column kernel vs the tail kernel depends on `threads`, so this is used for timing the
 * one-line CPU baseline, never as the parity checker.
 */
typedef struct {
    const float *a; int64_t rows, k, n; const int8_t *w; const float *s; const float *bias;
    float *out; int64_t chunk; int use_avx2; atomic_long next; int64_t num_chunks;
} colsplit_job;

static void *colsplit_worker(void *p) {
    colsplit_job *j = (colsplit_job *)p;
    for (;;) {
        int64_t c = atomic_fetch_add(&j->next, 1);
        if (c >= j->num_chunks) break;
        int64_t col_start = c * j->chunk;
        int64_t col_count = j->n - col_start < j->chunk ? j->n - col_start : j->chunk;
        for (int64_t r = 0; r < j->rows; r++) {
            if (j->use_avx2)
                oracle_cols_avx2(j->a + r * j->k, j->w, j->s, j->bias, j->out + r * j->n + col_start, col_start,
                                 col_count, j->k);
            else
                oracle_cols_scalar(j->a + r * j->k, j->w, j->s, j->bias, j->out + r * j->n + col_start,
                                   col_start, col_count, j->k);
        }
    }
    return NULL;
}

int oracle_matmul_quantized_b_colsplit(const float *a, int64_t rows, int64_t k, const int8_t *w, const float *s,
                                       int64_t n, const float *bias, float *out, int threads, int use_avx2) {
    if (threads < 1) threads = 1;
    colsplit_job j = {a, rows, k, n, w, s, bias, out, 0, use_avx2, 0, 0};
    int64_t chunk = (n + threads - 1) / threads;
    if (chunk < 64) chunk = 64;
    if (chunk > n) chunk = n;
    j.chunk = chunk;
    j.num_chunks = chunk > 0 ? (n + chunk - 1) / chunk : 0;
    atomic_init(&j.next, 0);
    pthread_t th[256];
    int nt = threads > 256 ? 256 : threads;
    for (int t = 1; t < nt; t++) pthread_create(&th[t], NULL, colsplit_worker, &j);
    colsplit_worker(&j);
    for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
    return OR_OK;
}

/* ---------------------------------------------------------------- softmax */

/* avx2_exp_ps — src/ops/softmax.rs:5-47 (Cody-Waite reduction + degree-6 polynomial). */
__attribute__((target("avx2,fma"))) static inline __m256 avx2_exp_ps(__m256 x) {
    x = _mm256_max_ps(x, _mm256_set1_ps(-87.336544f));
    x = _mm256_min_ps(x, _mm256_set1_ps(88.722839f));
    __m256 log2e = _mm256_set1_ps(1.4426950408889634f);
    __m256 fx = _mm256_round_ps(_mm256_mul_ps(x, log2e), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    __m256 c1 = _mm256_set1_ps(0.693145751953125f);
    __m256 c2 = _mm256_set1_ps(1.42860682030941723212e-6f);
    __m256 g = _mm256_sub_ps(_mm256_sub_ps(x, _mm256_mul_ps(fx, c1)), _mm256_mul_ps(fx, c2));
    __m256 p6 = _mm256_set1_ps(1.3888889e-3f);
    __m256 p5 = _mm256_set1_ps(8.3333333e-3f);
    __m256 p4 = _mm256_set1_ps(4.1666668e-2f);
    __m256 p3 = _mm256_set1_ps(1.6666667e-1f);
    __m256 p2 = _mm256_set1_ps(0.5f);
    __m256 p1 = _mm256_set1_ps(1.0f);
    __m256 y = _mm256_fmadd_ps(p6, g, p5);
    y = _mm256_fmadd_ps(y, g, p4);
    y = _mm256_fmadd_ps(y, g, p3);
    y = _mm256_fmadd_ps(y, g, p2);
    y = _mm256_fmadd_ps(y, g, p1);
    y = _mm256_fmadd_ps(y, g, p1);
    __m256i emm0 = _mm256_cvtps_epi32(fx);
    emm0 = _mm256_add_epi32(emm0, _mm256_set1_epi32(127));
    emm0 = _mm256_slli_epi32(emm0, 23);
    __m256 pow2n = _mm256_castsi256_ps(emm0);
    return _mm256_mul_ps(y, pow2n);
}

/* Scalar element of the polynomial above, exposed for the kernel-side exp tests. */
__attribute__((target("avx2,fma"))) float oracle_exp_poly(float x) {
    float tmp[8];
    _mm256_storeu_ps(tmp, avx2_exp_ps(_mm256_set1_ps(x)));
    return tmp[0];
}

/* compute_row_avx2 — src/ops/softmax.rs:315-416 (in == out allowed: the in-place path). */
__attribute__((target("avx2,fma"))) void oracle_softmax_row_avx2(const float *in_ptr, float *out_ptr, int64_t n) {
    __m256 v_max0 = _mm256_set1_ps(-INFINITY), v_max1 = _mm256_set1_ps(-INFINITY);
    __m256 v_max2 = _mm256_set1_ps(-INFINITY), v_max3 = _mm256_set1_ps(-INFINITY);
    int64_t i = 0;
    while (i + 32 <= n) {
        v_max0 = _mm256_max_ps(v_max0, _mm256_loadu_ps(in_ptr + i));
        v_max1 = _mm256_max_ps(v_max1, _mm256_loadu_ps(in_ptr + i + 8));
        v_max2 = _mm256_max_ps(v_max2, _mm256_loadu_ps(in_ptr + i + 16));
        v_max3 = _mm256_max_ps(v_max3, _mm256_loadu_ps(in_ptr + i + 24));
        i += 32;
    }
    __m256 v_max = _mm256_max_ps(_mm256_max_ps(v_max0, v_max1), _mm256_max_ps(v_max2, v_max3));
    while (i + 8 <= n) {
        v_max = _mm256_max_ps(v_max, _mm256_loadu_ps(in_ptr + i));
        i += 8;
    }
    float max_val = i > 0 ? hmax256(v_max) : -INFINITY;
    while (i < n) {
        if (in_ptr[i] > max_val) max_val = in_ptr[i];
        i++;
    }

    __m256 vm = _mm256_set1_ps(max_val);
    __m256 v_sum0 = _mm256_setzero_ps(), v_sum1 = _mm256_setzero_ps();
    __m256 v_sum2 = _mm256_setzero_ps(), v_sum3 = _mm256_setzero_ps();
    i = 0;
    while (i + 32 <= n) {
        __m256 e0 = avx2_exp_ps(_mm256_sub_ps(_mm256_loadu_ps(in_ptr + i), vm));
        __m256 e1 = avx2_exp_ps(_mm256_sub_ps(_mm256_loadu_ps(in_ptr + i + 8), vm));
        __m256 e2 = avx2_exp_ps(_mm256_sub_ps(_mm256_loadu_ps(in_ptr + i + 16), vm));
        __m256 e3 = avx2_exp_ps(_mm256_sub_ps(_mm256_loadu_ps(in_ptr + i + 24), vm));
        _mm256_storeu_ps(out_ptr + i, e0);
        _mm256_storeu_ps(out_ptr + i + 8, e1);
        _mm256_storeu_ps(out_ptr + i + 16, e2);
        _mm256_storeu_ps(out_ptr + i + 24, e3);
        v_sum0 = _mm256_add_ps(v_sum0, e0);
        v_sum1 = _mm256_add_ps(v_sum1, e1);
        v_sum2 = _mm256_add_ps(v_sum2, e2);
        v_sum3 = _mm256_add_ps(v_sum3, e3);
        i += 32;
    }
    __m256 v_sum = _mm256_add_ps(_mm256_add_ps(v_sum0, v_sum1), _mm256_add_ps(v_sum2, v_sum3));
    while (i + 8 <= n) {
        __m256 e = avx2_exp_ps(_mm256_sub_ps(_mm256_loadu_ps(in_ptr + i), vm));
        _mm256_storeu_ps(out_ptr + i, e);
        v_sum = _mm256_add_ps(v_sum, e);
        i += 8;
    }
    float sum_exp = i > 0 ? hsum256(v_sum) : 0.0f;
    while (i < n) {
        float e = expf(in_ptr[i] - max_val);
        out_ptr[i] = e;
        sum_exp += e;
        i++;
    }

    float inv_sum = sum_exp > 0.0f ? 1.0f / sum_exp : 1.0f;
    __m256 v_inv = _mm256_set1_ps(inv_sum);
    i = 0;
    while (i + 32 <= n) {
        __m256 v0 = _mm256_loadu_ps(out_ptr + i), v1 = _mm256_loadu_ps(out_ptr + i + 8);
        __m256 v2 = _mm256_loadu_ps(out_ptr + i + 16), v3 = _mm256_loadu_ps(out_ptr + i + 24);
        _mm256_storeu_ps(out_ptr + i, _mm256_mul_ps(v0, v_inv));
        _mm256_storeu_ps(out_ptr + i + 8, _mm256_mul_ps(v1, v_inv));
        _mm256_storeu_ps(out_ptr + i + 16, _mm256_mul_ps(v2, v_inv));
        _mm256_storeu_ps(out_ptr + i + 24, _mm256_mul_ps(v3, v_inv));
        i += 32;
    }
    while (i + 8 <= n) {
        _mm256_storeu_ps(out_ptr + i, _mm256_mul_ps(_mm256_loadu_ps(out_ptr + i), v_inv));
        i += 8;
    }
    while (i < n) {
        out_ptr[i] *= inv_sum;
        i++;
    }
}

/* compute_row_scalar — src/ops/softmax.rs:419-436. */
void oracle_softmax_row_scalar(const float *in_row, float *out_row, int64_t n) {
    float max_val = -INFINITY;
    for (int64_t i = 0; i < n; i++)
        if (in_row[i] > max_val) max_val = in_row[i];
    float sum_exp = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        float e = expf(in_row[i] - max_val);
        out_row[i] = e;
        sum_exp += e;
    }
    float inv_sum = sum_exp > 0.0f ? 1.0f / sum_exp : 1.0f;
    for (int64_t i = 0; i < n; i++) out_row[i] *= inv_sum;
}

/* softmax_inplace over the last axis, inner_size == 1 fast path — src/ops/softmax.rs:199-285. */
int oracle_softmax_rows_inplace(float *x, int64_t rows, int64_t n, int use_avx2) {
    if (rows <= 0 || n <= 0) return OR_OK; /* empty: nothing to do (:226-229) */
    for (int64_t r = 0; r < rows; r++) {
        if (use_avx2)
            oracle_softmax_row_avx2(x + r * n, x + r * n, n);
        else
            oracle_softmax_row_scalar(x + r * n, x + r * n, n);
    }
    return OR_OK;
}

/* General-axis softmax (src/ops/softmax.rs:143-196) for [outer][axis][inner] with inner > 1. */
int oracle_softmax_general(const float *in, float *out, int64_t outer, int64_t axis_size, int64_t inner) {
    int64_t stride = axis_size * inner;
    for (int64_t o = 0; o < outer; o++) {
        int64_t base = o * stride;
        for (int64_t in_i = 0; in_i < inner; in_i++) {
            float max_val = -INFINITY;
            for (int64_t a = 0; a < axis_size; a++) {
                float v = in[base + a * inner + in_i];
                if (v > max_val) max_val = v;
            }
            float sum_exp = 0.0f;
            for (int64_t a = 0; a < axis_size; a++) {
                float e = expf(in[base + a * inner + in_i] - max_val);
                out[base + a * inner + in_i] = e;
                sum_exp += e;
            }
            float inv_sum = sum_exp > 0.0f ? 1.0f / sum_exp : 1.0f;
            for (int64_t a = 0; a < axis_size; a++) out[base + a * inner + in_i] *= inv_sum;
        }
    }
    return OR_OK;
}

/* ----------------------------------------------------------------- argmax */

/* find_argmax_scalar — src/postprocess/ctc.rs:190-200. */
void oracle_find_argmax_scalar(const float *x, int64_t n, int64_t *idx_out, float *val_out) {
    int64_t max_idx = 0;
    float max_val = -INFINITY;
    for (int64_t i = 0; i < n; i++) {
        if (x[i] > max_val) {
            max_val = x[i];
            max_idx = i;
        }
    }
    *idx_out = max_idx;
    *val_out = max_val;
}

/* find_argmax_avx2 — src/postprocess/ctc.rs:202-258. */
__attribute__((target("avx2,fma"))) static void find_argmax_avx2(const float *ptr, int64_t n, int64_t *idx_out,
                                                                    float *val_out) {
    __m256 v_max = _mm256_set1_ps(-INFINITY);
    __m256i v_idx = _mm256_setzero_si256();
    __m256i cur_indices = _mm256_set_epi32(7, 6, 5, 4, 3, 2, 1, 0);
    __m256i v_step = _mm256_set1_epi32(8);
    int64_t i = 0;
    while (i + 8 <= n) {
        __m256 v = _mm256_loadu_ps(ptr + i);
        __m256 cmp = _mm256_cmp_ps(v, v_max, _CMP_GT_OQ);
        v_max = _mm256_blendv_ps(v_max, v, cmp);
        v_idx = _mm256_castps_si256(_mm256_blendv_ps(_mm256_castsi256_ps(v_idx), _mm256_castsi256_ps(cur_indices), cmp));
        cur_indices = _mm256_add_epi32(cur_indices, v_step);
        i += 8;
    }
    float max_buf[8];
    int32_t idx_buf[8];
    _mm256_storeu_ps(max_buf, v_max);
    _mm256_storeu_si256((__m256i *)idx_buf, v_idx);
    float best_val = max_buf[0];
    int64_t best_idx = (int64_t)(uint32_t)idx_buf[0];
    for (int lane = 1; lane < 8; lane++) {
        float v = max_buf[lane];
        int64_t id = (int64_t)(uint32_t)idx_buf[lane];
        if (v > best_val) {
            best_val = v;
            best_idx = id;
        } else if (v == best_val && id < best_idx) {
            best_idx = id;
        }
    }
    while (i < n) {
        float val = ptr[i];
        if (val > best_val) {
            best_val = val;
            best_idx = i;
        }
        i++;
    }
    *idx_out = best_idx;
    *val_out = best_val;
}

/* find_argmax dispatch — src/postprocess/ctc.rs:177-188 (AVX2 only for len >= 16). */
void oracle_find_argmax(const float *x, int64_t n, int use_avx2, int64_t *idx_out, float *val_out) {
    if (n <= 0) {
        *idx_out = 0;
        *val_out = -INFINITY;
        return;
    }
    if (use_avx2 && n >= 16)
        find_argmax_avx2(x, n, idx_out, val_out);
    else
        oracle_find_argmax_scalar(x, n, idx_out, val_out);
}

/* ------------------------------------------------------------ CTC collapse */

/*
 * The collapse and score of CtcDecoder::decode_batch — src/postprocess/ctc.rs:144-169 —
 * applied to per-timestep (argmax index, max probability) pairs. Line l covers timesteps
 * [line_offsets[l], line_offsets[l+1]). Emitted class indices are written to tokens
 * (token_offsets[l]..token_offsets[l+1]); score[l] is the f32 mean of the emitted maxima
 * (0 when nothing is emitted). Returns the total number of emitted tokens.
 */
int64_t oracle_ctc_collapse(const int32_t *idx, const float *prob, const int64_t *line_offsets, int64_t n_lines,
                            int32_t *tokens, int64_t *token_offsets, float *scores) {
    int64_t w = 0;
    for (int64_t l = 0; l < n_lines; l++) {
        token_offsets[l] = w;
        int64_t last_idx = 0;
        float sum = 0.0f;
        int64_t count = 0;
        for (int64_t t = line_offsets[l]; t < line_offsets[l + 1]; t++) {
            int64_t mi = idx[t];
            if (mi != 0 && mi != last_idx) {
                tokens[w++] = (int32_t)mi;
                sum += prob[t];
                count++;
            }
            last_idx = mi;
        }
        scores[l] = count == 0 ? 0.0f : sum / (float)count;
    }
    token_offsets[n_lines] = w;
    return w;
}

/* ----------------------------------------------------- whole head per row */

/*
 * One recognition line through the head exactly as the engine runs it: the MatMul arm
 * (src/engine/model.rs:1245-1272) -> matmul_quantized_b with the folded bias, the Softmax
 * arm (:1286-1302) -> softmax_inplace, then CtcDecoder's per-timestep find_argmax
 * (src/postprocess/ctc.rs:144-149). Emits (idx, prob) per timestep; optionally the raw
 * logits, the top-2 logit gap (max - second max) used to recognise near-ties and the row's
 * largest logit.
 */
typedef struct {
    const float *a; int64_t k, n; const int8_t *w; const float *s; const float *bias;
    const int64_t *offsets; int64_t n_units;
    int32_t *idx; float *prob; float *logits_out; float *gap; float *lmax; int use_avx2;
    atomic_long next;
} head_job;

static void head_rows(head_job *j, int64_t r0, int64_t r1, float *row_buf) {
    for (int64_t r = r0; r < r1; r++) {
        float *lg = j->logits_out ? j->logits_out + r * j->n : row_buf;
        if (j->use_avx2)
            oracle_cols_avx2(j->a + r * j->k, j->w, j->s, j->bias, lg, 0, j->n, j->k);
        else
            oracle_cols_scalar(j->a + r * j->k, j->w, j->s, j->bias, lg, 0, j->n, j->k);
        if (j->gap || j->lmax) {
            float m1 = -INFINITY, m2 = -INFINITY;
            for (int64_t c = 0; c < j->n; c++) {
                float v = lg[c];
                if (v > m1) {
                    m2 = m1;
                    m1 = v;
                } else if (v > m2) {
                    m2 = v;
                }
            }
            if (j->gap) j->gap[r] = m1 - m2;
            if (j->lmax) j->lmax[r] = m1;
        }
        float *p = row_buf;
        if (j->use_avx2)
            oracle_softmax_row_avx2(lg, p, j->n);
        else
            oracle_softmax_row_scalar(lg, p, j->n);
        int64_t mi;
        float mv;
        oracle_find_argmax(p, j->n, j->use_avx2, &mi, &mv);
        j->idx[r] = (int32_t)mi;
        j->prob[r] = mv;
    }
}

static void *head_worker(void *p) {
    head_job *j = (head_job *)p;
    float *row_buf = (float *)malloc(sizeof(float) * (size_t)(j->n > 0 ? j->n : 1));
    for (;;) {
        int64_t u = atomic_fetch_add(&j->next, 1);
        if (u >= j->n_units) break;
        head_rows(j, j->offsets[u], j->offsets[u + 1], row_buf);
    }
    free(row_buf);
    return NULL;
}

/*
 * Runs rows [line_offsets[0], line_offsets[n_lines]) with lines handed to `threads`
 * workers (each line serial, as the per-line Rayon workers of src/pipeline.rs:417-427).
 * Results do not depend on `threads`.
 */
int oracle_head_decode(const float *a, const int64_t *line_offsets, int64_t n_lines, int64_t k, const int8_t *w,
                       const float *s, int64_t n, const float *bias, int32_t *idx, float *prob, float *logits_out,
                       float *gap, float *lmax, int threads, int use_avx2) {
    if (n_lines <= 0) return OR_OK;
    if (threads < 1) threads = 1;
    head_job j = {a, k, n, w, s, bias, line_offsets, n_lines, idx, prob, logits_out, gap, lmax, use_avx2, 0};
    atomic_init(&j.next, 0);
    int nt = threads > 256 ? 256 : threads;
    if (nt > n_lines) nt = (int)n_lines;
    pthread_t th[256];
    for (int t = 1; t < nt; t++) pthread_create(&th[t], NULL, head_worker, &j);
    head_worker(&j);
    for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
    return OR_OK;
}

/*
 * One line whose rows go through the column-split projection (src/ops/matmul.rs:1297-1328,
 * the single-line path with the global pool enabled), then per-row softmax and argmax.
 * Used only to time the single-line CPU baseline.
 */
int oracle_head_decode_one_line(const float *a, int64_t rows, int64_t k, const int8_t *w, const float *s,
                                int64_t n, const float *bias, int32_t *idx, float *prob, float *logits_scratch,
                                int threads, int use_avx2) {
    oracle_matmul_quantized_b_colsplit(a, rows, k, w, s, n, bias, logits_scratch, threads, use_avx2);
    for (int64_t r = 0; r < rows; r++) {
        float *lg = logits_scratch + r * n;
        if (use_avx2)
            oracle_softmax_row_avx2(lg, lg, n);
        else
            oracle_softmax_row_scalar(lg, lg, n);
        int64_t mi;
        float mv;
        oracle_find_argmax(lg, n, use_avx2, &mi, &mv);
        idx[r] = (int32_t)mi;
        prob[r] = mv;
    }
    return OR_OK;
}

/* A plain f32 [rows][k] x [n][k]^T product with bias, used by the reference's INT8-vs-FP32
 * tolerance tests (src/ops/matmul.rs:1673-1697, :1812-1840) as the FP32 side. Accumulates in
 * f64 and rounds once, i.e. the exact product the FP32 kernel approximates. */
void oracle_matmul_f32_transposed_b(const float *a, int64_t rows, int64_t k, const float *b_t, int64_t n,
                                    const float *bias, float *out) {
    for (int64_t r = 0; r < rows; r++)
        for (int64_t j = 0; j < n; j++) {
            double acc = 0.0;
            for (int64_t i = 0; i < k; i++) acc += (double)a[r * k + i] * (double)b_t[j * k + i];
            out[r * n + j] = (float)acc + (bias ? bias[j] : 0.0f);
        }
}

/* ------------------------------------------------------- FP32 head (matmul_transposed_b) */

/*
 * The engine's default head (OcrEngineConfig.quantize_rec_head = false, src/pipeline.rs:59):
 * MatMul.12 runs matmul_transposed_b (src/ops/matmul.rs:514-897) on the FP32 [n][k] weight.
 * A recognition line runs inside a rec worker with ScopedDisableParallel
 * (src/pipeline.rs:417-427), so neither parallel branch is taken: with AVX2 and k % 8 == 0
 * the rows go through run_block (:648-742) in groups of TILE_ROWS = 3 (:1094), columns
 * 0..n - n%4 through transposed_b_tile_fma (:1025-1087) and the last n % 4 columns through
 * compute_transposed_b_cols_avx2 (:913-1000), which for fewer than 4 columns is
 * avx2_dot_product (:1120-1160); otherwise each row goes through
 * compute_transposed_b_cols_avx2 (AVX2) or compute_transposed_b_cols_scalar (:1097-1116).
 */

/* avx2_dot_product: src/ops/matmul.rs:1120-1160. */
__attribute__((target("avx2,fma"))) static float f32_dot_avx2(const float *a, const float *b, int64_t n) {
    int64_t i = 0;
    __m256 v0 = _mm256_setzero_ps(), v1 = _mm256_setzero_ps(), v2 = _mm256_setzero_ps(), v3 = _mm256_setzero_ps();
    while (i + 32 <= n) {
        v0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), v0);
        v1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), v1);
        v2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 16), _mm256_loadu_ps(b + i + 16), v2);
        v3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 24), _mm256_loadu_ps(b + i + 24), v3);
        i += 32;
    }
    v0 = _mm256_add_ps(_mm256_add_ps(v0, v1), _mm256_add_ps(v2, v3));
    while (i + 8 <= n) {
        v0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), v0);
        i += 8;
    }
    float sum = hsum256(v0);
    while (i < n) {
        sum += a[i] * b[i];
        i++;
    }
    return sum;
}

/* compute_transposed_b_cols_avx2: src/ops/matmul.rs:913-1000 (columns col_start .. +count). */
__attribute__((target("avx2,fma"))) static void f32_cols_avx2(const float *a_row, const float *b_t, const float *bias,
                                                             float *out, int64_t col_start, int64_t col_count,
                                                             int64_t k) {
    int64_t c = 0;
    while (c + 4 <= col_count) {
        const int64_t j0 = col_start + c;
        const float *b0 = b_t + j0 * k, *b1 = b0 + k, *b2 = b1 + k, *b3 = b2 + k;
        __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps(), acc2 = _mm256_setzero_ps(),
               acc3 = _mm256_setzero_ps();
        int64_t i = 0;
        while (i + 8 <= k) {
            __m256 va = _mm256_loadu_ps(a_row + i);
            acc0 = _mm256_fmadd_ps(va, _mm256_loadu_ps(b0 + i), acc0);
            acc1 = _mm256_fmadd_ps(va, _mm256_loadu_ps(b1 + i), acc1);
            acc2 = _mm256_fmadd_ps(va, _mm256_loadu_ps(b2 + i), acc2);
            acc3 = _mm256_fmadd_ps(va, _mm256_loadu_ps(b3 + i), acc3);
            i += 8;
        }
        float s0 = hsum256(acc0), s1 = hsum256(acc1), s2 = hsum256(acc2), s3 = hsum256(acc3);
        while (i < k) {
            const float av = a_row[i];
            s0 += av * b0[i];
            s1 += av * b1[i];
            s2 += av * b2[i];
            s3 += av * b3[i];
            i++;
        }
        if (bias) {
            out[c] = s0 + bias[j0];
            out[c + 1] = s1 + bias[j0 + 1];
            out[c + 2] = s2 + bias[j0 + 2];
            out[c + 3] = s3 + bias[j0 + 3];
        } else {
            out[c] = s0;
            out[c + 1] = s1;
            out[c + 2] = s2;
            out[c + 3] = s3;
        }
        c += 4;
    }
    while (c < col_count) {
        const int64_t j = col_start + c;
        const float dot = f32_dot_avx2(a_row, b_t + j * k, k);
        out[c] = bias ? dot + bias[j] : dot;
        c++;
    }
}

/* compute_transposed_b_cols_scalar: src/ops/matmul.rs:1097-1116 (Rust's f32 Sum folds from -0.0). */
static void f32_cols_scalar(const float *a_row, const float *b_t, const float *bias, float *out, int64_t col_start,
                            int64_t col_count, int64_t k) {
    for (int64_t c = 0; c < col_count; c++) {
        const int64_t j = col_start + c;
        const float *b = b_t + j * k;
        float dot = -0.0f;
        for (int64_t i = 0; i < k; i++) dot += a_row[i] * b[i];
        out[c] = bias ? dot + bias[j] : dot;
    }
}

/* transposed_b_tile_fma<MR>: src/ops/matmul.rs:1025-1087; MR rows x 4 columns from column c. */
__attribute__((target("avx2,fma"))) static void f32_tile(const float *a, const float *b, float *out, int64_t ldo,
                                                        int64_t c, const float *bias, int64_t k, int mr) {
    const float *b0 = b, *b1 = b + k, *b2 = b + 2 * k, *b3 = b + 3 * k;
    __m256 acc[12];
    for (int i = 0; i < 12; i++) acc[i] = _mm256_setzero_ps();
    for (int64_t i = 0; i < k; i += 8) {
        const __m256 bv0 = _mm256_loadu_ps(b0 + i), bv1 = _mm256_loadu_ps(b1 + i), bv2 = _mm256_loadu_ps(b2 + i),
                     bv3 = _mm256_loadu_ps(b3 + i);
        for (int r = 0; r < mr; r++) {
            const __m256 av = _mm256_loadu_ps(a + r * k + i);
            acc[r * 4] = _mm256_fmadd_ps(av, bv0, acc[r * 4]);
            acc[r * 4 + 1] = _mm256_fmadd_ps(av, bv1, acc[r * 4 + 1]);
            acc[r * 4 + 2] = _mm256_fmadd_ps(av, bv2, acc[r * 4 + 2]);
            acc[r * 4 + 3] = _mm256_fmadd_ps(av, bv3, acc[r * 4 + 3]);
        }
    }
    const __m128 bv = bias ? _mm_loadu_ps(bias + c) : _mm_setzero_ps();
    for (int r = 0; r < mr; r++) {
        const __m256 h01 = _mm256_hadd_ps(acc[r * 4], acc[r * 4 + 1]);
        const __m256 h23 = _mm256_hadd_ps(acc[r * 4 + 2], acc[r * 4 + 3]);
        const __m256 h0123 = _mm256_hadd_ps(h01, h23);
        __m128 sums = _mm_add_ps(_mm256_castps256_ps128(h0123), _mm256_extractf128_ps(h0123, 1));
        if (bias) sums = _mm_add_ps(sums, bv);
        _mm_storeu_ps(out + r * ldo, sums);
    }
}

/*
 * Rows [0, rows) of one line (rows <= 3 when blocked; any count otherwise) into out [rows][n]:
 * one run_block chunk (src/ops/matmul.rs:648-742) or run_row per row (:607-620).
 */
static void f32_line_rows(const float *a, int64_t rows, int64_t k, const float *b_t, int64_t n, const float *bias,
                          float *out, int use_avx2) {
    if (use_avx2 && k % 8 == 0) {
        const int64_t cols_full = n - n % 4;
        for (int64_t c = 0; c < cols_full; c += 4) f32_tile(a, b_t + c * k, out + c, n, c, bias, k, (int)rows);
        if (cols_full < n)
            for (int64_t r = 0; r < rows; r++)
                f32_cols_avx2(a + r * k, b_t, bias, out + r * n + cols_full, cols_full, n - cols_full, k);
        return;
    }
    for (int64_t r = 0; r < rows; r++) {
        if (use_avx2)
            f32_cols_avx2(a + r * k, b_t, bias, out + r * n, 0, n, k);
        else
            f32_cols_scalar(a + r * k, b_t, bias, out + r * n, 0, n, k);
    }
}

/* matmul_transposed_b over the rows of one line (the engine's per-line call). */
void oracle_matmul_transposed_b(const float *a, int64_t rows, int64_t k, const float *b_t, int64_t n,
                                const float *bias, float *out, int use_avx2) {
    const int64_t step = (use_avx2 && k % 8 == 0) ? 3 : (rows > 0 ? rows : 1);
    for (int64_t r0 = 0; r0 < rows; r0 += step) {
        const int64_t nr = rows - r0 < step ? rows - r0 : step;
        f32_line_rows(a + r0 * k, nr, k, b_t, n, bias, out + r0 * n, use_avx2);
    }
}

typedef struct {
    const float *a; int64_t k, n; const float *b_t; const float *bias;
    const int64_t *offsets; int64_t n_lines;
    int32_t *idx; float *prob; float *logits_out; float *gap; float *lmax; int use_avx2;
    atomic_long next;
} f32_job;

static void *f32_worker(void *p) {
    f32_job *j = (f32_job *)p;
    float *buf = (float *)malloc(sizeof(float) * (size_t)(3 * (j->n > 0 ? j->n : 1)));
    float *prow = (float *)malloc(sizeof(float) * (size_t)(j->n > 0 ? j->n : 1));
    for (;;) {
        const int64_t l = atomic_fetch_add(&j->next, 1);
        if (l >= j->n_lines) break;
        const int64_t r_begin = j->offsets[l], r_end = j->offsets[l + 1];
        const int64_t step = (j->use_avx2 && j->k % 8 == 0) ? 3 : 1;
        for (int64_t r0 = r_begin; r0 < r_end; r0 += step) {
            const int64_t nr = r_end - r0 < step ? r_end - r0 : step;
            float *lg = j->logits_out ? j->logits_out + r0 * j->n : buf;
            f32_line_rows(j->a + r0 * j->k, nr, j->k, j->b_t, j->n, j->bias, lg, j->use_avx2);
            for (int64_t rr = 0; rr < nr; rr++) {
                const int64_t r = r0 + rr;
                const float *row = lg + rr * j->n;
                if (j->gap || j->lmax) {
                    float m1 = -INFINITY, m2 = -INFINITY;
                    for (int64_t c = 0; c < j->n; c++) {
                        const float v = row[c];
                        if (v > m1) {
                            m2 = m1;
                            m1 = v;
                        } else if (v > m2) {
                            m2 = v;
                        }
                    }
                    if (j->gap) j->gap[r] = m1 - m2;
                    if (j->lmax) j->lmax[r] = m1;
                }
                if (j->use_avx2)
                    oracle_softmax_row_avx2(row, prow, j->n);
                else
                    oracle_softmax_row_scalar(row, prow, j->n);
                int64_t mi;
                float mv;
                oracle_find_argmax(prow, j->n, j->use_avx2, &mi, &mv);
                j->idx[r] = (int32_t)mi;
                j->prob[r] = mv;
            }
        }
    }
    free(prow);
    free(buf);
    return NULL;
}

/*
 * The FP32 head per timestep (matmul_transposed_b with the folded bias -> softmax ->
 * find_argmax), lines handed to `threads` workers. Results do not depend on `threads`.
 */
int oracle_head_decode_f32(const float *a, const int64_t *line_offsets, int64_t n_lines, int64_t k, const float *b_t,
                           int64_t n, const float *bias, int32_t *idx, float *prob, float *logits_out, float *gap,
                           float *lmax, int threads, int use_avx2) {
    if (n_lines <= 0) return OR_OK;
    if (threads < 1) threads = 1;
    f32_job j = {a, k, n, b_t, bias, line_offsets, n_lines, idx, prob, logits_out, gap, lmax, use_avx2, 0};
    atomic_init(&j.next, 0);
    int nt = threads > 256 ? 256 : threads;
    if (nt > n_lines) nt = (int)n_lines;
    pthread_t th[256];
    for (int t = 1; t < nt; t++) pthread_create(&th[t], NULL, f32_worker, &j);
    f32_worker(&j);
    for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
    return OR_OK;
}
