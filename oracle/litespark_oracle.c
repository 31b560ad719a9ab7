/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's CPU int4 decode kernels. Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * leg load this library, and only as the checker or the timed CPU baseline.
 * The product (harsh4b_b200) never links or calls it.
 *
 * What it follows (paths relative to the reference project root):
 *   cpu_kernels/litespark_int4.cpp:22-76    litespark_int4_i8_gemv_impl: one
 *       int32 dot product per row, epilogue float(acc) * act_scale * w_scale
 *       evaluated left to right, OpenMP row split if rows >= 64.
 *   cpu_kernels/litespark_int4.cpp:78-108   C ABI (x, weights, scales,
 *       activation_scale, output, rows, width).
 *   cpu_kernels/litespark_int4.cpp:160-259  litespark_gqa_decode: scores,
 *       max-subtracted softmax normalised before the value sum.
 *   cpu_lightspark.py:139-146 / :345-348   nibble layout: low nibble = even
 *       k, high nibble = odd k, two's complement.
 *   Third-party litespark-inference==1.0.3 (pyproject.toml:39; absent here,
 *       not vendored): rmsnorm_into, quantize_activation, add_inplace, called
 *       at cpu_lightspark.py:431-463. Their arithmetic is restated below as
 *       this project's contract; no reference test pins them.
 *
 * The reference kernel is ARM NEON (vdotq_s32); this file is portable C with
 * an optional AVX2 path for the row dot, both exact in int32.
 */
#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__AVX2__)
#include <immintrin.h>
#endif

/* ---- int4 x int8 row dot ------------------------------------------------ */

/* Literal restatement of litespark_int4.cpp:65-72 (the scalar tail loop,
 * which computes the same sum as the SDOT body). */
static int32_t row_dot_scalar(const uint8_t *row, const int8_t *x, int packed_width)
{
    int32_t acc = 0;
    for (int i = 0; i < packed_width; ++i) {
        const uint8_t byte = row[i];
        const int8_t low = (int8_t)(uint8_t)(byte << 4) >> 4;
        const int8_t high = (int8_t)byte >> 4;
        acc += (int32_t)low * x[2 * i];
        acc += (int32_t)high * x[2 * i + 1];
    }
    return acc;
}

#if defined(__AVX2__)
/* Same sum, 64 nibbles per step. Each nibble n is read as u = n ^ 8 = s + 8
 * (unsigned, 0..15) so _mm256_maddubs_epi16 (u8 x s8) applies; the bias
 * 8 * sum(x) is removed at the end. Pair sums stay within int16. */
static int32_t row_dot_avx2(const uint8_t *row, const int8_t *xe, const int8_t *xo,
                            int packed_width, int32_t x_sum)
{
    const __m256i flip = _mm256_set1_epi8((char)0x88);
    const __m256i nib = _mm256_set1_epi8(0x0F);
    const __m256i ones = _mm256_set1_epi16(1);
    __m256i acc = _mm256_setzero_si256();
    int i = 0;
    for (; i + 32 <= packed_width; i += 32) {
        const __m256i b = _mm256_xor_si256(_mm256_loadu_si256((const __m256i *)(row + i)), flip);
        const __m256i lo = _mm256_and_si256(b, nib);
        const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(b, 4), nib);
        const __m256i pe = _mm256_maddubs_epi16(lo, _mm256_loadu_si256((const __m256i *)(xe + i)));
        const __m256i po = _mm256_maddubs_epi16(hi, _mm256_loadu_si256((const __m256i *)(xo + i)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(_mm256_add_epi16(pe, po), ones));
    }
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    int32_t biased = _mm_cvtsi128_si32(s);
    for (; i < packed_width; ++i) {
        const uint8_t u = row[i] ^ 0x88;
        biased += (int32_t)(u & 15) * xe[i] + (int32_t)(u >> 4) * xo[i];
    }
    return biased - 8 * x_sum;
}
#endif

/* int32 accumulators for every row; acc may be NULL when only out is wanted.
 * use_simd = 0 forces the literal scalar restatement. */
static void gemv_rows(const int8_t *x, const uint8_t *weights, const float *scales,
                      float activation_scale, float *output, int32_t *acc_out,
                      int rows, int width, int use_simd)
{
    const int packed_width = width >> 1;
#if defined(__AVX2__)
    int8_t *xe = NULL, *xo = NULL;
    int32_t x_sum = 0;
    if (use_simd) {
        xe = (int8_t *)malloc((size_t)packed_width + 32);
        xo = (int8_t *)malloc((size_t)packed_width + 32);
        for (int i = 0; i < packed_width; ++i) {
            xe[i] = x[2 * i];
            xo[i] = x[2 * i + 1];
            x_sum += x[2 * i] + x[2 * i + 1];
        }
    }
#else
    (void)use_simd;
#endif
#pragma omp parallel for if (rows >= 64) schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t *row = weights + (ptrdiff_t)r * packed_width;
        int32_t acc;
#if defined(__AVX2__)
        acc = use_simd ? row_dot_avx2(row, xe, xo, packed_width, x_sum)
                       : row_dot_scalar(row, x, packed_width);
#else
        acc = row_dot_scalar(row, x, packed_width);
#endif
        if (acc_out) acc_out[r] = acc;
        /* litespark_int4.cpp:73-74: (float)acc * activation_scale * scale. */
        if (output) output[r] = (float)acc * activation_scale * scales[r];
    }
#if defined(__AVX2__)
    free(xe);
    free(xo);
#endif
}

/* Same C signature as litespark_int4_i8_gemv (litespark_int4.cpp:78-81), so
 * cpu_lightspark.LiteSparkQwen can take it as its int4_kernel. */
void oracle_int4_i8_gemv(const int8_t *x, const uint8_t *weights, const float *scales,
                         float activation_scale, float *output, int rows, int width)
{
    gemv_rows(x, weights, scales, activation_scale, output, NULL, rows, width, 1);
}

/* Exposes the int32 accumulators; simd = 0 runs the literal scalar loop. */
void oracle_int4_i8_gemv_acc(const int8_t *x, const uint8_t *weights, const float *scales,
                             float activation_scale, float *output, int32_t *acc,
                             int rows, int width, int simd)
{
    gemv_rows(x, weights, scales, activation_scale, output, acc, rows, width, simd);
}

/* ---- third-party kernel restatements (parity unpinned) ------------------ */

/* kernel.quantize_activation(values, quantized) -> dequant scale
 * (cpu_lightspark.py:433; semantics follow MLX/bitnet_mlx.py:17-23, the
 * only in-repo statement of per-token absmax int8 quantisation):
 *   m = max(absmax(v), 1e-5); qs = 127 / m (one fp32 division);
 *   q = clamp(rint(v * qs), -127, 127) (one fp32 multiply, half-to-even);
 *   returns m / 127 (one fp32 division), the scale the GEMV epilogue uses. */
float oracle_quantize_activation(const float *values, int8_t *quantized, int n)
{
    float m = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float a = fabsf(values[i]);
        if (a > m) m = a;
    }
    if (m < 1e-5f) m = 1e-5f;
    const float qs = 127.0f / m;
    for (int i = 0; i < n; ++i) {
        float t = rintf(values[i] * qs);
        if (t > 127.0f) t = 127.0f;
        if (t < -127.0f) t = -127.0f;
        quantized[i] = (int8_t)t;
    }
    return m / 127.0f;
}

/* kernel.rmsnorm_into(x, w, out, eps) (cpu_lightspark.py:431,447,461):
 *   out = (x * (1 / sqrt(sum(x^2) / n + eps))) * w
 * The sum of squares is accumulated in double and rounded once to fp32. */
void oracle_rmsnorm(const float *x, const float *w, float *out, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    const float mean = (float)ss / (float)n;
    const float inv = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * inv) * w[i];
}

/* kernel.add_inplace(x, y) (cpu_lightspark.py:445,459). */
void oracle_add_inplace(float *x, const float *y, int n)
{
    for (int i = 0; i < n; ++i) x[i] += y[i];
}

/* ---- single-token GQA (litespark_int4.cpp:160-259) ---------------------- */

/* keys/values: [time, kv_heads, head_dim] fp32; query/output heads ordered
 * [kv_head, group, head_dim]; scores: caller scratch [q_heads, score_stride]. */
void oracle_gqa_decode(const float *query, const float *keys, const float *values,
                       float *scores, float *output, int context, int kv_heads,
                       int groups, int head_dim, int score_stride)
{
    const int query_heads = kv_heads * groups;
    const int time_stride = kv_heads * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel for if (query_heads >= 8) schedule(static)
    for (int h = 0; h < query_heads; ++h) {
        const int kvh = h / groups;
        const float *q = query + (ptrdiff_t)h * head_dim;
        float *score = scores + (ptrdiff_t)h * score_stride;
        float maximum = -FLT_MAX;
        for (int t = 0; t < context; ++t) {
            const float *k = keys + (ptrdiff_t)t * time_stride + (ptrdiff_t)kvh * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; ++d) dot += q[d] * k[d];
            score[t] = dot * scale;
            if (score[t] > maximum) maximum = score[t];
        }
        float denominator = 0.0f;
        for (int t = 0; t < context; ++t) {
            const float p = expf(score[t] - maximum);
            score[t] = p;
            denominator += p;
        }
        const float inverse = 1.0f / denominator;
        for (int t = 0; t < context; ++t) score[t] *= inverse;
        float *o = output + (ptrdiff_t)h * head_dim;
        for (int d = 0; d < head_dim; ++d) {
            float sum = 0.0f;
            for (int t = 0; t < context; ++t)
                sum += score[t] * values[(ptrdiff_t)t * time_stride + (ptrdiff_t)kvh * head_dim + d];
            o[d] = sum;
        }
    }
}

/* Threads the OpenMP runtime will use (1 when built without OpenMP). */
int oracle_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
