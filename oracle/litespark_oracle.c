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
 *
 * Reduction orders and exp: the reference does not pin them (its RMSNorm is
 * third-party, and its NEON and numpy attention paths already sum in
 * different orders). On this int8-quantised model an order change alone
 * moves logits by ~0.1 (the quantiser turns last-ulp differences into code
 * flips), so the model-level functions below fix the order to the device
 * kernels' documented order and use one exp implementation, which makes
 * device-vs-oracle parity bit-exact. oracle_gqa_decode keeps the reference's
 * own order and is checked against the reference's known answers.
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

/* ---- arithmetic shared bit-for-bit with the device -------------------- */

/* exp(x) by Cody-Waite range reduction (x = n ln2 + r, |r| <= ln2/2, ln2 split
 * into a short high part and a low correction) and the degree-7 Taylor
 * polynomial of exp(r) in Horner form, then an exact scaling by 2^n. Inputs
 * below -87 return 0 and inputs above 88 are clamped to 88. Every operation
 * is a single IEEE fp32 op or fmaf, so the device (common.cuh, h4b::exp_cw)
 * produces the same bits. Within 2 ulp of exp on [-87, 88]. */
float oracle_expf(float x)
{
    if (x < -87.0f) return 0.0f;
    if (x > 88.0f) x = 88.0f;
    const float n = rintf(x * 1.44269504f);
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.42860682e-06f, r);
    float p = 1.98412698e-04f;
    p = fmaf(p, r, 1.38888889e-03f);
    p = fmaf(p, r, 8.33333333e-03f);
    p = fmaf(p, r, 4.16666667e-02f);
    p = fmaf(p, r, 1.66666667e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    union { uint32_t u; float f; } scale;
    scale.u = (uint32_t)((int)n + 127) << 23;
    return p * scale.f;
}

void oracle_exp_array(const float *x, float *out, int n)
{
    for (int i = 0; i < n; ++i) out[i] = oracle_expf(x[i]);
}

/* 32-lane butterfly sum (xor 16, 8, 4, 2, 1), the device's warp_sum. */
static float butterfly32(float lanes[32])
{
    float next[32];
    for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; ++l) next[l] = lanes[l] + lanes[l ^ o];
        memcpy(lanes, next, sizeof(next));
    }
    return lanes[0];
}

/* kernel.rmsnorm_into(x, w, out, eps) (cpu_lightspark.py:431,447,461):
 *   out = (x * (1 / sqrt(sum(x^2) / n + eps))) * w
 * with the sum of squares in the device's order: 256 partials, partial t
 * takes the 8-column groups g = t, t+256, ... with fmaf; each warp of 32
 * partials is summed by butterfly; the 8 warp sums are added in order. */
void oracle_rmsnorm(const float *x, const float *w, float *out, int n, float eps)
{
    float partial[256];
    const int groups = n >> 3;
    for (int t = 0; t < 256; ++t) {
        float ss = 0.0f;
        for (int g = t; g < groups; g += 256)
            for (int e = 0; e < 8; ++e) ss = fmaf(x[8 * g + e], x[8 * g + e], ss);
        partial[t] = ss;
    }
    float total = 0.0f;
    for (int warp = 0; warp < 8; ++warp) total += butterfly32(partial + 32 * warp);
    const float mean = total / (float)n;
    const float inv = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * inv) * w[i];
}

/* Lane l of a 128-wide head holds v[4l..4l+3]; its share of a dot product
 * is fma(a3,b3, fma(a2,b2, fma(a1,b1, a0*b0))), summed over lanes by
 * butterfly. */
static float head_dot(const float *a, const float *b)
{
    float lanes[32];
    for (int l = 0; l < 32; ++l) {
        const float *p = a + 4 * l, *q = b + 4 * l;
        lanes[l] = fmaf(p[3], q[3], fmaf(p[2], q[2], fmaf(p[1], q[1], p[0] * q[0])));
    }
    return butterfly32(lanes);
}

/* Per-head RMSNorm of q or k (cpu_lightspark.py:373-379): v / sqrt(mean(v^2)
 * + eps) * gamma, divide first, for heads of 128 in the device's order. */
void oracle_qk_norm(float *v, const float *gamma, int heads, float eps)
{
    for (int h = 0; h < heads; ++h) {
        float *x = v + 128 * h;
        const float ss = head_dot(x, x);
        const float root = sqrtf(ss / 128.0f + eps);
        for (int d = 0; d < 128; ++d) x[d] = (x[d] / root) * gamma[d];
    }
}

/* SiLU(gate) * up (cpu_lightspark.py:451-455): gate / (1 + exp(-gate)) * up. */
void oracle_silu_mul(const float *gate, const float *up, float *out, int n)
{
    for (int i = 0; i < n; ++i) out[i] = (gate[i] / (1.0f + oracle_expf(-gate[i]))) * up[i];
}

/* Single-token GQA in the device's split-K order (head_dim 128). The context
 * is cut into `splits` chunks of ceil(context/splits) tokens, each chunk into
 * sub-tiles of 64 tokens. Per sub-tile: scores s_t = head_dot(q, k_t) * scale,
 * m = max s, p_t = exp(s_t - m), l = butterfly over lanes of (p_lane +
 * p_lane+32), o[d] = sum_t p_t v_t[d] by fmaf in token order. Sub-tiles fold
 * into the chunk's running (m, l, o) with weights exp(m_old - m_new) and
 * exp(m_sub - m_new); chunks merge in order with weights exp(m_c - max m).
 * keys/values element (t, kv, d) sits at t * time_stride + kv * head_stride + d. */
#define SUBTILE 64
void oracle_gqa_splitk(const float *query, const float *keys, const float *values, float *output,
                       int context, int kv_heads, int groups, long time_stride, long head_stride, int splits)
{
    const float scale = 1.0f / sqrtf(128.0f);
    const int chunk = (context + splits - 1) / splits;
    const int query_heads = kv_heads * groups;
#pragma omp parallel for if (query_heads >= 8) schedule(static)
    for (int h = 0; h < query_heads; ++h) {
        const int kvh = h / groups;
        const float *q = query + 128 * h;
        float ms[64], ls[64], os[64][128];
        for (int c = 0; c < splits; ++c) {
            const int t0 = c * chunk < context ? c * chunk : context;
            const int t1 = t0 + chunk < context ? t0 + chunk : context;
            float m = -INFINITY, l = 0.0f, o[128];
            for (int d = 0; d < 128; ++d) o[d] = 0.0f;
            for (int base = t0; base < t1; base += SUBTILE) {
                const int n = t1 - base < SUBTILE ? t1 - base : SUBTILE;
                float sc[SUBTILE], p[SUBTILE];
                float mt = -INFINITY;
                for (int i = 0; i < n; ++i) {
                    const float *k = keys + (long)(base + i) * time_stride + kvh * head_stride;
                    sc[i] = head_dot(q, k) * scale;
                    mt = fmaxf(mt, sc[i]);
                }
                for (int i = 0; i < SUBTILE; ++i) p[i] = i < n ? oracle_expf(sc[i] - mt) : 0.0f;
                float lanes[32];
                for (int ln = 0; ln < 32; ++ln) lanes[ln] = p[ln] + p[ln + 32];
                const float lt = butterfly32(lanes);
                float ot[128];
                for (int d = 0; d < 128; ++d) ot[d] = 0.0f;
                for (int i = 0; i < n; ++i) {
                    const float *v = values + (long)(base + i) * time_stride + kvh * head_stride;
                    for (int d = 0; d < 128; ++d) ot[d] = fmaf(p[i], v[d], ot[d]);
                }
                const float mn = fmaxf(m, mt);
                const float c_old = oracle_expf(m - mn), c_new = oracle_expf(mt - mn);
                l = fmaf(l, c_old, lt * c_new);
                for (int d = 0; d < 128; ++d) o[d] = fmaf(o[d], c_old, ot[d] * c_new);
                m = mn;
            }
            ms[c] = m;
            ls[c] = l;
            memcpy(os[c], o, sizeof(o));
        }
        float mmax = -INFINITY;
        for (int c = 0; c < splits; ++c) mmax = fmaxf(mmax, ms[c]);
        float l = 0.0f, acc[128];
        for (int d = 0; d < 128; ++d) acc[d] = 0.0f;
        for (int c = 0; c < splits; ++c) {
            if (ls[c] == 0.0f) continue;
            const float wgt = oracle_expf(ms[c] - mmax);
            l = fmaf(ls[c], wgt, l);
            for (int d = 0; d < 128; ++d) acc[d] = fmaf(os[c][d], wgt, acc[d]);
        }
        const float inv = 1.0f / l;
        for (int d = 0; d < 128; ++d) output[128 * h + d] = acc[d] * inv;
    }
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
