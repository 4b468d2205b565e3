/*
 * CPU oracle for the MoE-layer hot path.  TEST INFRASTRUCTURE ONLY: the
 * checker for the CUDA path and the timed CPU baseline, never shipped in or
 * called by the product library.  Declarations and the list of pins are in
 * moe_oracle.h.
 *
 * Build: gcc -O2 -mavx2 -mfma -ffp-contract=off -fopenmp -shared -fPIC
 * (-ffp-contract=off matters: the reference's Rust code never contracts a*b+c,
 * and its AVX2 kernels fuse exactly where they call _mm256_fmadd_ps.)
 */
#include "moe_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int all_finite(const float *v, size_t n)
{
    for (size_t i = 0; i < n; i++)
        if (!isfinite(v[i]))
            return 0;
    return 1;
}

/* --------------------------------------------------------------------------
 * Dense dot products.
 * src/backend.rs:105-120 `dot_product`: eight lane accumulators over chunks
 * of eight (separate multiply and add), lanes folded in order starting from
 * -0.0 (Rust's f32 `Sum` identity), then the tail added sequentially.
 * ------------------------------------------------------------------------ */
float oracle_dot_f32(const float *a, const float *b, size_t n)
{
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t chunks = n / 8;
    for (size_t c = 0; c < chunks; c++)
        for (int l = 0; l < 8; l++) {
            float p = a[8 * c + l] * b[8 * c + l];
            lane[l] = lane[l] + p;
        }
    float s = -0.0f;
    for (int l = 0; l < 8; l++)
        s = s + lane[l];
    for (size_t i = chunks * 8; i < n; i++) {
        float p = a[i] * b[i];
        s = s + p;
    }
    return s;
}

static inline float bf16_bits_to_f32(uint16_t v)
{
    uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* src/dense.rs:58-73 `dot_bf16`: same shape, BF16 widened exactly. */
float oracle_dot_bf16(const uint16_t *a, const float *b, size_t n)
{
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t chunks = n / 8;
    for (size_t c = 0; c < chunks; c++)
        for (int l = 0; l < 8; l++) {
            float p = bf16_bits_to_f32(a[8 * c + l]) * b[8 * c + l];
            lane[l] = lane[l] + p;
        }
    float s = -0.0f;
    for (int l = 0; l < 8; l++)
        s = s + lane[l];
    for (size_t i = chunks * 8; i < n; i++) {
        float p = bf16_bits_to_f32(a[i]) * b[i];
        s = s + p;
    }
    return s;
}

/* src/router.rs:59-62: `row.iter().zip(hidden).map(|(a, b)| a * b).sum()` */
float oracle_dot_seq(const float *a, const float *b, size_t n)
{
    float s = -0.0f;
    for (size_t i = 0; i < n; i++) {
        float p = a[i] * b[i];
        s = s + p;
    }
    return s;
}

int oracle_router_logits(const void *w, int bf16, int E, int H, const float *h,
                         float *logits)
{
    if (E <= 0 || H <= 0)
        return ORACLE_ERR_SHAPE;
    if (!all_finite(h, (size_t)H))
        return ORACLE_ERR_NONFINITE;
    for (int e = 0; e < E; e++) {
        if (bf16)
            logits[e] = oracle_dot_bf16((const uint16_t *)w + (size_t)e * H, h, H);
        else
            logits[e] = oracle_dot_f32((const float *)w + (size_t)e * H, h, H);
    }
    return all_finite(logits, (size_t)E) ? ORACLE_OK : ORACLE_ERR_NONFINITE;
}

/* src/backend.rs:375-389 `softmax`: max fold, exp(x - max) with libm expf
 * (Rust's f32::exp calls the platform expf), sequential sum, divide. */
int oracle_softmax(float *v, int n)
{
    if (!all_finite(v, (size_t)n))
        return ORACLE_ERR_NONFINITE;
    float mx = -INFINITY;
    for (int i = 0; i < n; i++)
        mx = fmaxf(mx, v[i]);
    float sum = -0.0f;
    for (int i = 0; i < n; i++) {
        v[i] = expf(v[i] - mx);
        sum = sum + v[i];
    }
    for (int i = 0; i < n; i++)
        v[i] = v[i] / sum;
    return ORACLE_OK;
}

/* src/backend.rs:341-359 `rms_norm_into`. */
int oracle_rms_norm(const float *x, const float *w, int n, float eps, float *out)
{
    if (n <= 0)
        return ORACLE_ERR_SHAPE;
    if (!all_finite(x, (size_t)n))
        return ORACLE_ERR_NONFINITE;
    float ss = oracle_dot_f32(x, x, (size_t)n);
    float scale = sqrtf(ss / (float)n + eps);
    float inv = 1.0f / scale;
    for (int i = 0; i < n; i++) {
        float t = x[i] * inv;
        out[i] = t * (w ? w[i] : 1.0f);
    }
    return all_finite(out, (size_t)n) ? ORACLE_OK : ORACLE_ERR_NONFINITE;
}

/* --------------------------------------------------------------------------
 * Top-k.  src/olmoe.rs:2595-2621: order by f32::total_cmp descending, ties to
 * the lower expert index; slot order is the sorted order.  normalizer = sum of
 * the selected probabilities in slot order when norm_topk_prob, else 1.0.
 * A stable insertion into a K-long list yields the same sequence as the
 * reference's select_nth_unstable + sort (the comparator is a total order).
 * ------------------------------------------------------------------------ */
static inline int32_t total_key(float f)
{
    int32_t i;
    memcpy(&i, &f, 4);
    /* f32::total_cmp: flip the magnitude bits of negative values. */
    return i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1);
}

static inline int ranks_before(float pa, int a, float pb, int b)
{
    int32_t ka = total_key(pa), kb = total_key(pb);
    return ka > kb || (ka == kb && a < b);
}

void oracle_topk(const float *p, int E, int K, int norm_topk_prob, uint32_t *ids,
                 float *gates)
{
    int n = 0;
    int sel[256];
    for (int e = 0; e < E; e++) {
        int pos = n;
        while (pos > 0 && ranks_before(p[e], e, p[sel[pos - 1]], sel[pos - 1]))
            pos--;
        if (pos >= K)
            continue;
        int last = n < K ? n : K - 1;
        for (int j = last; j > pos; j--)
            sel[j] = sel[j - 1];
        sel[pos] = e;
        if (n < K)
            n++;
    }
    float normalizer = 1.0f;
    if (norm_topk_prob) {
        normalizer = -0.0f;
        for (int s = 0; s < K; s++)
            normalizer = normalizer + p[sel[s]];
    }
    for (int s = 0; s < K; s++) {
        ids[s] = (uint32_t)sel[s];
        gates[s] = p[sel[s]] / normalizer;
    }
}

/* src/router.rs:84-103 `select_top_k`: sort (score desc via partial_cmp, ties
 * to the lower id), truncate to K, softmax over the K kept scores. */
void oracle_select_topk_then_softmax(const float *scores, int E, int K,
                                     uint32_t *ids, float *gates)
{
    int sel[256];
    int n = 0;
    for (int e = 0; e < E; e++) {
        int pos = n;
        while (pos > 0 && (scores[e] > scores[sel[pos - 1]]))
            pos--;
        if (pos >= K)
            continue;
        int last = n < K ? n : K - 1;
        for (int j = last; j > pos; j--)
            sel[j] = sel[j - 1];
        sel[pos] = e;
        if (n < K)
            n++;
    }
    float mx = scores[sel[0]];
    float total = -0.0f;
    float ex[256];
    for (int s = 0; s < K; s++) {
        ex[s] = expf(scores[sel[s]] - mx);
        total = total + ex[s];
    }
    for (int s = 0; s < K; s++) {
        ids[s] = (uint32_t)sel[s];
        gates[s] = ex[s] / total;
    }
}

/* --------------------------------------------------------------------------
 * INT8 x FP32 dot products (src/int8_expert.rs).
 *
 * AVX2 path, src/int8_expert.rs:380-458 (single) and :653-781 (paired; same
 * per-row arithmetic): four banks of eight lanes, each lane an FMA chain over
 * 32-element chunks; banks folded (b0+b1)+(b2+b3); leftover 8-chunks FMA'd
 * into that; 8->4->2->1 horizontal fold; scalar tail with separate mul/add.
 * ------------------------------------------------------------------------ */
__attribute__((target("avx2,fma"))) static float hfold(__m256 v)
{
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 s4 = _mm_add_ps(lo, hi);
    __m128 s2 = _mm_add_ps(s4, _mm_movehl_ps(s4, s4));
    __m128 s1 = _mm_add_ss(s2, _mm_shuffle_ps(s2, s2, 1));
    return _mm_cvtss_f32(s1);
}

__attribute__((target("avx2,fma"))) static inline __m256 widen8(const int8_t *q)
{
    long long v;
    memcpy(&v, q, 8);
    return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_cvtsi64_si128(v)));
}

__attribute__((target("avx2,fma"))) float oracle_dot_i8_avx2(const int8_t *q,
                                                             const float *x,
                                                             size_t n)
{
    __m256 b0 = _mm256_setzero_ps(), b1 = _mm256_setzero_ps();
    __m256 b2 = _mm256_setzero_ps(), b3 = _mm256_setzero_ps();
    size_t c32 = n / 32;
    for (size_t c = 0; c < c32; c++) {
        const int8_t *qq = q + 32 * c;
        const float *xx = x + 32 * c;
        b0 = _mm256_fmadd_ps(widen8(qq), _mm256_loadu_ps(xx), b0);
        b1 = _mm256_fmadd_ps(widen8(qq + 8), _mm256_loadu_ps(xx + 8), b1);
        b2 = _mm256_fmadd_ps(widen8(qq + 16), _mm256_loadu_ps(xx + 16), b2);
        b3 = _mm256_fmadd_ps(widen8(qq + 24), _mm256_loadu_ps(xx + 24), b3);
    }
    __m256 t = _mm256_add_ps(_mm256_add_ps(b0, b1), _mm256_add_ps(b2, b3));
    size_t i = 32 * c32;
    for (; i + 8 <= n; i += 8)
        t = _mm256_fmadd_ps(widen8(q + i), _mm256_loadu_ps(x + i), t);
    float s = hfold(t);
    for (; i < n; i++) {
        float p = (float)q[i] * x[i];
        s = s + p;
    }
    return s;
}

/* Scalar fallback, src/int8_expert.rs:343-376: four 8-lane banks with
 * separate mul/add, an 8-lane remainder bank, per-lane fold
 * sum += b0+b1+b2+b3+rem (left to right), then the tail. */
float oracle_dot_i8_scalar(const int8_t *q, const float *x, size_t n)
{
    float s0[8] = {0}, s1[8] = {0}, s2[8] = {0}, s3[8] = {0}, sr[8] = {0};
    size_t c32 = n / 32;
    for (size_t c = 0; c < c32; c++)
        for (int l = 0; l < 8; l++) {
            const size_t o = 32 * c;
            float p0 = (float)q[o + l] * x[o + l];
            float p1 = (float)q[o + l + 8] * x[o + l + 8];
            float p2 = (float)q[o + l + 16] * x[o + l + 16];
            float p3 = (float)q[o + l + 24] * x[o + l + 24];
            s0[l] = s0[l] + p0;
            s1[l] = s1[l] + p1;
            s2[l] = s2[l] + p2;
            s3[l] = s3[l] + p3;
        }
    size_t i = 32 * c32;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) {
            float p = (float)q[i + l] * x[i + l];
            sr[l] = sr[l] + p;
        }
    float s = 0.0f;
    for (int l = 0; l < 8; l++) {
        float t = s0[l] + s1[l];
        t = t + s2[l];
        t = t + s3[l];
        t = t + sr[l];
        s = s + t;
    }
    for (; i < n; i++) {
        float p = (float)q[i] * x[i];
        s = s + p;
    }
    return s;
}

/* --------------------------------------------------------------------------
 * INT4 x FP32 dot products (src/int8_expert.rs:473-649).  Two signed nibbles
 * per byte: element 2i is the low nibble of byte i, element 2i+1 the high
 * one, each sign-extended from 4 bits.
 *
 * AVX2 path, :519-637 `dot_i4_f32_avx2` (and the paired :785-952, whose
 * per-row arithmetic is the same): per 32 elements (16 bytes) the nibbles
 * are split, interleaved back into element order, sign-extended, and FMA'd
 * into four 8-lane banks; then the INT8 path's fold, 8-chunks, horizontal
 * fold and scalar tail.
 * ------------------------------------------------------------------------ */
__attribute__((target("avx2,fma"))) static inline __m256 widen8_i4(const uint8_t *q)
{
    /* 4 bytes -> 8 sign-extended nibbles in element order (:586-604) */
    long long v = 0;
    for (int b = 0; b < 4; b++) {
        int lo = (int8_t)(q[b] << 4) >> 4, hi = (int8_t)q[b] >> 4;
        v |= (long long)(uint8_t)lo << (16 * b);
        v |= (long long)(uint8_t)hi << (16 * b + 8);
    }
    return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_cvtsi64_si128(v)));
}

__attribute__((target("avx2,fma"))) float oracle_dot_i4_avx2(const uint8_t *q,
                                                             const float *x,
                                                             size_t n)
{
    __m256 b0 = _mm256_setzero_ps(), b1 = _mm256_setzero_ps();
    __m256 b2 = _mm256_setzero_ps(), b3 = _mm256_setzero_ps();
    const __m128i m0f = _mm_set1_epi8(0x0F), c8 = _mm_set1_epi8(8);
    size_t c32 = n / 32;
    for (size_t c = 0; c < c32; c++) {
        const __m128i v = _mm_loadu_si128((const __m128i *)(q + 16 * c));
        const __m128i lo = _mm_and_si128(v, m0f);
        const __m128i hi = _mm_and_si128(_mm_srli_epi16(v, 4), m0f);
        const __m128i s_lo = _mm_sub_epi8(_mm_xor_si128(_mm_unpacklo_epi8(lo, hi), c8), c8);
        const __m128i s_hi = _mm_sub_epi8(_mm_xor_si128(_mm_unpackhi_epi8(lo, hi), c8), c8);
        const float *xx = x + 32 * c;
        b0 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(s_lo)),
                             _mm256_loadu_ps(xx), b0);
        b1 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(s_lo, 8))),
                             _mm256_loadu_ps(xx + 8), b1);
        b2 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(s_hi)),
                             _mm256_loadu_ps(xx + 16), b2);
        b3 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(s_hi, 8))),
                             _mm256_loadu_ps(xx + 24), b3);
    }
    __m256 t = _mm256_add_ps(_mm256_add_ps(b0, b1), _mm256_add_ps(b2, b3));
    size_t i = 32 * c32;
    for (; i + 8 <= n; i += 8)
        t = _mm256_fmadd_ps(widen8_i4(q + i / 2), _mm256_loadu_ps(x + i), t);
    float s = hfold(t);
    for (; i < n; i++) {
        const uint8_t b = q[i / 2];
        const int v = (i & 1) ? (int8_t)b >> 4 : (int8_t)(b << 4) >> 4;
        float p = (float)v * x[i];
        s = s + p;
    }
    return s;
}

/* Scalar fallback, :476-516: four scalar accumulators, each taking a pair
 * of products per 8-chunk, s0 + s1 + s2 + s3 left to right, then the tail. */
float oracle_dot_i4_scalar(const uint8_t *q, const float *x, size_t n)
{
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    size_t c8 = n / 8;
    for (size_t c = 0; c < c8; c++)
        for (int k = 0; k < 4; k++) {
            const uint8_t b = q[4 * c + k];
            const float a = (float)((int8_t)(b << 4) >> 4) * x[8 * c + 2 * k];
            const float d = (float)((int8_t)b >> 4) * x[8 * c + 2 * k + 1];
            const float pair = a + d;
            s[k] = s[k] + pair;
        }
    float sum = s[0] + s[1];
    sum = sum + s[2];
    sum = sum + s[3];
    for (size_t i = 8 * c8; i < n; i++) {
        const uint8_t b = q[i / 2];
        const int v = (i & 1) ? (int8_t)b >> 4 : (int8_t)(b << 4) >> 4;
        float p = (float)v * x[i];
        sum = sum + p;
    }
    return sum;
}

static int have_avx2(void)
{
    static int cached = -1;
    if (cached < 0) {
        __builtin_cpu_init();
        cached = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
    }
    return cached;
}

/* mode 0 = the AVX2 path when the CPU has it, else the scalar fallback;
 * int4: rows are packed nibbles (n/2 bytes). */
static inline float dot_q(const int8_t *q, const float *x, size_t n, int mode, int int4)
{
    if (int4)
        return (mode == 0 && have_avx2()) ? oracle_dot_i4_avx2((const uint8_t *)q, x, n)
                                          : oracle_dot_i4_scalar((const uint8_t *)q, x, n);
    return (mode == 0 && have_avx2()) ? oracle_dot_i8_avx2(q, x, n)
                                      : oracle_dot_i8_scalar(q, x, n);
}

/* src/int8_expert.rs:1058-1101 lane body: g = dot*sg, u = dot*su,
 * act = (g / (1 + exp(-g))) * u. */
static inline float swiglu_row(const int8_t *wg, const int8_t *wu, float sg, float su,
                               const float *x, int H, int mode, int int4)
{
    float g = dot_q(wg, x, (size_t)H, mode, int4) * sg;
    float u = dot_q(wu, x, (size_t)H, mode, int4) * su;
    float den = 1.0f + expf(-g);
    float silu = g / den;
    return silu * u;
}

/* Int8Expert::forward_single_threaded, src/int8_expert.rs:301-338; INT4
 * rows are H/2 (gate, up) and I/2 (down) bytes (:312-316). */
int oracle_expert_forward_q(const int8_t *w, const float *s, int H, int I, const float *x,
                            float *act, float *y, int mode, int int4)
{
    if (H <= 0 || I <= 0 || (int4 && ((H | I) & 1)))
        return ORACLE_ERR_SHAPE;
    if (!all_finite(x, (size_t)H))
        return ORACLE_ERR_NONFINITE;
    const size_t hs = int4 ? (size_t)H / 2 : (size_t)H, is = int4 ? (size_t)I / 2 : (size_t)I;
    const size_t n = hs * I;
    for (int r = 0; r < I; r++)
        act[r] = swiglu_row(w + (size_t)r * hs, w + n + (size_t)r * hs, s[r], s[I + r], x,
                            H, mode, int4);
    for (int r = 0; r < H; r++)
        y[r] = dot_q(w + 2 * n + (size_t)r * is, act, (size_t)I, mode, int4) * s[2 * I + r];
    return all_finite(y, (size_t)H) ? ORACLE_OK : ORACLE_ERR_NONFINITE;
}

int oracle_expert_forward(const int8_t *w, const float *s, int H, int I,
                          const float *x, float *act, float *y, int mode)
{
    return oracle_expert_forward_q(w, s, H, I, x, act, y, mode, 0);
}

/* Int8Expert::forward_reuse (src/int8_expert.rs:260-297): the same rows,
 * computed row-parallel (the reference uses Rayon par_iter_mut when the
 * matrix has >= 262,144 weights). */
static int expert_forward_rows_parallel(const int8_t *w, const float *s, int H, int I,
                                        const float *x, float *act, float *y, int mode,
                                        int nthreads, int int4)
{
    if (!all_finite(x, (size_t)H))
        return ORACLE_ERR_NONFINITE;
    const size_t hs = int4 ? (size_t)H / 2 : (size_t)H, is = int4 ? (size_t)I / 2 : (size_t)I;
    const size_t n = hs * I;
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int r = 0; r < I; r++)
        act[r] = swiglu_row(w + (size_t)r * hs, w + n + (size_t)r * hs, s[r], s[I + r], x,
                            H, mode, int4);
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int r = 0; r < H; r++)
        y[r] = dot_q(w + 2 * n + (size_t)r * is, act, (size_t)I, mode, int4) * s[2 * I + r];
    return all_finite(y, (size_t)H) ? ORACLE_OK : ORACLE_ERR_NONFINITE;
}

/* --------------------------------------------------------------------------
 * Table-driven expf restatement (the CUDA path's softmax exponential).
 * Published method: exp(x) = 2^(k/32) * P(r), k = round(x*32/ln2),
 * r = x*32/ln2 - k, P a degree-3 polynomial in r evaluated with FMAs in
 * double precision (Szabolcs Nagy's expf design in ARM optimized-routines,
 * also glibc's expf since 2.28).  The 2^(i/32) table is computed at load
 * time here (and in Python for the CUDA constant table) rather than typed in.
 * ------------------------------------------------------------------------ */
static double g_pow2_tab[32];
static int g_pow2_ready = 0;

static void pow2_init(void)
{
    if (g_pow2_ready)
        return;
    for (int i = 0; i < 32; i++)
        g_pow2_tab[i] = (double)exp2l((long double)i / 32.0L);
    g_pow2_ready = 1;
}

float oracle_expf_table(float x)
{
    pow2_init();
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
    const double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    if (x < -0x1.9fe368p6f)
        return 0.0f;
    if (x > 0x1.62e42ep6f)
        return INFINITY;
    double xd = (double)x;
    double kd = fma(inv_ln2_n, xd, shift);
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= shift;
    double r = fma(inv_ln2_n, xd, -kd);
    double base = g_pow2_tab[ki & 31];
    uint64_t bb;
    memcpy(&bb, &base, 8);
    bb += (ki >> 5) << 52; /* scale by 2^(k div 32); k fits comfortably */
    double sc;
    memcpy(&sc, &bb, 8);
    double z = fma(c0, r, c1);
    double r2 = r * r;
    double y = fma(c2, r, 1.0);
    y = fma(z, r2, y);
    y = y * sc;
    return (float)y;
}

uint64_t oracle_expf_table_mismatches(uint32_t bits_lo, uint32_t bits_hi, uint32_t stride)
{
    uint64_t bad = 0;
    if (stride == 0)
        stride = 1;
    for (uint64_t b = bits_lo; b <= bits_hi; b += stride) {
        uint32_t u = (uint32_t)b;
        float x;
        memcpy(&x, &u, 4);
        float a = expf(x), c = oracle_expf_table(x);
        if (memcmp(&a, &c, 4) != 0)
            bad++;
    }
    return bad;
}

/* --------------------------------------------------------------------------
 * One MoE layer.
 * Routing per token: src/olmoe.rs:2589-2621 (decode) and :3421-3466 (prefill).
 * Combine: x[j] += (w * y[j]) slot by slot (src/olmoe.rs:3147-3157); the
 * prefill path stores w*y in `contributions` then adds them per token in
 * slot order (:3551-3563, :3702-3714), which is the same arithmetic.
 * ------------------------------------------------------------------------ */
static int route_token(const oracle_layer *L, const float *h, uint32_t *ids, float *gates)
{
    float logits[256];
    int st = oracle_router_logits(L->router, L->router_bf16, L->E, L->H, h, logits);
    if (st)
        return st;
    st = oracle_softmax(logits, L->E);
    if (st)
        return st;
    oracle_topk(logits, L->E, L->K, L->norm_topk_prob, ids, gates);
    return ORACLE_OK;
}

int oracle_layer_forward(const oracle_layer *L, int T, const float *h,
                         const float *resid, float *out, uint32_t *ids_out,
                         float *gates_out, int32_t *seg_off, int32_t *use_token,
                         int32_t *use_slot, float *use_gate, int mode, int nthreads)
{
    const int H = L->H, I = L->I, E = L->E, K = L->K;
    if (H <= 0 || I <= 0 || E <= 0 || K <= 0 || K > E || E > 256 || T < 0)
        return ORACLE_ERR_SHAPE;
    if (nthreads < 1)
        nthreads = 1;
    if (L->int4 && ((H | I) & 1))
        return ORACLE_ERR_SHAPE;
    const size_t wpe = (size_t)3 * H * I / (L->int4 ? 2 : 1), spe = (size_t)2 * I + H;
    uint32_t *ids = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)T * K + 4);
    float *gates = (float *)malloc(sizeof(float) * (size_t)T * K + 4);
    int st = ORACLE_OK;
    for (int t = 0; t < T && !st; t++)
        st = route_token(L, h + (size_t)t * H, ids + (size_t)t * K, gates + (size_t)t * K);
    if (st)
        goto done;

    /* expert_uses: bucket routes by expert id, tokens ascending inside. */
    if (seg_off) {
        int32_t *cnt = (int32_t *)calloc((size_t)E + 1, sizeof(int32_t));
        for (size_t r = 0; r < (size_t)T * K; r++)
            cnt[ids[r] + 1]++;
        for (int e = 0; e < E; e++)
            cnt[e + 1] += cnt[e];
        memcpy(seg_off, cnt, sizeof(int32_t) * ((size_t)E + 1));
        for (int t = 0; t < T; t++)
            for (int s = 0; s < K; s++) {
                uint32_t e = ids[(size_t)t * K + s];
                int32_t pos = cnt[e]++;
                if (use_token)
                    use_token[pos] = t;
                if (use_slot)
                    use_slot[pos] = s;
                if (use_gate)
                    use_gate[pos] = gates[(size_t)t * K + s];
            }
        free(cnt);
    }

    for (size_t i = 0; i < (size_t)T * H; i++)
        out[i] = resid ? resid[i] : 0.0f;

    float *act = (float *)malloc(sizeof(float) * (size_t)I * K);
    float *y = (float *)malloc(sizeof(float) * (size_t)H * K);
    /* mode bit 1 forces the decode schedule (stacked decode configs) */
    int prefill = T > 1 && nthreads > 1 && !(mode & 2);
    mode &= 1;
    if (!prefill) {
        /* Decode schedule: every token independently, its K experts one per
         * worker, then the slot-ordered combine. */
        for (int t = 0; t < T && !st; t++) {
            const float *ht = h + (size_t)t * H;
            int errs = 0;
#pragma omp parallel for num_threads(nthreads) schedule(static, 1) reduction(| : errs)
            for (int s = 0; s < K; s++) {
                uint32_t e = ids[(size_t)t * K + s];
                errs |= oracle_expert_forward_q(L->experts + wpe * e, L->scales + spe * e, H, I,
                                                ht, act + (size_t)s * I, y + (size_t)s * H,
                                                mode, L->int4);
            }
            if (errs) {
                st = ORACLE_ERR_NONFINITE;
                break;
            }
            float *ot = out + (size_t)t * H;
            for (int s = 0; s < K; s++) {
                float w = gates[(size_t)t * K + s];
                const float *ys = y + (size_t)s * H;
                for (int j = 0; j < H; j++) {
                    float c = w * ys[j];
                    ot[j] = ot[j] + c;
                }
            }
        }
    } else {
        /* Prefill schedule: experts in ascending id, their tokens in order,
         * each token's expert forward row-parallel; contributions then the
         * per-token slot-ordered sum. */
        float *contrib = (float *)malloc(sizeof(float) * (size_t)T * K * H);
        int32_t *cnt = (int32_t *)calloc((size_t)E + 1, sizeof(int32_t));
        int32_t *tok = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * K);
        int32_t *slot = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * K);
        for (size_t r = 0; r < (size_t)T * K; r++)
            cnt[ids[r] + 1]++;
        for (int e = 0; e < E; e++)
            cnt[e + 1] += cnt[e];
        int32_t *fill = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
        memcpy(fill, cnt, sizeof(int32_t) * (size_t)E);
        for (int t = 0; t < T; t++)
            for (int s = 0; s < K; s++) {
                uint32_t e = ids[(size_t)t * K + s];
                int32_t pos = fill[e]++;
                tok[pos] = t;
                slot[pos] = s;
            }
        for (int e = 0; e < E && !st; e++) {
            for (int32_t u = cnt[e]; u < cnt[e + 1] && !st; u++) {
                int t = tok[u], s = slot[u];
                st = expert_forward_rows_parallel(L->experts + wpe * e, L->scales + spe * e, H,
                                                  I, h + (size_t)t * H, act, y, mode,
                                                  nthreads, L->int4);
                float w = gates[(size_t)t * K + s];
                float *c = contrib + ((size_t)t * K + s) * H;
                for (int j = 0; j < H; j++)
                    c[j] = w * y[j];
            }
        }
        for (int t = 0; t < T && !st; t++)
            for (int s = 0; s < K; s++) {
                const float *c = contrib + ((size_t)t * K + s) * H;
                float *ot = out + (size_t)t * H;
                for (int j = 0; j < H; j++)
                    ot[j] = ot[j] + c[j];
            }
        free(contrib);
        free(cnt);
        free(tok);
        free(slot);
        free(fill);
    }
    if (!st && !all_finite(out, (size_t)T * H))
        st = ORACLE_ERR_NONFINITE;
    free(act);
    free(y);
done:
    if (!st && ids_out)
        memcpy(ids_out, ids, sizeof(uint32_t) * (size_t)T * K);
    if (!st && gates_out)
        memcpy(gates_out, gates, sizeof(float) * (size_t)T * K);
    free(ids);
    free(gates);
    return st;
}

int oracle_stack_forward(const oracle_layer *layers, int nlayers, int T, float *x,
                         float eps, uint32_t *ids, float *gates, int mode, int nthreads)
{
    if (nlayers <= 0 || T <= 0)
        return ORACLE_ERR_SHAPE;
    const int H = layers[0].H, K = layers[0].K;
    float *h = (float *)malloc(sizeof(float) * (size_t)T * H);
    float *nx = (float *)malloc(sizeof(float) * (size_t)T * H);
    int st = ORACLE_OK;
    for (int l = 0; l < nlayers && !st; l++) {
        for (int t = 0; t < T && !st; t++)
            st = oracle_rms_norm(x + (size_t)t * H, layers[l].norm_w, H, eps,
                                 h + (size_t)t * H);
        if (st)
            break;
        st = oracle_layer_forward(&layers[l], T, h, x, nx,
                                  ids ? ids + (size_t)l * T * K : NULL,
                                  gates ? gates + (size_t)l * T * K : NULL, NULL, NULL, NULL,
                                  NULL, mode | 2, nthreads > 1 ? nthreads : 1);
        memcpy(x, nx, sizeof(float) * (size_t)T * H);
    }
    free(h);
    free(nx);
    return st;
}

/* --------------------------------------------------------------------------
 * Seeded synthetic inputs.  Integer-only derivations (weights, scales) are
 * shared bit-for-bit with the CUDA generator; normals are host-only.
 * ------------------------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

uint64_t oracle_synth_key(uint64_t seed, uint32_t kind, uint32_t layer, uint32_t expert)
{
    uint64_t k = mix64(seed ^ 0x6a09e667f3bcc909ULL);
    return mix64(k ^ ((uint64_t)kind << 48) ^ ((uint64_t)layer << 24) ^ (uint64_t)expert);
}

static inline uint64_t rng_at(uint64_t key, uint64_t i)
{
    return mix64(key + (i + 1) * 0x9E3779B97F4A7C15ULL);
}

void oracle_synth_expert(uint64_t seed, int layer, int expert, int H, int I, int8_t *w,
                         float *s)
{
    const size_t nw = (size_t)3 * H * I, ns = (size_t)2 * I + H;
    uint64_t kw = oracle_synth_key(seed, 1, (uint32_t)layer, (uint32_t)expert);
    uint64_t ks = oracle_synth_key(seed, 2, (uint32_t)layer, (uint32_t)expert);
#pragma omp parallel for schedule(static)
    for (size_t j = 0; j < (nw + 3) / 4; j++) {
        uint64_t u = rng_at(kw, j);
        for (int b = 0; b < 4 && 4 * j + b < nw; b++) {
            uint32_t piece = (uint32_t)(u >> (16 * b)) & 0xffffu;
            w[4 * j + b] = (int8_t)((int)((piece * 255u) >> 16) - 127);
        }
    }
    for (size_t r = 0; r < ns; r++) {
        float f = (float)(rng_at(ks, r) >> 40) * 0x1p-24f;
        float t = f * 9e-4f;
        s[r] = 1e-4f + t;
    }
}

void oracle_synth_normal(uint64_t seed, uint32_t kind, uint32_t layer, size_t n,
                         float stddev, float *out)
{
    uint64_t k = oracle_synth_key(seed, kind, layer, 0);
    for (size_t j = 0; 2 * j < n; j++) {
        double a = (double)((rng_at(k, 2 * j) >> 11) + 1) * 0x1p-53;
        double b = (double)(rng_at(k, 2 * j + 1) >> 11) * 0x1p-53;
        double r = sqrt(-2.0 * log(a));
        double th = 6.283185307179586 * b;
        out[2 * j] = (float)((double)stddev * r * cos(th));
        if (2 * j + 1 < n)
            out[2 * j + 1] = (float)((double)stddev * r * sin(th));
    }
}

/* --------------------------------------------------------------------------
 * Generators of the reference's own kernel tests, restated so their cases can
 * be replayed against the CUDA path.
 * src/gpu_expert.rs:517-530: xorshift32 (13, 17, 5) seeded seed*2654435761
 * (at least 1); weights (next % 255) as u8 reinterpreted as i8 by the kernel;
 * scales 0.002 + (next % 1000) * 1e-5.
 * ------------------------------------------------------------------------ */
void oracle_gen_xorshift32_expert(uint32_t seed, int H, int I, int8_t *w, float *s)
{
    uint32_t st = seed * 2654435761u;
    if (st < 1)
        st = 1;
#define NEXT32() (st ^= st << 13, st ^= st >> 17, st ^= st << 5, st)
    for (size_t k = 0; k < (size_t)3 * H * I; k++) {
        uint32_t v = NEXT32();
        w[k] = (int8_t)(uint8_t)(v % 255u);
    }
    for (size_t r = 0; r < (size_t)2 * I + H; r++) {
        uint32_t v = NEXT32();
        float t = (float)(v % 1000u) * 1e-5f;
        s[r] = 0.002f + t;
    }
#undef NEXT32
}

/* src/int8_expert.rs:1188-1229 (GateUpBenchCase::new): xorshift64 (13, 7, 17)
 * from `seed`; weights `next() as u8`; scales
 * (0.5 + (next % 1000)/1000) / (127 * sqrt(cols)); input (next % 2001)/1000 - 1. */
void oracle_gen_xorshift64_case(uint64_t seed, int H, int I, int8_t *w, float *s, float *x)
{
    uint64_t st = seed;
#define NEXT64() (st ^= st << 13, st ^= st >> 7, st ^= st << 17, st)
    for (size_t k = 0; k < (size_t)3 * H * I; k++)
        w[k] = (int8_t)(uint8_t)NEXT64();
    for (size_t r = 0; r < (size_t)2 * I + H; r++) {
        int cols = r < (size_t)2 * I ? H : I;
        float f = (float)(NEXT64() % 1000u) / 1000.0f;
        float num = 0.5f + f;
        float den = 127.0f * sqrtf((float)cols);
        s[r] = num / den;
    }
    for (int c = 0; c < H; c++) {
        float f = (float)(NEXT64() % 2001u) / 1000.0f;
        x[c] = f - 1.0f;
    }
#undef NEXT64
}

/* libm expf over consecutive float bit patterns (the comparator for the
 * device exponential). */
void oracle_expf_libm_range(uint32_t bits_lo, size_t count, float *out)
{
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < count; i++) {
        uint32_t u = bits_lo + (uint32_t)i;
        float x;
        memcpy(&x, &u, 4);
        out[i] = expf(x);
    }
}
