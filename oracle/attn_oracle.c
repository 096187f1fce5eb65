/*
 * attn_oracle.c -- TEST INFRASTRUCTURE ONLY (never linked into the product).
 *
 * Plain-C restatement of the reference CPU attention path.  It follows the
 * reference's arithmetic order closely (32x256 tiles, online softmax, the
 * degree-5 exp polynomial, the 16-accumulator dot product, two-step rsqrt) so
 * that, compiled with the same flags, it agrees with the reference build to a
 * few ulps.  It is the checker the CUDA kernels are measured against; it is
 * pinned in turn against the reference itself (oracle/_ref) and against the
 * golden vectors under tests/golden/.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include "attn_oracle.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HQ     16
#define HKV    8
#define D      128
#define GROUP  2
#define TILE_Q 32   /* kernel/attention.c:48-50 */
#define TILE_K 256  /* kernel/attention.c:51-53 */
#define QSTRIDE (HQ * D)
#define KSTRIDE (HKV * D)
#define MASKED (-1e38f) /* kernel/attention.c:173, :293 */

/* exp(x): clamp to [-88, 88], n = round-half-away(x / ln 2), Cody-Waite
 * reduction r = x - n*ln2 in two steps, degree-5 Taylor polynomial by Horner,
 * then scale by 2^n through the exponent field.  kernel/attention.c:67-95. */
static inline float poly_exp(float x)
{
    if (x < -88.0f) x = -88.0f;
    if (x > 88.0f) x = 88.0f;
    float n = roundf(x * 1.4426950408889634f);
    float r = fmaf(-n, 6.93147182464599609375e-1f, x);
    r = fmaf(-n, -1.90465429995776716e-9f, r);
    float p = 1.0f / 120.0f;
    p = fmaf(r, p, 1.0f / 24.0f);
    p = fmaf(r, p, 1.0f / 6.0f);
    p = fmaf(r, p, 1.0f / 2.0f);
    p = fmaf(r, p, 1.0f);
    p = fmaf(r, p, 1.0f);
    int32_t bits = ((int32_t)n + 127) << 23;
    float two_n;
    memcpy(&two_n, &bits, sizeof two_n);
    return p * two_n;
}

/* Sum of four lanes in pairs: (a0 + a1) + (a2 + a3). */
static inline float pair_sum4(const float a[4]) { return (a[0] + a[1]) + (a[2] + a[3]); }

/* 128-long dot product with 16 fused accumulators: element i feeds
 * accumulator i mod 16; the four 4-lane groups are added pairwise, then the
 * lanes pairwise.  kernel/attention.c:100-114. */
static inline float dot128(const float *a, const float *b)
{
    float acc[16] = {0};
    for (int i = 0; i < D; i += 16)
        for (int j = 0; j < 16; j++) acc[j] = fmaf(a[i + j], b[i + j], acc[j]);
    float lanes[4];
    for (int j = 0; j < 4; j++) lanes[j] = (acc[j] + acc[4 + j]) + (acc[8 + j] + acc[12 + j]);
    return pair_sum4(lanes);
}

/* One query tile of one KV head with both of its query heads, K/V rows given
 * by base pointer + row stride.  This is the shared body of _flash_worker
 * (kernel/attention.c:252-362) and _chunked_flash_worker (:413-525); the two
 * differ only in the K/V addressing and in the causal offset. */
static void flash_tile(const float *q, const float *kbase, const float *vbase, size_t kv_row_stride,
                       float *out, int kv_h, int t_q0, int t_q1, int kv_limit, int pos_offset,
                       int Sk, float scale)
{
    float m_tile[TILE_Q], l_tile[TILE_Q];
    float *o_tile = (float *)malloc(sizeof(float) * TILE_Q * D);
    float *s_tile = (float *)malloc(sizeof(float) * TILE_Q * TILE_K);
    int tq = t_q1 - t_q0;

    for (int g = 0; g < GROUP; g++) {
        int q_h = kv_h * GROUP + g; /* kernel/attention.c:271 */
        for (int i = 0; i < tq; i++) { m_tile[i] = MASKED; l_tile[i] = 0.f; }
        memset(o_tile, 0, sizeof(float) * (size_t)tq * D);

        for (int kv_start = 0; kv_start < kv_limit; kv_start += TILE_K) {
            int kv_end = kv_start + TILE_K;
            if (kv_end > Sk) kv_end = Sk;
            int tkv = kv_end - kv_start;

            for (int i = 0; i < tq; i++) {
                int q_pos = pos_offset + t_q0 + i;
                const float *qv = q + (size_t)(t_q0 + i) * QSTRIDE + (size_t)q_h * D;
                float *sp = s_tile + i * TILE_K;
                for (int j = 0; j < tkv; j++) {
                    int k_pos = kv_start + j;
                    if (k_pos > q_pos) { sp[j] = MASKED; continue; }
                    sp[j] = dot128(qv, kbase + (size_t)k_pos * kv_row_stride) * scale;
                }
            }

            for (int i = 0; i < tq; i++) {
                float *sp = s_tile + i * TILE_K;
                float m_old = m_tile[i], m_new = m_old;
                for (int j = 0; j < tkv; j++)
                    if (sp[j] > m_new) m_new = sp[j];
                float rescale = expf(m_old - m_new);
                float l_new = l_tile[i] * rescale;
                float *oi = o_tile + (size_t)i * D;
                for (int d = 0; d < D; d++) oi[d] *= rescale;
                int j = 0;
                for (; j + 3 < tkv; j += 4) {
                    float e[4];
                    for (int u = 0; u < 4; u++) { e[u] = poly_exp(sp[j + u] - m_new); sp[j + u] = e[u]; }
                    l_new += pair_sum4(e);
                }
                for (; j < tkv; j++) { sp[j] = expf(sp[j] - m_new); l_new += sp[j]; }
                for (j = 0; j < tkv; j++) {
                    const float *vt = vbase + (size_t)(kv_start + j) * kv_row_stride;
                    float p = sp[j];
                    for (int d = 0; d < D; d++) oi[d] = fmaf(p, vt[d], oi[d]);
                }
                m_tile[i] = m_new;
                l_tile[i] = l_new;
            }
        }

        for (int i = 0; i < tq; i++) { /* kernel/attention.c:347-360 */
            float inv_l = (l_tile[i] > 0.f) ? 1.f / l_tile[i] : 0.f;
            const float *oi = o_tile + (size_t)i * D;
            float *dst = out + (size_t)(t_q0 + i) * QSTRIDE + (size_t)q_h * D;
            for (int d = 0; d < D; d++) dst[d] = oi[d] * inv_l;
        }
    }
    free(o_tile);
    free(s_tile);
}

void oracle_attention_prefill(const float *q, const float *k, const float *v, float *out, int Sq,
                              int Sk, float scale)
{
    int ntq = (Sq + TILE_Q - 1) / TILE_Q; /* kernel/attention.c:376 */
    long tasks = (long)HKV * ntq;
#pragma omp parallel for schedule(dynamic, 1)
    for (long t = 0; t < tasks; t++) {
        int kv_h = (int)(t / ntq), qt = (int)(t % ntq);
        int t_q0 = qt * TILE_Q, t_q1 = t_q0 + TILE_Q;
        if (t_q1 > Sq) t_q1 = Sq;
        /* K/V token-major: row stride 8*128, head offset kv_h*128 (:295-296). */
        flash_tile(q, k + (size_t)kv_h * D, v + (size_t)kv_h * D, KSTRIDE, out, kv_h, t_q0, t_q1,
                   t_q1, 0, Sk, scale);
    }
}

void oracle_attention_chunked_prefill(const float *q, const float *cache_k, const float *cache_v,
                                      int max_seq, float *out, int chunk_len, int pos_offset,
                                      float scale)
{
    int Sk = pos_offset + chunk_len; /* kernel/attention.c:536 */
    int ntq = (chunk_len + TILE_Q - 1) / TILE_Q;
    long tasks = (long)HKV * ntq;
#pragma omp parallel for schedule(dynamic, 1)
    for (long t = 0; t < tasks; t++) {
        int kv_h = (int)(t / ntq), qt = (int)(t % ntq);
        int t_q0 = qt * TILE_Q, t_q1 = t_q0 + TILE_Q;
        if (t_q1 > chunk_len) t_q1 = chunk_len;
        const float *kh = cache_k + (size_t)kv_h * max_seq * D;
        const float *vh = cache_v + (size_t)kv_h * max_seq * D;
        /* head-first rows, stride 128; causal end pos_offset + t_q1 (:443). */
        flash_tile(q, kh, vh, D, out, kv_h, t_q0, t_q1, pos_offset + t_q1, pos_offset, Sk, scale);
    }
}

void oracle_attention_decode(const float *q, const float *cache_k, const float *cache_v,
                             int max_seq, float *out, int kv_len, float scale)
{
#pragma omp parallel for schedule(dynamic, 1)
    for (int kv_h = 0; kv_h < HKV; kv_h++) {
        const float *K = cache_k + (size_t)kv_h * max_seq * D;
        const float *V = cache_v + (size_t)kv_h * max_seq * D;
        float *scores = (float *)malloc(sizeof(float) * (size_t)(kv_len > 0 ? kv_len : 1));
        for (int g = 0; g < GROUP; g++) { /* kernel/attention.c:169-191 */
            int q_h = kv_h * GROUP + g;
            const float *qv = q + (size_t)q_h * D;
            float mx = MASKED;
            for (int t = 0; t < kv_len; t++) {
                scores[t] = dot128(qv, K + (size_t)t * D) * scale;
                if (scores[t] > mx) mx = scores[t];
            }
            float sum = 0.f;
            for (int t = 0; t < kv_len; t++) { scores[t] = expf(scores[t] - mx); sum += scores[t]; }
            float inv = 1.f / sum;
            for (int t = 0; t < kv_len; t++) scores[t] *= inv;
            float *o = out + (size_t)q_h * D;
            memset(o, 0, sizeof(float) * D);
            for (int t = 0; t < kv_len; t++) {
                const float *vt = V + (size_t)t * D;
                for (int d = 0; d < D; d++) o[d] = fmaf(scores[t], vt[d], o[d]);
            }
        }
        free(scores);
    }
}

/* 1/sqrt(v): an 8-bit estimate refined by two Newton-Raphson steps
 * r <- r * (3 - v*r*r)/2, as kernel/ops.c:44-50 does with vrsqrte/vrsqrts. */
static float rsqrt_nr2(float v)
{
    float r = 1.0f / sqrtf(v);
    uint32_t u;
    memcpy(&u, &r, sizeof u);
    u &= 0xFFFF8000u; /* keep 8 mantissa bits: the estimate's precision */
    memcpy(&r, &u, sizeof u);
    r = r * ((3.0f - (v * r) * r) * 0.5f);
    r = r * ((3.0f - (v * r) * r) * 0.5f);
    return r;
}

void oracle_rmsnorm_rows(float *out, const float *x, const float *weight, int rows, int dim,
                         float eps)
{
#pragma omp parallel for schedule(static)
    for (int row = 0; row < rows; row++) {
        const float *xr = x + (size_t)row * dim;
        float *orow = out + (size_t)row * dim;
        /* Sum of squares: 4 lanes, element i feeds lane i mod 4 (ops.c:28-41). */
        float lane[4] = {0, 0, 0, 0};
        int i = 0;
        for (; i + 15 < dim; i += 16)
            for (int b = 0; b < 16; b += 4)
                for (int j = 0; j < 4; j++) lane[j] = fmaf(xr[i + b + j], xr[i + b + j], lane[j]);
        float ss = pair_sum4(lane);
        for (; i < dim; i++) ss += xr[i] * xr[i];
        float rs = rsqrt_nr2(ss / (float)dim + eps);
        for (i = 0; i < dim; i++) orow[i] = (xr[i] * rs) * weight[i];
    }
}

/* Interleaved M-RoPE section of frequency j (kernel/ops.c:139-155): with
 * sections [24,20,20] the first 60 frequencies cycle T,H,W; the rest are T. */
static inline int mrope_section(int j) { return j < 60 ? j % 3 : 0; }

static inline float inv_freq(int j, float theta)
{
    return 1.0f / powf(theta, (float)(2 * j) / (float)D); /* kernel/ops.c:208-211 */
}

void oracle_mrope_cos_sin_3d(float *cos_out, float *sin_out, const int *pos_ids, int seq_len,
                             float theta)
{
    float f[D / 2];
    for (int j = 0; j < D / 2; j++) f[j] = inv_freq(j, theta);
    for (int t = 0; t < seq_len; t++)
        for (int j = 0; j < D / 2; j++) {
            int pos = pos_ids[mrope_section(j) * seq_len + t];
            float ang = (float)pos * f[j];
            cos_out[(size_t)t * (D / 2) + j] = cosf(ang);
            sin_out[(size_t)t * (D / 2) + j] = sinf(ang);
        }
}

void oracle_mrope_table(float *cos_tab, float *sin_tab, int max_seq, float theta)
{
    for (int pos = 0; pos < max_seq; pos++) /* kernel/ops.c:168-180 */
        for (int j = 0; j < D / 2; j++) {
            float ang = (float)pos * inv_freq(j, theta);
            cos_tab[(size_t)pos * (D / 2) + j] = cosf(ang);
            sin_tab[(size_t)pos * (D / 2) + j] = sinf(ang);
        }
}

void oracle_rope_rows(float *x, int heads, const float *c, const float *s)
{
    for (int h = 0; h < heads; h++) { /* kernel/ops.c:248-266 */
        float *xh = x + (size_t)h * D;
        for (int j = 0; j < D / 2; j++) {
            float lo = xh[j], hi = xh[j + D / 2];
            xh[j] = lo * c[j] - hi * s[j];
            xh[j + D / 2] = hi * c[j] + lo * s[j];
        }
    }
}

void oracle_qk_norm_rope(float *q, float *k, const float *q_norm, const float *k_norm,
                         const float *token_cos, const float *token_sin, int seq_len, float eps)
{
    oracle_rmsnorm_rows(q, q, q_norm, seq_len * HQ, D, eps);  /* kernel/decoder.c:73-74 */
    oracle_rmsnorm_rows(k, k, k_norm, seq_len * HKV, D, eps); /* kernel/decoder.c:75-76 */
#pragma omp parallel for schedule(static)
    for (int t = 0; t < seq_len; t++) { /* kernel/ops.c:425-439 */
        const float *c = token_cos + (size_t)t * (D / 2);
        const float *s = token_sin + (size_t)t * (D / 2);
        oracle_rope_rows(q + (size_t)t * QSTRIDE, HQ, c, s);
        oracle_rope_rows(k + (size_t)t * KSTRIDE, HKV, c, s);
    }
}
