/*
 * tos_oracle.c - CPU restatement of TensorOS runtime/nn's decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see tos_oracle.h).  Written from the reference's
 * behaviour, not copied: each function names the reference lines whose fp32
 * operation order it reproduces.  Lane-parallel SSE2 code in the reference is
 * restated with explicit per-lane scalar arrays; IEEE fp32 add/mul are
 * lane-wise, so the results are identical.  Build with
 *   gcc -std=gnu11 -O2 -msse2 -mno-fma -ffp-contract=off
 * (no FMA contraction, no excess precision).
 */
#include "tos_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* fp16 -> fp32, exact incl. subnormals, +-0, Inf/NaN: llm.c:71-104 */
float orc_fp16_to_fp32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0x1F) return bits_f(sign | 0x7F800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return bits_f(sign);
        /* subnormal: value = m * 2^-24, normalise */
        int sh = 0;
        while (!(m & 0x400u)) { m <<= 1; sh++; }
        m &= 0x3FFu;
        return bits_f(sign | ((uint32_t)(113 - sh) << 23) | (m << 13));
    }
    return bits_f(sign | ((e + 112u) << 23) | (m << 13));
}

/* fp32 -> fp16, round to nearest even (IEEE), used for the fp16 KV cache
 * (no reference counterpart: the reference cache is fp32, llm.h:100-101). */
uint16_t orc_fp32_to_fp16(float f)
{
    uint32_t x = f_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) {
        if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((a >> 13) & 0x3FFu));
        return (uint16_t)(sign | 0x7C00u);
    }
    int e = (int)(a >> 23);
    if (e < 113) {                       /* below 2^-14: fp16 subnormal or zero */
        int shift = 126 - e;
        if (shift > 24) return sign;
        uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        if (e == 0) return sign;         /* fp32 subnormal: far below 2^-25 */
        uint32_t r = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    int e16 = e - 112;
    if (e16 >= 31) return (uint16_t)(sign | 0x7C00u);
    uint32_t base = ((uint32_t)e16 << 10) | ((a >> 13) & 0x3FFu);
    uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (base & 1u))) base++;
    return (uint16_t)(sign | base);
}

/* llm.c:123-131: (1 + x/256)^256 by eight squarings, clamped at +-88 */
float orc_expf(float x)
{
    if (x > 88.0f) return 3.4e38f;
    if (x < -88.0f) return 0.0f;
    float y = 1.0f + x / 256.0f;
    for (int i = 0; i < 8; i++) y = y * y;
    return y;
}

/* llm.c:112-121: IEEE square root (sqrtss) */
float orc_sqrtf(float x) { return sqrtf(x); }

/* Q4_0 block dot, llm.c:148-174.  Element 2j is the low nibble of qs[j],
 * 2j+1 the high nibble, value (nibble-8).  Chain c (0..7) of the two 4-lane
 * accumulators takes elements 8k+c, k = 0..3, starting from +0.0f.  Then
 * t_l = chain_l + chain_{l+4}, r = ((t0+t1)+t2)+t3, result r*d. */
float orc_q4_0_dot32(const void *block, const float *x)
{
    const uint8_t *p = (const uint8_t *)block;
    uint16_t hd = (uint16_t)(p[0] | (p[1] << 8));
    float d = orc_fp16_to_fp32(hd);
    const uint8_t *qs = p + 2;
    float ch[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < 4; k++) {
        for (int c = 0; c < 8; c++) {
            int e = 8 * k + c;
            uint8_t byte = qs[e >> 1];
            int nib = (e & 1) ? (byte >> 4) : (byte & 0x0F);
            float q = (float)(nib - 8);
            float prod = q * x[e];
            ch[c] = ch[c] + prod;
        }
    }
    float t0 = ch[0] + ch[4], t1 = ch[1] + ch[5], t2 = ch[2] + ch[6], t3 = ch[3] + ch[7];
    float r = ((t0 + t1) + t2) + t3;
    return r * d;
}

/* Q8_0 block dot, llm.c:187-209: same lane tree over int8 values. */
float orc_q8_0_dot32(const void *block, const float *x)
{
    const uint8_t *p = (const uint8_t *)block;
    uint16_t hd = (uint16_t)(p[0] | (p[1] << 8));
    float d = orc_fp16_to_fp32(hd);
    const int8_t *qs = (const int8_t *)(p + 2);
    float ch[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < 4; k++) {
        for (int c = 0; c < 8; c++) {
            int e = 8 * k + c;
            float prod = (float)qs[e] * x[e];
            ch[c] = ch[c] + prod;
        }
    }
    float t0 = ch[0] + ch[4], t1 = ch[1] + ch[5], t2 = ch[2] + ch[6], t3 = ch[3] + ch[7];
    float r = ((t0 + t1) + t2) + t3;
    return r * d;
}

/* llm.c:221-289: serial fp32 sum over blocks (Q4_0/Q8_0); F16 uses one 4-lane
 * accumulator then a left-to-right horizontal sum and a scalar tail; F32 uses
 * the 8-wide two-accumulator tree.  Unknown types give 0. */
float orc_vec_dot(const void *w, const float *x, int n, int type)
{
    float sum = 0.0f;
    int nb = n / 32;
    if (type == ORC_TYPE_Q4_0) {
        const uint8_t *b = (const uint8_t *)w;
        for (int i = 0; i < nb; i++) sum = sum + orc_q4_0_dot32(b + 18 * (size_t)i, x + 32 * i);
    } else if (type == ORC_TYPE_Q8_0) {
        const uint8_t *b = (const uint8_t *)w;
        for (int i = 0; i < nb; i++) sum = sum + orc_q8_0_dot32(b + 34 * (size_t)i, x + 32 * i);
    } else if (type == ORC_TYPE_F16) {
        const uint16_t *h = (const uint16_t *)w;
        float acc[4] = {0, 0, 0, 0};
        int i = 0;
        for (; i + 4 <= n; i += 4)
            for (int l = 0; l < 4; l++) acc[l] = acc[l] + orc_fp16_to_fp32(h[i + l]) * x[i + l];
        sum = sum + (((acc[0] + acc[1]) + acc[2]) + acc[3]);
        for (; i < n; i++) sum = sum + orc_fp16_to_fp32(h[i]) * x[i];
    } else if (type == ORC_TYPE_F32) {
        const float *f = (const float *)w;
        float a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= n; i += 8)
            for (int l = 0; l < 4; l++) {
                a0[l] = a0[l] + f[i + l] * x[i + l];
                a1[l] = a1[l] + f[i + 4 + l] * x[i + 4 + l];
            }
        float t[4];
        for (int l = 0; l < 4; l++) t[l] = a0[l] + a1[l];
        sum = sum + (((t[0] + t[1]) + t[2]) + t[3]);
        for (; i < n; i++) sum = sum + f[i] * x[i];
    }
    return sum;
}

/* llm.c:292-301 */
size_t orc_row_bytes(int in_dim, int type)
{
    switch (type) {
    case ORC_TYPE_Q4_0: return (size_t)(in_dim / 32) * 18;
    case ORC_TYPE_Q8_0: return (size_t)(in_dim / 32) * 34;
    case ORC_TYPE_F16: return (size_t)in_dim * 2;
    default: return (size_t)in_dim * 4;
    }
}

/* llm.c:329-349 (C path; the x86 JIT of llm.c:332-341 is not the oracle) */
void orc_gemv(float *out, const void *w, const float *x, int out_dim, int in_dim, int type)
{
    size_t rb = orc_row_bytes(in_dim, type);
    for (int i = 0; i < out_dim; i++)
        out[i] = orc_vec_dot((const uint8_t *)w + rb * (size_t)i, x, in_dim, type);
}

typedef struct {
    float *out; const void *w; const float *x;
    int r0, r1, in_dim, type;
} gemv_job_t;

static void *gemv_worker(void *arg)
{
    gemv_job_t *j = (gemv_job_t *)arg;
    size_t rb = orc_row_bytes(j->in_dim, j->type);
    for (int i = j->r0; i < j->r1; i++)
        j->out[i] = orc_vec_dot((const uint8_t *)j->w + rb * (size_t)i, j->x, j->in_dim, j->type);
    return NULL;
}

/* Same result as orc_gemv (rows are independent); rows split over threads. */
void orc_gemv_threads(float *out, const void *w, const float *x, int out_dim, int in_dim,
                      int type, int n_threads)
{
    if (n_threads <= 1 || out_dim < 64) { orc_gemv(out, w, x, out_dim, in_dim, type); return; }
    if (n_threads > 64) n_threads = 64;
    pthread_t th[64];
    gemv_job_t jobs[64];
    for (int t = 0; t < n_threads; t++) {
        jobs[t].out = out; jobs[t].w = w; jobs[t].x = x;
        jobs[t].r0 = (int)((long long)out_dim * t / n_threads);
        jobs[t].r1 = (int)((long long)out_dim * (t + 1) / n_threads);
        jobs[t].in_dim = in_dim; jobs[t].type = type;
        pthread_create(&th[t], NULL, gemv_worker, &jobs[t]);
    }
    for (int t = 0; t < n_threads; t++) pthread_join(th[t], NULL);
}

/* llm.c:352-362 */
static float get_f(const void *data, int idx, int type)
{
    if (type == ORC_TYPE_F32) return ((const float *)data)[idx];
    if (type == ORC_TYPE_F16) return orc_fp16_to_fp32(((const uint16_t *)data)[idx]);
    return 0.0f;
}

/* llm.c:365-410: dequantise one embedding row */
void orc_embed(float *out, const void *embd, int type, int dim, int token)
{
    const uint8_t *row = (const uint8_t *)embd + orc_row_bytes(dim, type) * (size_t)token;
    if (type == ORC_TYPE_F32) {
        for (int i = 0; i < dim; i++) out[i] = ((const float *)row)[i];
    } else if (type == ORC_TYPE_F16) {
        for (int i = 0; i < dim; i++) out[i] = orc_fp16_to_fp32(((const uint16_t *)row)[i]);
    } else if (type == ORC_TYPE_Q4_0) {
        for (int b = 0; b < dim / 32; b++) {
            const uint8_t *blk = row + 18 * (size_t)b;
            float d = orc_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int j = 0; j < 16; j++) {
                out[32 * b + 2 * j] = (float)((blk[2 + j] & 0x0F) - 8) * d;
                out[32 * b + 2 * j + 1] = (float)((blk[2 + j] >> 4) - 8) * d;
            }
        }
    } else if (type == ORC_TYPE_Q8_0) {
        for (int b = 0; b < dim / 32; b++) {
            const uint8_t *blk = row + 34 * (size_t)b;
            float d = orc_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int j = 0; j < 32; j++) out[32 * b + j] = (float)(int8_t)blk[2 + j] * d;
        }
    } else {
        for (int i = 0; i < dim; i++) out[i] = 0.0f;
    }
}

/* llm.c:416-442: four serial lane sums of x^2 (lane = i mod 4), combined
 * left to right, scalar tail, ss = 1/sqrt(ss/dim + eps), out = (x*ss)*w.
 * The reference fixes eps = 1e-6f (llm.c:431). */
void orc_rmsnorm(float *out, const float *x, const void *w, int wtype, int dim, float eps)
{
    float lane[4] = {0, 0, 0, 0};
    int i = 0;
    for (; i + 4 <= dim; i += 4)
        for (int l = 0; l < 4; l++) lane[l] = lane[l] + x[i + l] * x[i + l];
    float ss = ((lane[0] + lane[1]) + lane[2]) + lane[3];
    for (; i < dim; i++) ss = ss + x[i] * x[i];
    ss = 1.0f / orc_sqrtf(ss / (float)dim + eps);
    for (i = 0; i < dim; i++) out[i] = (x[i] * ss) * get_f(w, i, wtype);
}

/* llm.c:460-492: the cos/sin pair for element pair i of a head at pos.
 * ln(base) by halving + cubic series, frequency through orc_expf, angle
 * reduced by repeated +-2*pi in fp32, then Taylor cos/sin. */
void orc_rope_cs(int pos, int i, int head_dim, float base, float *cos_out, float *sin_out)
{
    float exponent = -(float)i / (float)head_dim;
    float b = base;
    int k = 0;
    while (b > 2.0f) { b *= 0.5f; k++; }
    float m1 = b - 1.0f;
    float log_base = (float)k * 0.6931472f + m1 * (1.0f - m1 * (0.5f - m1 * 0.3333f));
    float freq = orc_expf(exponent * log_base);
    float theta = (float)pos * freq;
    const float pi = 3.14159265f;
    const float two_pi = 2.0f * pi;
    while (theta > pi) theta -= two_pi;
    while (theta < -pi) theta += two_pi;
    float t2 = theta * theta;
    *cos_out = 1.0f - t2 * (0.5f - t2 * (0.04166667f - t2 * 0.001388889f));
    *sin_out = theta * (1.0f - t2 * (0.1666667f - t2 * (0.008333333f - t2 * 0.000198413f)));
}

/* llm.c:460-500: rotate adjacent pairs (v[i], v[i+1]) */
void orc_rope(float *vec, int pos, int head_dim, float base)
{
    for (int i = 0; i < head_dim; i += 2) {
        float c, s;
        orc_rope_cs(pos, i, head_dim, base, &c, &s);
        float v0 = vec[i], v1 = vec[i + 1];
        vec[i] = v0 * c - v1 * s;
        vec[i + 1] = v0 * s + v1 * c;
    }
}

/* llm_rope applied to every head of n_rows rows of length row_len (heads of
 * hd elements), row r at position pos[r] (llm.c:668-671 per position). */
void orc_rope_rows(float *rows, int n_rows, int row_len, int hd, const int *pos, float base)
{
    for (int r = 0; r < n_rows; r++)
        for (int h = 0; h + hd <= row_len; h += hd) orc_rope(rows + (size_t)r * row_len + h, pos[r], hd, base);
}

/* llm.c:506-532 */
void orc_softmax(float *x, int n)
{
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = orc_expf(x[i] - mx);
        sum = sum + x[i];
    }
    float inv = 1.0f / (sum + 1e-10f);
    for (int i = 0; i < n; i++) x[i] = x[i] * inv;
}

/* llm.c:538-544 */
void orc_silu(float *x, int n)
{
    for (int i = 0; i < n; i++) {
        float s = 1.0f / (1.0f + orc_expf(-x[i]));
        x[i] = x[i] * s;
    }
}

/* llm.c:551-577: 8-wide two-accumulator dot, horizontal sum, scalar tail */
float orc_dot_f32(const float *a, const float *b, int n)
{
    float a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 4; l++) {
            a0[l] = a0[l] + a[i + l] * b[i + l];
            a1[l] = a1[l] + a[i + 4 + l] * b[i + 4 + l];
        }
    float t[4];
    for (int l = 0; l < 4; l++) t[l] = a0[l] + a1[l];
    float sum = ((t[0] + t[1]) + t[2]) + t[3];
    for (; i < n; i++) sum = sum + a[i] * b[i];
    return sum;
}

/* llm.c:580-596, 599-614, 617-632 */
void orc_axpy_f32(float *dst, float s, const float *src, int n)
{ for (int i = 0; i < n; i++) dst[i] = dst[i] + s * src[i]; }
void orc_vadd_f32(float *dst, const float *src, int n)
{ for (int i = 0; i < n; i++) dst[i] = dst[i] + src[i]; }
void orc_vmul_f32(float *dst, const float *src, int n)
{ for (int i = 0; i < n; i++) dst[i] = dst[i] * src[i]; }

/* llm.c:1129-1140: first strict maximum wins */
int orc_argmax(const float *x, int n)
{
    int best = 0;
    float bv = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > bv) { bv = x[i]; best = i; }
    return best;
}

/* llm.c:1143-1175: the first k indices insertion-sorted by value
 * (descending), then every later element inserted if strictly larger than
 * the smallest kept one and bubbled up */
static void orc_partial_sort_desc(int *idx, const float *v, int n, int k)
{
    for (int i = 0; i < k && i < n; i++) idx[i] = i;
    for (int i = 1; i < k && i < n; i++) {
        int key = idx[i];
        float kv = v[key];
        int j = i - 1;
        while (j >= 0 && v[idx[j]] < kv) { idx[j + 1] = idx[j]; j--; }
        idx[j + 1] = key;
    }
    for (int i = k; i < n; i++) {
        int last = (k < n) ? k - 1 : n - 1;
        if (v[i] > v[idx[last]]) {
            idx[last] = i;
            int j = last - 1;
            while (j >= 0 && v[idx[j]] < v[idx[j + 1]]) { int t = idx[j]; idx[j] = idx[j + 1]; idx[j + 1] = t; j--; }
        }
    }
}

/* llm.c:1177-1246 llm_sample: top-40, softmax of (l - max)/T with
 * llm_expf, nucleus 0.9, renormalise, inverse-CDF draw; the TSC read
 * (llm.c:1226-1233) is replaced by the caller's 32-bit entropy word, mixed
 * and reduced to r in [0, 1) as the reference does */
int orc_sample(const float *logits, int n, float temperature, uint32_t entropy)
{
    if (temperature <= 0.001f) return orc_argmax(logits, n);
    int idx[40];
    float pr[40];
    int k = 40 < n ? 40 : n;
    orc_partial_sort_desc(idx, logits, n, k);
    float mx = logits[idx[0]], sum = 0.0f;
    for (int i = 0; i < k; i++) {
        pr[i] = orc_expf((logits[idx[i]] - mx) / temperature);
        sum += pr[i];
    }
    float inv = 1.0f / (sum + 1e-10f);
    for (int i = 0; i < k; i++) pr[i] *= inv;
    float cum = 0.0f;
    int cut = k;
    for (int i = 0; i < k; i++) {
        cum += pr[i];
        if (cum >= 0.9f) { cut = i + 1; break; }
    }
    if (cut < k) {
        sum = 0.0f;
        for (int i = 0; i < cut; i++) sum += pr[i];
        inv = 1.0f / (sum + 1e-10f);
        for (int i = 0; i < cut; i++) pr[i] *= inv;
    }
    uint32_t lo = entropy;
    lo = lo ^ (lo >> 16);
    lo = lo * 0x45d9f3bU;
    float r = (float)(lo % 10000) / 10000.0f;
    float cdf = 0.0f;
    for (int i = 0; i < cut; i++) {
        cdf += pr[i];
        if (cdf >= r) return idx[i];
    }
    return idx[cut - 1];
}

static float kv_at(const void *c, int kv_type, size_t idx)
{
    if (kv_type == ORC_TYPE_F16) return orc_fp16_to_fp32(((const uint16_t *)c)[idx]);
    return ((const float *)c)[idx];
}

/* llm.c:683-714: per head, scores over t <= pos, softmax, serial PV sum. */
void orc_attention(float *out, const float *q, const void *kc, const void *vc,
                   int kv_type, int n_heads, int n_kv, int hd, int pos)
{
    int kv_dim = n_kv * hd;
    int group = n_heads / n_kv;
    int n = pos + 1;
    float *sc = (float *)malloc(sizeof(float) * (size_t)n);
    float *kt = (float *)malloc(sizeof(float) * (size_t)hd);
    float *head = (float *)malloc(sizeof(float) * (size_t)hd);
    float scale = 1.0f / orc_sqrtf((float)hd);
    for (int h = 0; h < n_heads; h++) {
        int kvh = h / group;
        const float *qh = q + (size_t)h * hd;
        for (int t = 0; t < n; t++) {
            for (int d = 0; d < hd; d++) kt[d] = kv_at(kc, kv_type, (size_t)t * kv_dim + (size_t)kvh * hd + d);
            sc[t] = orc_dot_f32(qh, kt, hd) * scale;
        }
        orc_softmax(sc, n);
        for (int d = 0; d < hd; d++) head[d] = 0.0f;
        for (int t = 0; t < n; t++)
            for (int d = 0; d < hd; d++)
                head[d] = head[d] + sc[t] * kv_at(vc, kv_type, (size_t)t * kv_dim + (size_t)kvh * hd + d);
        for (int d = 0; d < hd; d++) out[(size_t)h * hd + d] = head[d];
    }
    free(sc); free(kt); free(head);
}

/* quantize4.c:122-156: 20-byte block {float scale; u8 data[16]}, same lane
 * tree as Q4_0, result scale * hsum. */
float orc_q4f_dot_block(const void *block20, const float *x)
{
    const uint8_t *p = (const uint8_t *)block20;
    float scale;
    memcpy(&scale, p, 4);
    const uint8_t *qs = p + 4;
    float ch[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < 4; k++)
        for (int c = 0; c < 8; c++) {
            int e = 8 * k + c;
            uint8_t byte = qs[e >> 1];
            int nib = (e & 1) ? (byte >> 4) : (byte & 0x0F);
            ch[c] = ch[c] + (float)(nib - 8) * x[e];
        }
    float t0 = ch[0] + ch[4], t1 = ch[1] + ch[5], t2 = ch[2] + ch[6], t3 = ch[3] + ch[7];
    return scale * (((t0 + t1) + t2) + t3);
}

/* quantize4.c:169-198: rows independent, serial over blocks per row
 * (in_dim a multiple of 32). */
void orc_q4f_gemv(float *out, const void *blocks, const float *x, int out_dim, int in_dim)
{
    int bpr = (in_dim + 31) / 32;
    const uint8_t *w = (const uint8_t *)blocks;
    for (int i = 0; i < out_dim; i++) {
        float s = 0.0f;
        for (int b = 0; b < bpr; b++)
            s = s + orc_q4f_dot_block(w + 20 * ((size_t)i * bpr + b), x + 32 * b);
        out[i] = s;
    }
}

/* ---------------- whole model: llm_forward_token, llm.c:641-743 ---------- */

typedef struct {
    orc_model_desc_t d;
    int hd, kv_dim;
    size_t kv_elem;
    void *kc, *vc;
    float *x, *xn, *q, *k, *v, *att, *g, *u, *fd;
} orc_model_t;

void *orc_model_create(const orc_model_desc_t *d)
{
    orc_model_t *m = (orc_model_t *)calloc(1, sizeof(orc_model_t));
    if (!m) return NULL;
    m->d = *d;
    m->hd = d->dim / d->n_heads;
    m->kv_dim = d->n_kv_heads * m->hd;
    m->kv_elem = d->kv_type == ORC_TYPE_F16 ? 2 : 4;
    size_t kv = (size_t)d->n_layers * d->max_seq * m->kv_dim;
    m->kc = calloc(kv, m->kv_elem);
    m->vc = calloc(kv, m->kv_elem);
    int mx = d->dim > d->ff_dim ? d->dim : d->ff_dim;
    m->x = (float *)calloc((size_t)mx, 4); m->xn = (float *)calloc((size_t)mx, 4);
    m->q = (float *)calloc((size_t)mx, 4); m->k = (float *)calloc((size_t)mx, 4);
    m->v = (float *)calloc((size_t)mx, 4); m->att = (float *)calloc((size_t)mx, 4);
    m->g = (float *)calloc((size_t)mx, 4); m->u = (float *)calloc((size_t)mx, 4);
    m->fd = (float *)calloc((size_t)mx, 4);
    if (!m->kc || !m->vc || !m->x || !m->fd) { orc_model_free(m); return NULL; }
    return m;
}

void orc_model_free(void *p)
{
    orc_model_t *m = (orc_model_t *)p;
    if (!m) return;
    free(m->kc); free(m->vc); free(m->x); free(m->xn); free(m->q); free(m->k);
    free(m->v); free(m->att); free(m->g); free(m->u); free(m->fd);
    free(m);
}

const void *orc_model_kcache(void *p, int L)
{
    orc_model_t *m = (orc_model_t *)p;
    return (const uint8_t *)m->kc + (size_t)L * m->d.max_seq * m->kv_dim * m->kv_elem;
}

const void *orc_model_vcache(void *p, int L)
{
    orc_model_t *m = (orc_model_t *)p;
    return (const uint8_t *)m->vc + (size_t)L * m->d.max_seq * m->kv_dim * m->kv_elem;
}

const float *orc_model_hidden(void *p)
{
    return ((orc_model_t *)p)->xn;
}

void orc_forward_token(void *p, float *logits, int token, int pos)
{
    orc_model_t *m = (orc_model_t *)p;
    const orc_model_desc_t *d = &m->d;
    int dim = d->dim, hd = m->hd, kvd = m->kv_dim, ff = d->ff_dim;
    /* rows of a GEMV are independent, so splitting them over threads gives
     * the same bits as the single-threaded reference loop */
    long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
    int nt = ncpu > 16 ? 16 : (ncpu < 1 ? 1 : (int)ncpu);
    orc_embed(m->x, d->token_embd, d->embd_type, dim, token);
    for (int L = 0; L < d->n_layers; L++) {
        orc_rmsnorm(m->xn, m->x, d->attn_norm[L], ORC_TYPE_F32, dim, d->norm_eps);
        orc_gemv_threads(m->q, d->wq[L], m->xn, d->n_heads * hd, dim, d->wtype, nt);
        orc_gemv_threads(m->k, d->wk[L], m->xn, kvd, dim, d->wtype, nt);
        orc_gemv_threads(m->v, d->wv[L], m->xn, kvd, dim, d->wtype, nt);
        for (int h = 0; h < d->n_heads; h++) orc_rope(m->q + (size_t)h * hd, pos, hd, d->rope_base);
        for (int h = 0; h < d->n_kv_heads; h++) orc_rope(m->k + (size_t)h * hd, pos, hd, d->rope_base);
        size_t off = ((size_t)L * d->max_seq + (size_t)pos) * kvd;
        if (d->kv_type == ORC_TYPE_F16) {
            uint16_t *kc = (uint16_t *)m->kc + off, *vc = (uint16_t *)m->vc + off;
            for (int i = 0; i < kvd; i++) { kc[i] = orc_fp32_to_fp16(m->k[i]); vc[i] = orc_fp32_to_fp16(m->v[i]); }
        } else {
            float *kc = (float *)m->kc + off, *vc = (float *)m->vc + off;
            for (int i = 0; i < kvd; i++) { kc[i] = m->k[i]; vc[i] = m->v[i]; }
        }
        orc_attention(m->att, m->q, orc_model_kcache(m, L), orc_model_vcache(m, L), d->kv_type,
                      d->n_heads, d->n_kv_heads, hd, pos);
        orc_gemv_threads(m->fd, d->wo[L], m->att, dim, dim, d->wtype, nt);
        orc_vadd_f32(m->x, m->fd, dim);
        orc_rmsnorm(m->xn, m->x, d->ffn_norm[L], ORC_TYPE_F32, dim, d->norm_eps);
        orc_gemv_threads(m->g, d->wgate[L], m->xn, ff, dim, d->wtype, nt);
        orc_gemv_threads(m->u, d->wup[L], m->xn, ff, dim, d->wtype, nt);
        orc_silu(m->g, ff);
        orc_vmul_f32(m->g, m->u, ff);
        orc_gemv_threads(m->fd, d->wdown[L], m->g, dim, ff, d->wtype, nt);
        orc_vadd_f32(m->x, m->fd, dim);
    }
    orc_rmsnorm(m->xn, m->x, d->output_norm, ORC_TYPE_F32, dim, d->norm_eps);
    const void *head = d->output_weight ? d->output_weight : d->token_embd;
    int ht = d->output_weight ? d->out_type : d->embd_type;
    orc_gemv_threads(logits, head, m->xn, d->vocab_size, dim, ht, nt);
}

/* llm.c:1279-1288 + 1290-1347 with temperature 0 and no text stops */
int orc_generate_greedy(void *p, const int *prompt, int n_prompt, int n_gen, int *out)
{
    orc_model_t *m = (orc_model_t *)p;
    float *logits = (float *)malloc(sizeof(float) * (size_t)m->d.vocab_size);
    if (!logits) return -1;
    int pos = 0;
    for (int i = 0; i < n_prompt; i++) orc_forward_token(m, logits, prompt[i], pos++);
    int next = orc_argmax(logits, m->d.vocab_size);
    int g = 0;
    for (; g < n_gen && pos < m->d.max_seq; g++) {
        out[g] = next;
        orc_forward_token(m, logits, next, pos++);
        next = orc_argmax(logits, m->d.vocab_size);
    }
    free(logits);
    return g;
}
