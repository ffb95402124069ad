/*
 * tos_synth.c - seeded synthetic inputs (see include/tos_synth.h).
 *
 * Counter-based: value i of (seed, stream) is hash(seed, stream, i), so the
 * output is identical for any thread count.  Per block b, counters
 * 16*b + 0..15 are used: 0,1 for the scale's normal, 2.. for the payload.
 */
#include "tos_synth.h"

#include <math.h>
#include <pthread.h>
#include <string.h>

static uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t tos_synth_u64(uint64_t seed, uint64_t stream, uint64_t index)
{
    uint64_t key = mix64(seed + 0x9E3779B97F4A7C15ull * (stream + 1ull));
    return mix64(key ^ (index * 0xD1B54A32D192ED03ull + 0x2545F4914F6CDD1Dull));
}

/* uniform in (0, 1) with 53 random bits */
static double unif(uint64_t u) { return ((double)(u >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

static double normal_at(uint64_t seed, uint64_t stream, uint64_t c0)
{
    double u1 = unif(tos_synth_u64(seed, stream, c0));
    double u2 = unif(tos_synth_u64(seed, stream, c0 + 1));
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586476925 * u2);
}

uint16_t tos_synth_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u)
        return (uint16_t)(sign | (a > 0x7F800000u ? (0x7E00u | ((a >> 13) & 0x3FFu)) : 0x7C00u));
    int e = (int)(a >> 23);
    if (e < 113) {
        int shift = 126 - e;
        if (e == 0 || shift > 24) return sign;
        uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t r = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
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

enum { K_NF32, K_NF16, K_Q40, K_Q80, K_Q4F };

typedef struct {
    int kind;
    void *out;
    size_t lo, hi;
    uint64_t seed, stream;
    float a, b;
} job_t;

static void run_range(const job_t *j)
{
    for (size_t i = j->lo; i < j->hi; i++) {
        switch (j->kind) {
        case K_NF32:
            ((float *)j->out)[i] = (float)(j->a + j->b * normal_at(j->seed, j->stream, 2 * (uint64_t)i));
            break;
        case K_NF16: {
            float v = (float)(j->a + j->b * normal_at(j->seed, j->stream, 2 * (uint64_t)i));
            ((uint16_t *)j->out)[i] = tos_synth_f32_to_f16(v);
            break;
        }
        case K_Q40: {
            uint8_t *blk = (uint8_t *)j->out + 18 * i;
            float s = (float)fabs(j->a * normal_at(j->seed, j->stream, 16 * (uint64_t)i));
            uint16_t h = tos_synth_f32_to_f16(s);
            blk[0] = (uint8_t)(h & 0xFF);
            blk[1] = (uint8_t)(h >> 8);
            uint64_t r0 = tos_synth_u64(j->seed, j->stream, 16 * (uint64_t)i + 2);
            uint64_t r1 = tos_synth_u64(j->seed, j->stream, 16 * (uint64_t)i + 3);
            memcpy(blk + 2, &r0, 8);
            memcpy(blk + 10, &r1, 8);
            break;
        }
        case K_Q80: {
            uint8_t *blk = (uint8_t *)j->out + 34 * i;
            float s = (float)fabs(j->a * normal_at(j->seed, j->stream, 16 * (uint64_t)i));
            uint16_t h = tos_synth_f32_to_f16(s);
            blk[0] = (uint8_t)(h & 0xFF);
            blk[1] = (uint8_t)(h >> 8);
            for (int w = 0; w < 8; w++) {
                uint64_t r = tos_synth_u64(j->seed, j->stream, 16 * (uint64_t)i + 2 + (uint64_t)w);
                for (int k = 0; k < 4; k++) {
                    uint32_t u16 = (uint32_t)((r >> (16 * k)) & 0xFFFFu);
                    int v = (int)((u16 * 255u) >> 16) - 127;   /* uniform in [-127, 127] */
                    blk[2 + 4 * w + k] = (uint8_t)(int8_t)v;
                }
            }
            break;
        }
        case K_Q4F: {
            uint8_t *blk = (uint8_t *)j->out + 20 * i;
            float s = (float)fabs(j->a * normal_at(j->seed, j->stream, 16 * (uint64_t)i));
            memcpy(blk, &s, 4);
            uint64_t r0 = tos_synth_u64(j->seed, j->stream, 16 * (uint64_t)i + 2);
            uint64_t r1 = tos_synth_u64(j->seed, j->stream, 16 * (uint64_t)i + 3);
            memcpy(blk + 4, &r0, 8);
            memcpy(blk + 12, &r1, 8);
            break;
        }
        }
    }
}

static void *worker(void *arg)
{
    run_range((const job_t *)arg);
    return NULL;
}

static void run(int kind, void *out, size_t n, uint64_t seed, uint64_t stream,
                float a, float b, int n_threads)
{
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 128) n_threads = 128;
    if ((size_t)n_threads > n / 4096 + 1) n_threads = (int)(n / 4096 + 1);
    job_t jobs[128];
    pthread_t th[128];
    for (int t = 0; t < n_threads; t++) {
        jobs[t].kind = kind; jobs[t].out = out;
        jobs[t].lo = n * (size_t)t / (size_t)n_threads;
        jobs[t].hi = n * (size_t)(t + 1) / (size_t)n_threads;
        jobs[t].seed = seed; jobs[t].stream = stream; jobs[t].a = a; jobs[t].b = b;
    }
    if (n_threads == 1) { run_range(&jobs[0]); return; }
    int started = 0;
    for (int t = 0; t < n_threads; t++) {
        if (pthread_create(&th[t], NULL, worker, &jobs[t]) != 0) break;
        started++;
    }
    for (int t = started; t < n_threads; t++) run_range(&jobs[t]);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
}

void tos_synth_normal_f32(float *out, size_t n, uint64_t seed, uint64_t stream,
                          float mean, float std, int n_threads)
{ run(K_NF32, out, n, seed, stream, mean, std, n_threads); }

void tos_synth_normal_f16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream,
                          float mean, float std, int n_threads)
{ run(K_NF16, out, n, seed, stream, mean, std, n_threads); }

void tos_synth_q4_0(void *out, size_t n_blocks, uint64_t seed, uint64_t stream,
                    float scale_std, int n_threads)
{ run(K_Q40, out, n_blocks, seed, stream, scale_std, 0.0f, n_threads); }

void tos_synth_q8_0(void *out, size_t n_blocks, uint64_t seed, uint64_t stream,
                    float scale_std, int n_threads)
{ run(K_Q80, out, n_blocks, seed, stream, scale_std, 0.0f, n_threads); }

void tos_synth_q4f(void *out, size_t n_blocks, uint64_t seed, uint64_t stream,
                   float scale_std, int n_threads)
{ run(K_Q4F, out, n_blocks, seed, stream, scale_std, 0.0f, n_threads); }

void tos_synth_tokens(int32_t *out, size_t n, int32_t vocab, uint64_t seed, uint64_t stream)
{
    for (size_t i = 0; i < n; i++)
        out[i] = (int32_t)(tos_synth_u64(seed, stream, (uint64_t)i) % (uint64_t)vocab);
}
