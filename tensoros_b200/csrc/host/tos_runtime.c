/*
 * tos_runtime.c - C11 host side of the B200 decode path: library state,
 * status handling, registered weights, device-pointer operators and the
 * host-pointer drop-ins that mirror runtime/nn/llm.c's static operators.
 *
 * The drop-ins keep the reference's signatures (void / float / int returns)
 * and its zero-on-unsupported-type behaviour; their status is recorded in a
 * thread-local slot (tos_last_status).  All device work goes through the
 * tosk_* launchers; nothing here computes results on the CPU.
 */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "tos_internal.h"

tos_lib_t tos_g;
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static _Thread_local int t_status;

int tos_set_status(int st)
{
    t_status = st;
    return st;
}

int tos_last_status(void) { return t_status; }

const char *tos_status_string(int st)
{
    switch (st) {
    case TOS_OK: return "ok";
    case TOS_EINVAL: return "invalid argument";
    case TOS_ENOMEM: return "out of memory";
    case TOS_ECUDA: return "CUDA error";
    case TOS_ENCCL: return "collective error";
    case TOS_ETIMEOUT: return "device wait timed out";
    case TOS_ENOTSUP: return "not supported";
    case TOS_ENODEV: return "no CUDA device";
    default: return "unknown status";
    }
}

int tos_from_cuda(int e)
{
    if (e == cudaSuccess) return TOS_OK;
    if (e < 0) return e;   /* already a tos_status_t (e.g. TOS_ENCCL from a collective) */
    if (e == cudaErrorMemoryAllocation) return TOS_ENOMEM;
    if (e == cudaErrorInvalidValue) return TOS_EINVAL;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return TOS_ENODEV;
    return TOS_ECUDA;
}

int tos_device_count(void)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int tos_init(int device)
{
    pthread_mutex_lock(&g_mu);
    int rc = TOS_OK;
    if (tos_g.inited) {
        if (device >= 0 && device != tos_g.device) rc = TOS_EINVAL;
        else cudaSetDevice(tos_g.device);
        pthread_mutex_unlock(&g_mu);
        return tos_set_status(rc);
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        pthread_mutex_unlock(&g_mu);
        return tos_set_status(TOS_ENODEV);
    }
    if (device < 0) cudaGetDevice(&device);
    if (device >= n) {
        pthread_mutex_unlock(&g_mu);
        return tos_set_status(TOS_EINVAL);
    }
    int e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&tos_g.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc((void **)&tos_g.err_dev, sizeof(int));
    /* the library stream does not synchronise with the legacy default
     * stream: every device write here goes on it, and is complete on return */
    if (e == cudaSuccess) e = cudaMemsetAsync(tos_g.err_dev, 0, sizeof(int), tos_g.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(tos_g.stream);
    if (e != cudaSuccess) {
        pthread_mutex_unlock(&g_mu);
        return tos_set_status(tos_from_cuda(e));
    }
    tos_g.device = device;
    tos_g.inited = 1;
    pthread_mutex_unlock(&g_mu);
    return tos_set_status(TOS_OK);
}

int tos_ensure_init(void)
{
    if (tos_g.inited) return TOS_OK;
    return tos_init(-1);
}

void tos_weight_cache_clear(void);

int tos_shutdown(void)
{
    if (!tos_g.inited) return TOS_OK;
    tos_weight_cache_clear();
    cudaStreamSynchronize(tos_g.stream);
    if (tos_g.scratch) cudaFree(tos_g.scratch);
    if (tos_g.err_dev) cudaFree(tos_g.err_dev);
    cudaStreamDestroy(tos_g.stream);
    memset(&tos_g, 0, sizeof(tos_g));
    return tos_set_status(TOS_OK);
}

void *tos_stream(void) { return tos_ensure_init() == TOS_OK ? (void *)tos_g.stream : NULL; }

cudaStream_t tos_pick_stream(void *s) { return s ? (cudaStream_t)s : tos_g.stream; }

int tos_rope_args_ok(int pos, float base)
{
    return pos >= 0 && pos < TOS_MAX_POS && base == base && base < 3.4e38f && base > -3.4e38f;
}

int tos_synchronize(void)
{
    if (tos_ensure_init() != TOS_OK) return tos_set_status(TOS_ENODEV);
    int rc = tos_from_cuda(cudaStreamSynchronize(tos_g.stream));
    if (rc == TOS_OK) rc = tos_check_device_error();
    return tos_set_status(rc);
}

/* Reads and clears the device error word of the bounded waits. */
int tos_check_device_error(void)
{
    int h = 0;
    if (cudaMemcpyAsync(&h, tos_g.err_dev, sizeof(int), cudaMemcpyDeviceToHost, tos_g.stream) != cudaSuccess ||
        cudaStreamSynchronize(tos_g.stream) != cudaSuccess)
        return TOS_ECUDA;
    if (h != 0) {
        cudaMemsetAsync(tos_g.err_dev, 0, sizeof(int), tos_g.stream);
        cudaStreamSynchronize(tos_g.stream);
        return TOS_ETIMEOUT;
    }
    return TOS_OK;
}

void *tos_scratch(size_t bytes)
{
    if (bytes <= tos_g.scratch_bytes) return tos_g.scratch;
    cudaStreamSynchronize(tos_g.stream);
    if (tos_g.scratch) cudaFree(tos_g.scratch);
    tos_g.scratch = NULL;
    tos_g.scratch_bytes = 0;
    size_t sz = bytes < (1u << 20) ? (1u << 20) : bytes;
    if (cudaMalloc(&tos_g.scratch, sz) != cudaSuccess) return NULL;
    tos_g.scratch_bytes = sz;
    return tos_g.scratch;
}

/* ------------------------------------------------------------------ weights */

static size_t block_bytes(int type) { return type == TOS_TYPE_Q4_0 ? 18 : 34; }

int tos_weight_create_dev(tos_weight_t **out, const void *dev_blocks, int out_dim, int in_dim,
                          int type, void *stream)
{
    if (!out || !dev_blocks || out_dim <= 0 || in_dim <= 0 || in_dim % 32) return tos_set_status(TOS_EINVAL);
    if (type != TOS_TYPE_Q4_0 && type != TOS_TYPE_Q8_0) return tos_set_status(TOS_ENOTSUP);
    int rc = tos_ensure_init();
    if (rc) return tos_set_status(rc);
    tos_weight_t *w = (tos_weight_t *)calloc(1, sizeof(*w));
    if (!w) return tos_set_status(TOS_ENOMEM);
    int e = tosk_qmat_alloc(&w->m, type, out_dim, in_dim, tos_pick_stream(stream));
    if (e) { free(w); return tos_set_status(tos_from_cuda(e)); }
    const void *srcs[1] = {dev_blocks};
    int rows[1] = {out_dim};
    e = tosk_qmat_repack(&w->m, srcs, rows, 1, 0, tos_pick_stream(stream));
    if (e) { tosk_qmat_free(&w->m); free(w); return tos_set_status(tos_from_cuda(e)); }
    *out = w;
    return tos_set_status(TOS_OK);
}

int tos_weight_create(tos_weight_t **out, const void *host_blocks, int out_dim, int in_dim, int type)
{
    if (!out || !host_blocks || out_dim <= 0 || in_dim <= 0 || in_dim % 32) return tos_set_status(TOS_EINVAL);
    if (type != TOS_TYPE_Q4_0 && type != TOS_TYPE_Q8_0) return tos_set_status(TOS_ENOTSUP);
    int rc = tos_ensure_init();
    if (rc) return tos_set_status(rc);
    size_t bytes = (size_t)out_dim * (size_t)(in_dim / 32) * block_bytes(type);
    void *stage = NULL;
    int e = cudaMalloc(&stage, bytes);
    if (e) return tos_set_status(tos_from_cuda(e));
    e = cudaMemcpyAsync(stage, host_blocks, bytes, cudaMemcpyHostToDevice, tos_g.stream);
    if (!e) rc = tos_weight_create_dev(out, stage, out_dim, in_dim, type, tos_g.stream);
    else rc = tos_from_cuda(e);
    cudaStreamSynchronize(tos_g.stream);
    cudaFree(stage);
    return tos_set_status(rc);
}

void tos_weight_destroy(tos_weight_t *w)
{
    if (!w) return;
    if (tos_g.inited) cudaStreamSynchronize(tos_g.stream);
    tosk_qmat_free(&w->m);
    free(w);
}

size_t tos_weight_device_bytes(const tos_weight_t *w) { return w ? w->m.bytes : 0; }

/* Cache of weights registered implicitly by host pointer (tos_gemv). */
typedef struct wcache {
    const void *key;
    int out_dim, in_dim, type;
    tos_weight_t *w;
    struct wcache *next;
} wcache_t;
static wcache_t *g_cache;

void tos_weight_cache_clear(void)
{
    pthread_mutex_lock(&g_mu);
    wcache_t *c = g_cache;
    g_cache = NULL;
    pthread_mutex_unlock(&g_mu);
    while (c) {
        wcache_t *n = c->next;
        tos_weight_destroy(c->w);
        free(c);
        c = n;
    }
}

static tos_weight_t *cached_weight(const void *host, int out_dim, int in_dim, int type)
{
    pthread_mutex_lock(&g_mu);
    for (wcache_t *c = g_cache; c; c = c->next)
        if (c->key == host && c->out_dim == out_dim && c->in_dim == in_dim && c->type == type) {
            pthread_mutex_unlock(&g_mu);
            return c->w;
        }
    pthread_mutex_unlock(&g_mu);
    tos_weight_t *w = NULL;
    if (tos_weight_create(&w, host, out_dim, in_dim, type) != TOS_OK) return NULL;
    wcache_t *c = (wcache_t *)calloc(1, sizeof(*c));
    if (!c) { tos_weight_destroy(w); return NULL; }
    c->key = host; c->out_dim = out_dim; c->in_dim = in_dim; c->type = type; c->w = w;
    pthread_mutex_lock(&g_mu);
    c->next = g_cache;
    g_cache = c;
    pthread_mutex_unlock(&g_mu);
    return w;
}

/* ------------------------------------------------- device-pointer operators */

#define DEV_PROLOGUE() \
    int rc_ = tos_ensure_init(); \
    if (rc_) return tos_set_status(rc_)

int tos_gemv_dev(const tos_weight_t *w, const float *x, float *out, void *stream)
{
    DEV_PROLOGUE();
    if (!w || !x || !out) return tos_set_status(TOS_EINVAL);
    /* programmatic dependent launch: weight prefetch overlaps the previous
     * kernel; x is read only after that kernel completes */
    return tos_set_status(tos_from_cuda(tosk_gemv(&w->m, x, NULL, out, NULL, TOSK_GEMV_EXACT, tos_g.err_dev, 1,
                                                  tos_pick_stream(stream))));
}

int tos_gemv_norm_dev(const tos_weight_t *w, const float *x, const float *norm_w, float eps,
                      float *out, void *stream)
{
    DEV_PROLOGUE();
    if (!w || !x || !out || !norm_w) return tos_set_status(TOS_EINVAL);
    tosk_norm_t nrm = {norm_w, eps};
    return tos_set_status(tos_from_cuda(tosk_gemv(&w->m, x, &nrm, out, NULL, TOSK_GEMV_EXACT, tos_g.err_dev, 1,
                                                  tos_pick_stream(stream))));
}

int tos_gemv_mode_dev(const tos_weight_t *w, const float *x, const float *norm_w, float eps,
                      float *out, int mode, void *stream)
{
    DEV_PROLOGUE();
    if (!w || !x || !out) return tos_set_status(TOS_EINVAL);
    if (mode != TOS_GEMV_EXACT && mode != TOS_GEMV_FAST) return tos_set_status(TOS_EINVAL);
    tosk_norm_t nrm = {norm_w, eps};
    return tos_set_status(tos_from_cuda(tosk_gemv(&w->m, x, norm_w ? &nrm : NULL, out, NULL, mode,
                                                  tos_g.err_dev, 1, tos_pick_stream(stream))));
}

int tos_block_dots_dev(const void *blocks, int type, const float *x, int n_blocks, float *out, void *stream)
{
    DEV_PROLOGUE();
    if (n_blocks < 0 || (n_blocks && (!blocks || !x || !out))) return tos_set_status(TOS_EINVAL);
    if (type != TOS_TYPE_Q4_0 && type != TOS_TYPE_Q8_0) return tos_set_status(TOS_ENOTSUP);
    return tos_set_status(tos_from_cuda(tosk_block_dots(blocks, type, x, n_blocks, out, tos_pick_stream(stream))));
}

int tos_rmsnorm_dev(float *out, const float *x, const void *w, int wtype, int dim, float eps, void *stream)
{
    DEV_PROLOGUE();
    if (dim < 0 || (dim && (!out || !x || !w))) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_rmsnorm(out, x, w, wtype, dim, eps, 0, tos_pick_stream(stream))));
}

int tos_rope_dev(float *vec, int n_vec, int pos, int head_dim, float base, void *stream)
{
    DEV_PROLOGUE();
    if (n_vec < 0 || head_dim <= 0 || (head_dim & 1) || !tos_rope_args_ok(pos, base)) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_rope(vec, n_vec, NULL, pos, head_dim, base, tos_pick_stream(stream))));
}

int tos_softmax_dev(float *x, int n, void *stream)
{
    DEV_PROLOGUE();
    if (n < 0) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_softmax(x, n, tos_pick_stream(stream))));
}

int tos_silu_dev(float *x, int n, void *stream)
{
    DEV_PROLOGUE();
    return tos_set_status(tos_from_cuda(tosk_silu(x, n, tos_pick_stream(stream))));
}

int tos_vadd_dev(float *d, const float *s, int n, void *stream)
{
    DEV_PROLOGUE();
    return tos_set_status(tos_from_cuda(tosk_vadd(d, s, n, tos_pick_stream(stream))));
}

int tos_vmul_dev(float *d, const float *s, int n, void *stream)
{
    DEV_PROLOGUE();
    return tos_set_status(tos_from_cuda(tosk_vmul(d, s, n, tos_pick_stream(stream))));
}

int tos_axpy_dev(float *d, float sc, const float *s, int n, void *stream)
{
    DEV_PROLOGUE();
    return tos_set_status(tos_from_cuda(tosk_axpy(d, sc, s, n, tos_pick_stream(stream))));
}

int tos_dot_dev(const float *a, const float *b, int n, float *out, void *stream)
{
    DEV_PROLOGUE();
    if (n < 0 || !out) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_dot(a, b, n, out, tos_pick_stream(stream))));
}

int tos_embed_dev(float *out, const void *embd, int type, int dim, int token, void *stream)
{
    DEV_PROLOGUE();
    if (!out || !embd || dim <= 0 || token < 0) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_embed(out, embd, type, dim, NULL, token, 0, tos_pick_stream(stream))));
}

int tos_argmax_dev(const float *x, int n, int *out_index, void *stream)
{
    DEV_PROLOGUE();
    if (!x || n <= 0 || !out_index) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_argmax(x, n, out_index, NULL, 0, tos_pick_stream(stream))));
}

size_t tos_gemm_workspace_bytes(int m, int out_dim, int in_dim)
{
    return tosk_gemm_ws_bytes(m, out_dim, in_dim);
}

int tos_gemm_dev(const tos_weight_t *w, const float *x, int m, float *y, void *ws, size_t ws_bytes,
                 void *stream)
{
    DEV_PROLOGUE();
    if (!w || !x || !y || !ws || m <= 0) return tos_set_status(TOS_EINVAL);
    if (ws_bytes < tosk_gemm_ws_bytes(m, w->m.rows, w->m.cols)) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_gemm_q(&w->m, x, m, y, ws, ws_bytes, tos_g.err_dev, 1,
                                                    tos_pick_stream(stream))));
}

int tos_argmax_sharded_dev(const float *x, int n, int world, int *out_index, void *stream)
{
    DEV_PROLOGUE();
    if (!x || n <= 0 || world <= 0 || n % world || !out_index) return tos_set_status(TOS_EINVAL);
    cudaStream_t st = tos_pick_stream(stream);
    /* the pairs live in the library scratch: order after the caller's stream */
    if (st != tos_g.stream && cudaStreamSynchronize(st) != cudaSuccess) return tos_set_status(TOS_ECUDA);
    int *pairs = (int *)tos_scratch((size_t)world * 2 * sizeof(int));
    if (!pairs) return tos_set_status(TOS_ENOMEM);
    const int per = n / world;
    int e = 0;
    for (int r = 0; !e && r < world; r++)
        e = tosk_argmax_slice(x + (size_t)r * per, per, r * per, r == 0, pairs + 2 * r, 0, st);
    if (!e) e = tosk_argmax_pairs(pairs, world, out_index, 0, st);
    if (!e) e = cudaStreamSynchronize(st);
    return tos_set_status(tos_from_cuda(e));
}

size_t tos_attention_workspace_bytes(int n_heads, int max_ctx)
{
    if (n_heads <= 0 || max_ctx <= 0) return 0;
    return tosk_attention_ws_bytes(n_heads, max_ctx);
}

int tos_attention_dev(float *out, const float *q, const void *k_cache, const void *v_cache,
                      int kv_type, int n_heads, int n_kv, int head_dim, int pos, int max_ctx,
                      int mode, void *ws, size_t ws_bytes, void *stream)
{
    DEV_PROLOGUE();
    if (!out || !q || !k_cache || !v_cache || !ws) return tos_set_status(TOS_EINVAL);
    if (pos < 0 || pos >= max_ctx) return tos_set_status(TOS_EINVAL);
    if (mode != TOS_ATTN_EXACT && mode != TOS_ATTN_FAST) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_attention(out, q, k_cache, v_cache, kv_type, n_heads, n_kv,
                                                       head_dim, NULL, pos, max_ctx, mode, ws, ws_bytes,
                                                       tos_g.err_dev, 0, tos_pick_stream(stream))));
}

/* ------------------------------------------------- host-pointer drop-ins */

/* Copies n bytes H2D into the scratch region at offset off. */
static int h2d(size_t off, const void *src, size_t n)
{
    return cudaMemcpyAsync((char *)tos_g.scratch + off, src, n, cudaMemcpyHostToDevice, tos_g.stream);
}

static int finish_to_host(void *dst, size_t off, size_t n)
{
    int e = cudaMemcpyAsync(dst, (char *)tos_g.scratch + off, n, cudaMemcpyDeviceToHost, tos_g.stream);
    if (!e) e = cudaStreamSynchronize(tos_g.stream);
    return e;
}

static size_t al(size_t v) { return (v + 255) & ~(size_t)255; }

static void zero_f(float *out, int n)
{
    if (out && n > 0) memset(out, 0, sizeof(float) * (size_t)n);
}

static size_t row_bytes(int in_dim, int type)
{
    switch (type) {
    case TOS_TYPE_Q4_0: return (size_t)(in_dim / 32) * 18;
    case TOS_TYPE_Q8_0: return (size_t)(in_dim / 32) * 34;
    case TOS_TYPE_F16: return (size_t)in_dim * 2;
    default: return (size_t)in_dim * 4;
    }
}

void tos_gemv(float *out, const void *weight, const float *x, int out_dim, int in_dim, int type)
{
    if (out_dim <= 0) { tos_set_status(TOS_OK); return; }
    zero_f(out, out_dim);
    if (!out || !weight || !x || in_dim < 0) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    int e;
    if (type == TOS_TYPE_Q4_0 || type == TOS_TYPE_Q8_0) {
        /* llm_vec_dot uses nb = n/32 blocks; trailing elements are ignored and
         * the row stride (llm_row_bytes) is the same as for (n/32)*32 columns */
        in_dim = (in_dim / 32) * 32;
        if (in_dim == 0) { tos_set_status(TOS_OK); return; }   /* nb = 0: rows sum to 0 */
        tos_weight_t *w = cached_weight(weight, out_dim, in_dim, type);
        if (!w) { tos_set_status(TOS_ENOMEM); return; }
        size_t ox = 0, oo = al((size_t)in_dim * 4);
        if (!tos_scratch(oo + (size_t)out_dim * 4)) { tos_set_status(TOS_ENOMEM); return; }
        e = h2d(ox, x, (size_t)in_dim * 4);
        if (!e) e = tosk_gemv(&w->m, (const float *)((char *)tos_g.scratch + ox), NULL,
                              (float *)((char *)tos_g.scratch + oo), NULL, TOSK_GEMV_EXACT, tos_g.err_dev, 0,
                              tos_g.stream);
        if (!e) e = finish_to_host(out, oo, (size_t)out_dim * 4);
    } else if (type == TOS_TYPE_F16 || type == TOS_TYPE_F32) {
        size_t wb = row_bytes(in_dim, type) * (size_t)out_dim;
        size_t ow = 0, ox = al(wb), oo = ox + al((size_t)in_dim * 4 + 4);
        if (!tos_scratch(oo + (size_t)out_dim * 4)) { tos_set_status(TOS_ENOMEM); return; }
        e = h2d(ow, weight, wb);
        if (!e && in_dim) e = h2d(ox, x, (size_t)in_dim * 4);
        if (!e) e = tosk_gemv_float((char *)tos_g.scratch + ow, type, (const float *)((char *)tos_g.scratch + ox),
                                    (float *)((char *)tos_g.scratch + oo), out_dim, in_dim, tos_g.stream);
        if (!e) e = finish_to_host(out, oo, (size_t)out_dim * 4);
    } else {
        tos_set_status(TOS_OK);   /* llm_vec_dot: unknown type sums to 0 */
        return;
    }
    if (e) { zero_f(out, out_dim); tos_set_status(tos_from_cuda(e)); return; }
    tos_set_status(tos_check_device_error());
}

float tos_vec_dot(const void *weight, const float *x, int n, int type)
{
    float r = 0.0f;
    tos_gemv(&r, weight, x, 1, n, type);
    return r;
}

static float block_dot_host(const void *block, const float *x, int type)
{
    if (!block || !x) { tos_set_status(TOS_EINVAL); return 0.0f; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return 0.0f; }
    size_t bb = block_bytes(type);
    size_t ob = 0, ox = 256, oo = 512;
    if (!tos_scratch(1024)) { tos_set_status(TOS_ENOMEM); return 0.0f; }
    float r = 0.0f;
    int e = h2d(ob, block, bb);
    if (!e) e = h2d(ox, x, 128);
    if (!e) e = tosk_block_dots((char *)tos_g.scratch + ob, type, (const float *)((char *)tos_g.scratch + ox), 1,
                                (float *)((char *)tos_g.scratch + oo), tos_g.stream);
    if (!e) e = finish_to_host(&r, oo, 4);
    tos_set_status(tos_from_cuda(e));
    return e ? 0.0f : r;
}

float tos_q4_0_dot32(const void *block, const float *x) { return block_dot_host(block, x, TOS_TYPE_Q4_0); }
float tos_q8_0_dot32(const void *block, const float *x) { return block_dot_host(block, x, TOS_TYPE_Q8_0); }

void tos_embed(float *out, const void *embd, int type, int dim, int token)
{
    zero_f(out, dim);
    if (!out || !embd || dim <= 0 || token < 0) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    if (type != TOS_TYPE_Q4_0 && type != TOS_TYPE_Q8_0 && type != TOS_TYPE_F16 && type != TOS_TYPE_F32) {
        tos_set_status(TOS_OK);
        return;
    }
    size_t rb = row_bytes(dim, type);
    size_t oe = 0, oo = al(rb);
    if (!tos_scratch(oo + (size_t)dim * 4)) { tos_set_status(TOS_ENOMEM); return; }
    /* only the token's row travels; the kernel indexes row 0 of it */
    int e = h2d(oe, (const char *)embd + rb * (size_t)token, rb);
    if (!e) e = tosk_embed((float *)((char *)tos_g.scratch + oo), (char *)tos_g.scratch + oe, type, dim, NULL, 0, 0,
                           tos_g.stream);
    if (!e) e = finish_to_host(out, oo, (size_t)dim * 4);
    tos_set_status(tos_from_cuda(e));
}

void tos_rmsnorm(float *out, const float *x, const void *w, int dim, int wtype)
{
    if (dim <= 0) { tos_set_status(TOS_OK); return; }
    if (!out || !x || !w) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { zero_f(out, dim); tos_set_status(TOS_ENODEV); return; }
    size_t wb = wtype == TOS_TYPE_F16 ? (size_t)dim * 2 : (wtype == TOS_TYPE_F32 ? (size_t)dim * 4 : 0);
    size_t ox = 0, ow = al((size_t)dim * 4), oo = ow + al(wb + 4);
    if (!tos_scratch(oo + (size_t)dim * 4)) { tos_set_status(TOS_ENOMEM); return; }
    int e = h2d(ox, x, (size_t)dim * 4);
    if (!e && wb) e = h2d(ow, w, wb);
    if (!e) e = tosk_rmsnorm((float *)((char *)tos_g.scratch + oo), (const float *)((char *)tos_g.scratch + ox),
                             (char *)tos_g.scratch + ow, wtype, dim, 1e-6f, 0, tos_g.stream);
    if (!e) e = finish_to_host(out, oo, (size_t)dim * 4);
    tos_set_status(tos_from_cuda(e));
}

/* In-place operators on one host vector: copy in, run, copy back. */
static void inplace1(float *x, int n, int op, float a, const float *src)
{
    if (n <= 0) { tos_set_status(TOS_OK); return; }
    if (!x || (op >= 2 && !src)) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    size_t ox = 0, os = al((size_t)n * 4);
    if (!tos_scratch(os + (size_t)n * 4)) { tos_set_status(TOS_ENOMEM); return; }
    float *dx = (float *)((char *)tos_g.scratch + ox), *ds = (float *)((char *)tos_g.scratch + os);
    int e = h2d(ox, x, (size_t)n * 4);
    if (!e && op >= 2) e = h2d(os, src, (size_t)n * 4);
    if (!e) {
        switch (op) {
        case 0: e = tosk_softmax(dx, n, tos_g.stream); break;
        case 1: e = tosk_silu(dx, n, tos_g.stream); break;
        case 2: e = tosk_vadd(dx, ds, n, tos_g.stream); break;
        case 3: e = tosk_vmul(dx, ds, n, tos_g.stream); break;
        case 4: e = tosk_axpy(dx, a, ds, n, tos_g.stream); break;
        }
    }
    if (!e) e = finish_to_host(x, ox, (size_t)n * 4);
    tos_set_status(tos_from_cuda(e));
}

void tos_softmax(float *x, int n) { inplace1(x, n, 0, 0.0f, NULL); }
void tos_silu(float *x, int n) { inplace1(x, n, 1, 0.0f, NULL); }
void tos_vadd_f32(float *dst, const float *src, int n) { inplace1(dst, n, 2, 0.0f, src); }
void tos_vmul_f32(float *dst, const float *src, int n) { inplace1(dst, n, 3, 0.0f, src); }
void tos_axpy_f32(float *dst, float s, const float *src, int n) { inplace1(dst, n, 4, s, src); }

void tos_rope(float *vec, int pos, int head_dim, float base)
{
    if (head_dim <= 0) { tos_set_status(TOS_OK); return; }
    if (!vec || (head_dim & 1) || !tos_rope_args_ok(pos, base)) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    if (!tos_scratch((size_t)head_dim * 4)) { tos_set_status(TOS_ENOMEM); return; }
    int e = h2d(0, vec, (size_t)head_dim * 4);
    if (!e) e = tosk_rope((float *)tos_g.scratch, 1, NULL, pos, head_dim, base, tos_g.stream);
    if (!e) e = finish_to_host(vec, 0, (size_t)head_dim * 4);
    tos_set_status(tos_from_cuda(e));
}

float tos_dot_f32(const float *a, const float *b, int n)
{
    if (n <= 0) { tos_set_status(TOS_OK); return 0.0f; }
    if (!a || !b) { tos_set_status(TOS_EINVAL); return 0.0f; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return 0.0f; }
    size_t oa = 0, ob = al((size_t)n * 4), oo = ob + al((size_t)n * 4);
    if (!tos_scratch(oo + 4)) { tos_set_status(TOS_ENOMEM); return 0.0f; }
    float r = 0.0f;
    int e = h2d(oa, a, (size_t)n * 4);
    if (!e) e = h2d(ob, b, (size_t)n * 4);
    if (!e) e = tosk_dot((const float *)((char *)tos_g.scratch + oa), (const float *)((char *)tos_g.scratch + ob), n,
                         (float *)((char *)tos_g.scratch + oo), tos_g.stream);
    if (!e) e = finish_to_host(&r, oo, 4);
    tos_set_status(tos_from_cuda(e));
    return e ? 0.0f : r;
}

int tos_argmax(const float *logits, int n)
{
    if (!logits || n <= 0) { tos_set_status(TOS_EINVAL); return 0; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return 0; }
    size_t ox = 0, oo = al((size_t)n * 4);
    if (!tos_scratch(oo + 8)) { tos_set_status(TOS_ENOMEM); return 0; }
    int r = 0;
    int e = h2d(ox, logits, (size_t)n * 4);
    if (!e) e = tosk_argmax((const float *)tos_g.scratch, n, (int *)((char *)tos_g.scratch + oo), NULL, 0, tos_g.stream);
    if (!e) e = finish_to_host(&r, oo, 4);
    tos_set_status(tos_from_cuda(e));
    return e ? 0 : r;
}

/* llm_sample (llm.c:1177-1246) with the caller's entropy word in place of
 * the timestamp; temperature <= 0.001 is llm_argmax */
int tos_sample(const float *logits, int n, float temperature, uint32_t entropy)
{
    if (!logits || n <= 0) { tos_set_status(TOS_EINVAL); return 0; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return 0; }
    size_t ox = 0, oo = al((size_t)n * 4);
    if (!tos_scratch(oo + 8)) { tos_set_status(TOS_ENOMEM); return 0; }
    int r = 0;
    int e = h2d(ox, logits, (size_t)n * 4);
    if (!e) e = tosk_sample((const float *)tos_g.scratch, n, temperature, entropy,
                            (int *)((char *)tos_g.scratch + oo), tos_g.stream);
    if (!e) e = finish_to_host(&r, oo, 4);
    tos_set_status(tos_from_cuda(e));
    return e ? 0 : r;
}

int tos_sample_dev(const float *logits, int n, float temperature, uint32_t entropy, int *out_index, void *stream)
{
    DEV_PROLOGUE();
    if (!logits || n <= 0 || !out_index) return tos_set_status(TOS_EINVAL);
    return tos_set_status(tos_from_cuda(tosk_sample(logits, n, temperature, entropy, out_index,
                                                    tos_pick_stream(stream))));
}

float tos_q4_dot_block(const void *block20, const float *x)
{
    float r = 0.0f;
    tos_q4_gemv(&r, block20, x, 1, 32);
    return r;
}

void tos_q4_gemv(float *out, const void *blocks20, const float *x, int out_dim, int in_dim)
{
    if (out_dim <= 0) { tos_set_status(TOS_OK); return; }
    zero_f(out, out_dim);
    if (!out || !blocks20 || !x || in_dim <= 0 || in_dim % 32) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    size_t wb = (size_t)out_dim * (size_t)(in_dim / 32) * 20;
    size_t ow = 0, ox = al(wb), oo = ox + al((size_t)in_dim * 4);
    if (!tos_scratch(oo + (size_t)out_dim * 4)) { tos_set_status(TOS_ENOMEM); return; }
    int e = h2d(ow, blocks20, wb);
    if (!e) e = h2d(ox, x, (size_t)in_dim * 4);
    if (!e) e = tosk_q4f_gemv((char *)tos_g.scratch + ow, (const float *)((char *)tos_g.scratch + ox),
                              (float *)((char *)tos_g.scratch + oo), out_dim, in_dim, tos_g.stream);
    if (!e) e = finish_to_host(out, oo, (size_t)out_dim * 4);
    tos_set_status(tos_from_cuda(e));
}
