/*
 * tos_tf.c - C11 host side of the fp32 transformer engine
 * (runtime/nn/transformer.c:92-366) on the GPU: host-pointer drop-ins for
 * tf_rmsnorm and tf_swiglu_ffn, and a device-resident engine model for
 * tf_forward_token / tf_cached_attention / kv_cache_reset.  Results are
 * bit-identical to the reference's (tf_engine.cu keeps its orders).
 */
#include <stdlib.h>
#include <string.h>

#include "tos_internal.h"

struct tos_tf_model {
    tos_tf_desc_t d;
    int hd;
    float *w;              /* every weight, one allocation (offsets below) */
    size_t o_layer;        /* floats per layer */
    size_t o_wq, o_wk, o_wv, o_wo, o_w1, o_w2, o_w3, o_ra, o_rf;
    float *embd, *rms_final;
    float *kc, *vc;        /* [layers][heads][max_seq][head_dim] */
    float *x, *xn, *q, *k, *v, *att, *tmp, *g, *u, *logits;
    cudaStream_t st;
};

static size_t al4(size_t v) { return (v + 63) & ~(size_t)63; }   /* 256-byte steps of floats */

/* ---------------------------------------------------------- drop-ins */

void tos_tf_rmsnorm(float *out, const float *x, const float *w, int dim)
{
    if (dim <= 0) { tos_set_status(TOS_OK); return; }
    if (!out || !x || !w) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    const size_t n = (size_t)dim;
    if (!tos_scratch(3 * al4(n) * 4)) { tos_set_status(TOS_ENOMEM); return; }
    float *dx = (float *)tos_g.scratch, *dw = dx + al4(n), *dout = dw + al4(n);
    int e = cudaMemcpyAsync(dx, x, n * 4, cudaMemcpyHostToDevice, tos_g.stream);
    if (!e) e = cudaMemcpyAsync(dw, w, n * 4, cudaMemcpyHostToDevice, tos_g.stream);
    if (!e) e = tosk_tf_rmsnorm(dout, dx, dw, dim, tos_g.stream);
    if (!e) e = cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, tos_g.stream);
    if (!e) e = cudaStreamSynchronize(tos_g.stream);
    tos_set_status(tos_from_cuda(e));
}

void tos_tf_swiglu_ffn(float *out, const float *x, const float *w1, const float *w2, const float *w3, int dim,
                       int ff_dim)
{
    if (dim <= 0) { tos_set_status(TOS_OK); return; }
    if (!out || !x || !w1 || !w2 || !w3 || ff_dim <= 0) { tos_set_status(TOS_EINVAL); return; }
    if (tos_ensure_init()) { tos_set_status(TOS_ENODEV); return; }
    const size_t d = (size_t)dim, f = (size_t)ff_dim, mat = al4(d * f);
    if (!tos_scratch((3 * mat + 2 * al4(d) + 2 * al4(f)) * 4)) { tos_set_status(TOS_ENOMEM); return; }
    float *dw1 = (float *)tos_g.scratch, *dw2 = dw1 + mat, *dw3 = dw2 + mat;
    float *dx = dw3 + mat, *dout = dx + al4(d), *dg = dout + al4(d), *du = dg + al4(f);
    cudaStream_t st = tos_g.stream;
    int e = cudaMemcpyAsync(dw1, w1, d * f * 4, cudaMemcpyHostToDevice, st);
    if (!e) e = cudaMemcpyAsync(dw2, w2, d * f * 4, cudaMemcpyHostToDevice, st);
    if (!e) e = cudaMemcpyAsync(dw3, w3, d * f * 4, cudaMemcpyHostToDevice, st);
    if (!e) e = cudaMemcpyAsync(dx, x, d * 4, cudaMemcpyHostToDevice, st);
    /* transformer.c:129-183: gate = W1 x, up = W3 x, silu(gate) * up, W2 h */
    if (!e) e = tosk_tf_matvec(dw1, dx, dg, ff_dim, dim, 1, st);
    if (!e) e = tosk_tf_matvec(dw3, dx, du, ff_dim, dim, 1, st);
    if (!e) e = tosk_tf_silu_mul(dg, du, ff_dim, st);
    if (!e) e = tosk_tf_matvec(dw2, dg, dout, dim, ff_dim, 1, st);
    if (!e) e = cudaMemcpyAsync(out, dout, d * 4, cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaStreamSynchronize(st);
    tos_set_status(tos_from_cuda(e));
}

/* ------------------------------------------------------------- model */

void tos_tf_model_destroy(tos_tf_model_t *m)
{
    if (!m) return;
    if (m->st) cudaStreamSynchronize(m->st);
    void *bufs[] = {m->w, m->embd, m->rms_final, m->kc, m->vc, m->x, m->xn, m->q, m->k, m->v,
                    m->att, m->tmp, m->g, m->u, m->logits};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++)
        if (bufs[i]) cudaFree(bufs[i]);
    if (m->st) cudaStreamDestroy(m->st);
    free(m);
}

int tos_tf_model_create(tos_tf_model_t **out, const tos_tf_desc_t *d)
{
    if (!out) return tos_set_status(TOS_EINVAL);
    *out = NULL;
    if (!d || d->dim <= 0 || d->num_heads <= 0 || d->dim % d->num_heads || d->ff_dim <= 0 || d->num_layers <= 0 ||
        d->vocab_size <= 0 || d->max_seq <= 0 || !d->tok_embed || !d->rms_final || !d->wq || !d->wk || !d->wv ||
        !d->wo || !d->w1 || !d->w2 || !d->w3 || !d->rms_att || !d->rms_ffn)
        return tos_set_status(TOS_EINVAL);
    /* the matvec kernels stage their input vector in shared memory */
    if ((size_t)d->dim * 4 > 200 * 1024 || (size_t)d->ff_dim * 4 > 200 * 1024 || (size_t)d->max_seq * 4 > 200 * 1024)
        return tos_set_status(TOS_ENOTSUP);
    int rc = tos_ensure_init();
    if (rc) return tos_set_status(rc);
    tos_tf_model_t *m = (tos_tf_model_t *)calloc(1, sizeof(*m));
    if (!m) return tos_set_status(TOS_ENOMEM);
    m->d = *d;
    m->hd = d->dim / d->num_heads;
    const size_t D = (size_t)d->dim, F = (size_t)d->ff_dim, L = (size_t)d->num_layers;
    m->o_wq = 0;
    m->o_wk = m->o_wq + al4(D * D);
    m->o_wv = m->o_wk + al4(D * D);
    m->o_wo = m->o_wv + al4(D * D);
    m->o_w1 = m->o_wo + al4(D * D);
    m->o_w2 = m->o_w1 + al4(D * F);
    m->o_w3 = m->o_w2 + al4(D * F);
    m->o_ra = m->o_w3 + al4(D * F);
    m->o_rf = m->o_ra + al4(D);
    m->o_layer = m->o_rf + al4(D);
    const size_t kv = L * (size_t)d->num_heads * (size_t)d->max_seq * (size_t)m->hd;
    int e = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking);
    if (!e) e = cudaMalloc((void **)&m->w, L * m->o_layer * 4);
    if (!e) e = cudaMalloc((void **)&m->embd, (size_t)d->vocab_size * D * 4);
    if (!e) e = cudaMalloc((void **)&m->rms_final, D * 4);
    if (!e) e = cudaMalloc((void **)&m->kc, kv * 4);
    if (!e) e = cudaMalloc((void **)&m->vc, kv * 4);
    float **vecs[] = {&m->x, &m->xn, &m->q, &m->k, &m->v, &m->att, &m->tmp};
    for (size_t i = 0; !e && i < sizeof(vecs) / sizeof(vecs[0]); i++) e = cudaMalloc((void **)vecs[i], D * 4);
    if (!e) e = cudaMalloc((void **)&m->g, F * 4);
    if (!e) e = cudaMalloc((void **)&m->u, F * 4);
    if (!e) e = cudaMalloc((void **)&m->logits, (size_t)d->vocab_size * 4);
    /* every device write on the model's stream (it does not synchronise
     * with the legacy default stream) */
    for (int l = 0; !e && l < d->num_layers; l++) {
        float *b = m->w + (size_t)l * m->o_layer;
        const struct { const float *src; size_t off, n; } up[] = {
            {d->wq[l], m->o_wq, D * D}, {d->wk[l], m->o_wk, D * D}, {d->wv[l], m->o_wv, D * D},
            {d->wo[l], m->o_wo, D * D}, {d->w1[l], m->o_w1, D * F}, {d->w2[l], m->o_w2, D * F},
            {d->w3[l], m->o_w3, D * F}, {d->rms_att[l], m->o_ra, D}, {d->rms_ffn[l], m->o_rf, D}};
        for (size_t i = 0; !e && i < sizeof(up) / sizeof(up[0]); i++) {
            if (!up[i].src) e = cudaErrorInvalidValue;
            else e = cudaMemcpyAsync(b + up[i].off, up[i].src, up[i].n * 4, cudaMemcpyHostToDevice, m->st);
        }
    }
    if (!e) e = cudaMemcpyAsync(m->embd, d->tok_embed, (size_t)d->vocab_size * D * 4, cudaMemcpyHostToDevice, m->st);
    if (!e) e = cudaMemcpyAsync(m->rms_final, d->rms_final, D * 4, cudaMemcpyHostToDevice, m->st);
    /* kv_cache_init (transformer.c:46-65) zeroes the cache */
    if (!e) e = cudaMemsetAsync(m->kc, 0, kv * 4, m->st);
    if (!e) e = cudaMemsetAsync(m->vc, 0, kv * 4, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);
    if (e) {
        tos_tf_model_destroy(m);
        return tos_set_status(tos_from_cuda(e));
    }
    *out = m;
    return tos_set_status(TOS_OK);
}

/* kv_cache_reset (transformer.c:67-70): the sequence restarts at position
 * 0; attention reads only positions up to the current one, so the rows of
 * the previous sequence need no clearing. */
int tos_tf_reset(tos_tf_model_t *m) { return tos_set_status(m ? TOS_OK : TOS_EINVAL); }

/* tf_cached_attention (transformer.c:193-247) on the model's cache: q, k, v
 * and out are host vectors of head_dim floats. */
int tos_tf_cached_attention(tos_tf_model_t *m, float *out, const float *q, const float *k, const float *v, int layer,
                            int head, int pos)
{
    if (!m || !out || !q || !k || !v || layer < 0 || layer >= m->d.num_layers || head < 0 ||
        head >= m->d.num_heads || pos < 0 || pos >= m->d.max_seq)
        return tos_set_status(TOS_EINVAL);
    const size_t hb = (size_t)m->hd * 4;
    int e = cudaMemcpyAsync(m->q, q, hb, cudaMemcpyHostToDevice, m->st);
    if (!e) e = cudaMemcpyAsync(m->k, k, hb, cudaMemcpyHostToDevice, m->st);
    if (!e) e = cudaMemcpyAsync(m->v, v, hb, cudaMemcpyHostToDevice, m->st);
    if (!e) e = tosk_tf_attention(m->att, m->hd, m->q, m->k, m->v, m->hd, m->kc, m->vc, layer, head, 1, m->d.num_heads,
                                  m->hd, m->d.max_seq, pos, m->st);
    if (!e) e = cudaMemcpyAsync(out, m->att, hb, cudaMemcpyDeviceToHost, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);
    return tos_set_status(tos_from_cuda(e));
}

/* tf_forward_token (transformer.c:255-366): tok_embed is the token's
 * embedding row (host, dim floats), logits (host, vocab_size floats) may be
 * NULL. */
int tos_tf_forward_token(tos_tf_model_t *m, float *logits, const float *tok_embed, int pos)
{
    if (!m || !tok_embed || pos < 0 || pos >= m->d.max_seq) return tos_set_status(TOS_EINVAL);
    const int D = m->d.dim, F = m->d.ff_dim;
    cudaStream_t st = m->st;
    int e = cudaMemcpyAsync(m->x, tok_embed, (size_t)D * 4, cudaMemcpyHostToDevice, st);
    for (int l = 0; !e && l < m->d.num_layers; l++) {
        const float *b = m->w + (size_t)l * m->o_layer;
        e = tosk_tf_rmsnorm(m->xn, m->x, b + m->o_ra, D, st);
        if (!e) e = tosk_tf_matvec(b + m->o_wq, m->xn, m->q, D, D, 0, st);   /* scalar order */
        if (!e) e = tosk_tf_matvec(b + m->o_wk, m->xn, m->k, D, D, 0, st);
        if (!e) e = tosk_tf_matvec(b + m->o_wv, m->xn, m->v, D, D, 0, st);
        if (!e) e = tosk_tf_attention(m->att, m->hd, m->q, m->k, m->v, m->hd, m->kc, m->vc, l, 0, m->d.num_heads,
                                      m->d.num_heads, m->hd, m->d.max_seq, pos, st);
        if (!e) e = tosk_tf_matvec(b + m->o_wo, m->att, m->tmp, D, D, 1, st);
        if (!e) e = tosk_tf_add(m->x, m->tmp, D, st);
        if (!e) e = tosk_tf_rmsnorm(m->xn, m->x, b + m->o_rf, D, st);
        if (!e) e = tosk_tf_matvec(b + m->o_w1, m->xn, m->g, F, D, 1, st);
        if (!e) e = tosk_tf_matvec(b + m->o_w3, m->xn, m->u, F, D, 1, st);
        if (!e) e = tosk_tf_silu_mul(m->g, m->u, F, st);
        if (!e) e = tosk_tf_matvec(b + m->o_w2, m->g, m->tmp, D, F, 1, st);
        if (!e) e = tosk_tf_add(m->x, m->tmp, D, st);
    }
    if (!e) e = tosk_tf_rmsnorm(m->xn, m->x, m->rms_final, D, st);
    /* weight-tied output: logits = embedding rows . xn (transformer.c:355-365) */
    if (!e) e = tosk_tf_matvec(m->embd, m->xn, m->logits, m->d.vocab_size, D, 1, st);
    if (!e && logits)
        e = cudaMemcpyAsync(logits, m->logits, (size_t)m->d.vocab_size * 4, cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaStreamSynchronize(st);
    return tos_set_status(tos_from_cuda(e));
}
