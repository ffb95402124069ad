/*
 * ref_tf_hosted.c - hosted build of the reference's fp32 transformer engine
 * (test infrastructure, oracle/_ref only).
 *
 * Textually includes the UNMODIFIED runtime/nn/transformer.c so that its
 * operators (tf_rmsnorm, tf_swiglu_ffn, tf_cached_attention,
 * tf_forward_token) can be called from a hosted process and their results
 * recorded.  The engine's compile-time limits (transformer.h: 128 model
 * dims, 256 positions, 8 heads and layers) are raised before the include,
 * as the llm.c harness does, so that the parity cases can use larger
 * shapes; the engine's static KV store grows with them (zero pages until
 * touched).  Its tensor_cpu helpers (runtime/tensor/tensor_cpu.c) are
 * linked unmodified.
 */
#include "runtime/nn/transformer.h"

#undef TF_MAX_SEQ
#define TF_MAX_SEQ 1024
#undef TF_MAX_DIM
#define TF_MAX_DIM 512
#undef TF_MAX_HEADS
#define TF_MAX_HEADS 16
#undef TF_MAX_LAYERS
#define TF_MAX_LAYERS 4

#include "runtime/nn/transformer.c"

#include <stdlib.h>
#include <string.h>

int ref_tf_max_dim(void) { return TF_MAX_DIM; }
int ref_tf_max_seq(void) { return TF_MAX_SEQ; }

void ref_tf_rmsnorm(float *out, const float *x, const float *w, int dim) { tf_rmsnorm(out, x, w, dim); }

void ref_tf_swiglu_ffn(float *out, const float *x, const float *w1, const float *w2, const float *w3, int dim,
                       int ff_dim)
{
    tf_swiglu_ffn(out, x, w1, w2, w3, dim, ff_dim);
}

/* A tf_model_t over caller-owned fp32 weights (the engine's own structs,
 * transformer.h); one model at a time (the KV store is static). */
typedef struct {
    int dim, num_heads, ff_dim, num_layers, vocab_size, max_seq;
    const float *const *wq, *const *wk, *const *wv, *const *wo;
    const float *const *w1, *const *w2, *const *w3;
    const float *const *rms_att, *const *rms_ffn;
    const float *tok_embed, *rms_final;
} ref_tf_desc_t;

static tf_block_weights_t g_blocks[TF_MAX_LAYERS];
static tf_model_t g_model;

int ref_tf_model_init(const ref_tf_desc_t *d)
{
    if (d->num_layers > TF_MAX_LAYERS || d->dim > TF_MAX_DIM || d->num_heads > TF_MAX_HEADS ||
        d->max_seq > TF_MAX_SEQ || d->ff_dim > 4 * TF_MAX_DIM || d->dim % d->num_heads)
        return -1;
    memset(&g_model, 0, sizeof(g_model));
    for (int L = 0; L < d->num_layers; L++) {
        tf_block_weights_t *b = &g_blocks[L];
        b->wq = (float *)d->wq[L]; b->wk = (float *)d->wk[L]; b->wv = (float *)d->wv[L]; b->wo = (float *)d->wo[L];
        b->w1 = (float *)d->w1[L]; b->w2 = (float *)d->w2[L]; b->w3 = (float *)d->w3[L];
        b->rms_att = (float *)d->rms_att[L]; b->rms_ffn = (float *)d->rms_ffn[L];
    }
    g_model.dim = d->dim;
    g_model.num_heads = d->num_heads;
    g_model.head_dim = d->dim / d->num_heads;
    g_model.ff_dim = d->ff_dim;
    g_model.num_layers = d->num_layers;
    g_model.vocab_size = d->vocab_size;
    g_model.max_seq = d->max_seq;
    g_model.layers = g_blocks;
    g_model.tok_embed = (float *)d->tok_embed;
    g_model.rms_final = (float *)d->rms_final;
    kv_cache_init(&g_model.cache, d->max_seq, g_model.head_dim, d->num_heads, d->num_layers);
    return 0;
}

void ref_tf_forward_token(float *logits, const float *tok_embed_row, int pos)
{
    tf_forward_token(&g_model, logits, tok_embed_row, pos);
}

void ref_tf_cached_attention(float *out, const float *q, const float *k, const float *v, int layer, int head, int pos)
{
    tf_cached_attention(out, q, k, v, &g_model.cache, layer, head, pos);
}

void ref_tf_reset(void) { kv_cache_reset(&g_model.cache); }
