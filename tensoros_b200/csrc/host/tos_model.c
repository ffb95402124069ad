/*
 * tos_model.c - device-resident decoder mirroring llm_forward_token
 * (runtime/nn/llm.c:641-743) and the greedy generate loop (llm.c:1255-1347).
 *
 * Per token the stream runs 5 kernels per layer plus 3:
 *   embed (llm.c:650)
 *   per layer: [rmsnorm + q|k|v GEMV + RoPE + KV store]   llm.c:657-681
 *              [attention scores] [softmax + PV]            llm.c:683-714
 *              [o GEMV + residual]                          llm.c:717-718
 *              [rmsnorm + gate|up GEMV + SiLU*up]           llm.c:723-729
 *              [down GEMV + residual]                       llm.c:732-733
 *   [rmsnorm + LM-head GEMV] [argmax]                       llm.c:737-742, 1129
 * Every launch uses programmatic dependent launch, so a GEMV's weight
 * prefetch overlaps the tail of the kernel before it, and the whole sequence
 * is captured once into a CUDA graph.  The token and position live in device
 * memory (4+4 bytes copied in per call) so the same graph serves every step.
 *
 * Weights are uploaded from the caller's GGUF buffers and repacked into the
 * GEMV plane layout: q|k|v rows concatenated, gate/up rows interleaved
 * (row 2i = gate i, row 2i+1 = up i) so the SiLU*up epilogue sees both.
 *
 * Sharded over G GPUs (tos_model_create_sharded; plan in tos_shard.c) each
 * rank keeps its slice of rows of every projection and its heads' KV cache,
 * and the stream adds four in-place all-gathers per layer (attention output,
 * residual after o, SwiGLU output, residual after down) and, after the LM
 * head, an all-gather of the ranks' (value, index) argmax pairs; the plain
 * (non-chained) step also gathers the logits for tos_model_forward_token.
 */
#include <stdlib.h>
#include <string.h>

#include "tos_internal.h"

struct tos_model {
    tos_model_desc_t d;
    tos_shard_plan_t sp;      /* this rank's rows (everything when world == 1) */
    void *comm;               /* NCCL communicator when world > 1 */
    int hd, kv_dim, q_dim, esz;   /* kv_dim, q_dim: this rank's rows */
    tosk_qmat_t *wqkv, *wo, *wgu, *wdown;
    tosk_qmat_t lm;
    void *embd;
    float *norms;             /* [n_layers][2][dim], then output norm [dim] */
    void *kc, *vc;            /* [n_layers][max_seq][kv_dim] */
    float *x, *q, *att, *h, *logits;   /* x, att, h: full vectors; q, logits: local rows */
    float *logits_full;       /* sharded: gathered logits */
    int *pairs;               /* sharded: [world][2] argmax (value bits, index) */
    float2 *rope;             /* [max_seq][hd/2] */
    void *ws;
    size_t ws_bytes;
    int *io;                  /* device: token, pos, next, err, ring count */
    int *io_host;             /* pinned mirror */
    int *ring;                /* device: tokens produced by tos_model_decode */
    cudaStream_t st;
    cudaGraphExec_t gexec, gexec_chain;
    int have_graph, have_chain;   /* 1: captured, -1: capture unavailable (eager launches) */
    /* one fused kernel per token (decode_step.cu) when FAST on one GPU */
    int fused;
    tosk_step_t step;
    tosk_step_layer_t *step_layers;   /* device [n_layers] */
    unsigned *step_sync;
    /* sharded fused step: the exchange words (tosk_step_ll_words), one
     * allocation shared with the peers through CUDA IPC; peer_base[r] is
     * rank r's, mapped here */
    void *xch;
    size_t xch_bytes;
    void *peer_base[TOSK_MAX_WORLD];
    size_t dev_bytes;
    /* batched prompt pass (allocated on first use): up to pf_cap tokens */
    int pf_cap;
    int *pf_toks;
    float *pf_x, *pf_qkv, *pf_q, *pf_att, *pf_h;
    void *pf_ws;
    size_t pf_ws_bytes;
    /* batched decode (allocated on first use): up to bd_cap sequences, each
     * with its own KV cache [n_layers][bd_cap][max_seq][kv_dim] */
    int bd_cap;
    void *bd_kc, *bd_vc;
    int *bd_io;               /* device: tokens[cap], positions[cap], next[cap], slots[cap] */
    int *bd_host;             /* pinned mirror */
    float *bd_x, *bd_qkv, *bd_q, *bd_att, *bd_h, *bd_logits;
    void *bd_ws;
    size_t bd_ws_bytes;
};

static size_t qrow_bytes(int cols, int type)
{
    return (size_t)(cols / 32) * (type == TOS_TYPE_Q4_0 ? 18 : 34);
}

static size_t embd_row_bytes(int dim, int type)
{
    switch (type) {
    case TOS_TYPE_Q4_0: return (size_t)(dim / 32) * 18;
    case TOS_TYPE_Q8_0: return (size_t)(dim / 32) * 34;
    case TOS_TYPE_F16: return (size_t)dim * 2;
    default: return (size_t)dim * 4;
    }
}

static int dmalloc(tos_model_t *m, void **p, size_t bytes)
{
    int e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) m->dev_bytes += bytes;
    return e;
}

/* Upload n host GGUF matrices (rows[i] x cols, same type) through the staging
 * buffer and repack them into one plane matrix. */
static int upload_qmat(tos_model_t *m, tosk_qmat_t *dst, const void *const *hsrc, const int *rows,
                       int n, int interleave, int type, int cols, void *stage)
{
    int total = 0;
    for (int i = 0; i < n; i++) total += rows[i];
    int e = tosk_qmat_alloc(dst, type, total, cols, m->st);
    if (e) return e;
    m->dev_bytes += dst->bytes;
    const void *dsrc[4];
    size_t off = 0;
    for (int i = 0; i < n; i++) {
        size_t b = qrow_bytes(cols, type) * (size_t)rows[i];
        dsrc[i] = (char *)stage + off;
        e = cudaMemcpyAsync((char *)stage + off, hsrc[i], b, cudaMemcpyHostToDevice, m->st);
        if (e) return e;
        off += (b + 255) & ~(size_t)255;
    }
    e = tosk_qmat_repack(dst, dsrc, rows, n, interleave, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);   /* staging is reused next */
    return e;
}

void tos_model_destroy(tos_model_t *m)
{
    if (!m) return;
    if (m->st) cudaStreamSynchronize(m->st);
    /* graphs holding collectives go before the communicator */
    if (m->have_graph > 0) cudaGraphExecDestroy(m->gexec);
    if (m->have_chain > 0) cudaGraphExecDestroy(m->gexec_chain);
    int mapped = 0;
    for (int r = 0; r < TOSK_MAX_WORLD; r++)
        if (m->peer_base[r] && r != m->sp.rank) {
            cudaIpcCloseMemHandle(m->peer_base[r]);
            mapped = 1;
        }
    if (mapped && m->comm && m->pairs) {
        /* every rank has closed its mappings of the others' exchange
         * buffers before any rank frees its own */
        tos_nccl_all_gather(m->pairs + 2 * m->sp.rank, m->pairs, 2, 1, m->comm, m->st);
        cudaStreamSynchronize(m->st);
    }
    if (m->comm) tos_nccl_comm_destroy(m->comm);
    for (int L = 0; m->wqkv && L < m->d.n_layers; L++) {
        tosk_qmat_free(&m->wqkv[L]);
        tosk_qmat_free(&m->wo[L]);
        tosk_qmat_free(&m->wgu[L]);
        tosk_qmat_free(&m->wdown[L]);
    }
    free(m->wqkv); free(m->wo); free(m->wgu); free(m->wdown);
    tosk_qmat_free(&m->lm);
    void *bufs[] = {m->xch, m->embd, m->norms, m->kc, m->vc, m->x, m->q, m->att, m->h, m->logits,
                    m->step_layers, m->step_sync,
                    m->logits_full, m->pairs, m->rope, m->ws, m->io, m->ring,
                    m->pf_toks, m->pf_x, m->pf_qkv, m->pf_q, m->pf_att, m->pf_h,
                    m->pf_ws, m->bd_kc, m->bd_vc, m->bd_io, m->bd_x, m->bd_qkv,
                    m->bd_q, m->bd_att, m->bd_h, m->bd_logits, m->bd_ws};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++)
        if (bufs[i]) cudaFree(bufs[i]);
    if (m->io_host) cudaFreeHost(m->io_host);
    if (m->bd_host) cudaFreeHost(m->bd_host);
    if (m->st) cudaStreamDestroy(m->st);
    free(m);
}

static int validate(const tos_model_desc_t *d)
{
    if (!d || d->dim <= 0 || d->n_layers <= 0 || d->n_heads <= 0 || d->n_kv_heads <= 0 ||
        d->ff_dim <= 0 || d->vocab_size <= 0 || d->max_seq <= 0)
        return TOS_EINVAL;
    if (d->dim % d->n_heads || d->n_heads % d->n_kv_heads) return TOS_EINVAL;
    if (d->max_seq > TOS_MAX_POS || !tos_rope_args_ok(0, d->rope_base)) return TOS_EINVAL;
    int hd = d->dim / d->n_heads;
    if (hd & 1) return TOS_EINVAL;
    if (d->dim % 32 || d->ff_dim % 32) return TOS_ENOTSUP;
    if (d->wtype != TOS_TYPE_Q4_0 && d->wtype != TOS_TYPE_Q8_0) return TOS_ENOTSUP;
    if (d->kv_type != TOS_TYPE_F32 && d->kv_type != TOS_TYPE_F16) return TOS_ENOTSUP;
    if (d->attn_mode != TOS_ATTN_EXACT && d->attn_mode != TOS_ATTN_FAST) return TOS_EINVAL;
    if (d->gemv_mode != TOS_GEMV_EXACT && d->gemv_mode != TOS_GEMV_FAST) return TOS_EINVAL;
    const void *head = d->output_weight ? d->output_weight : d->token_embd;
    int ht = d->output_weight ? d->out_type : d->embd_type;
    if (!head || (ht != TOS_TYPE_Q4_0 && ht != TOS_TYPE_Q8_0)) return TOS_ENOTSUP;
    if (!d->token_embd || !d->output_norm || !d->attn_norm || !d->ffn_norm || !d->wq || !d->wk ||
        !d->wv || !d->wo || !d->wgate || !d->wup || !d->wdown)
        return TOS_EINVAL;
    return TOS_OK;
}

/* The fused per-token kernel (decode_step.cu) runs the step when the
 * descriptor asks for it (fused_step), the model uses FAST arithmetic on one
 * GPU and the device and shapes allow it. */
/* Sharded fused step: every rank maps every other rank's exchange buffer
 * (CUDA IPC handles swapped with one all-gather on the model's
 * communicator); the kernel's epilogues then store into the peers' vectors
 * directly over NVLink. */
static int map_peers(tos_model_t *m)
{
    const int G = m->sp.world, R = m->sp.rank;
    /* epochs start above 0: a zeroed area holds no word of any exchange */
    m->xch_bytes = tosk_step_ll_words(m->d.n_heads * m->hd, m->d.dim, m->d.ff_dim) * 8;
    int e = dmalloc(m, &m->xch, m->xch_bytes);
    if (!e) e = cudaMemsetAsync(m->xch, 0, m->xch_bytes, m->st);
    if (e) return e;
    cudaIpcMemHandle_t mine;
    e = cudaIpcGetMemHandle(&mine, m->xch);
    if (e) return e;
    const size_t hb = sizeof(cudaIpcMemHandle_t);   /* 64 bytes */
    char *dh = NULL;
    char all[TOSK_MAX_WORLD * sizeof(cudaIpcMemHandle_t)];
    e = cudaMalloc((void **)&dh, hb * (size_t)G);
    if (!e) e = cudaMemcpyAsync(dh + hb * (size_t)R, &mine, hb, cudaMemcpyHostToDevice, m->st);
    if (!e) e = tos_nccl_all_gather(dh + hb * (size_t)R, dh, hb / 4, 1, m->comm, m->st);
    if (!e) e = cudaMemcpyAsync(all, dh, hb * (size_t)G, cudaMemcpyDeviceToHost, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);
    if (dh) cudaFree(dh);
    for (int r = 0; !e && r < G; r++) {
        if (r == R) {
            m->peer_base[r] = m->xch;
            continue;
        }
        cudaIpcMemHandle_t hr;
        memcpy(&hr, all + hb * (size_t)r, hb);
        e = cudaIpcOpenMemHandle(&m->peer_base[r], hr, cudaIpcMemLazyEnablePeerAccess);
    }
    return e;
}

static int setup_step(tos_model_t *m)
{
    const tos_model_desc_t *d = &m->d;
    if (d->gemv_mode != TOS_GEMV_FAST || d->attn_mode != TOS_ATTN_FAST || !d->fused_step) return 0;
    if (m->sp.world > TOSK_MAX_WORLD) return 0;
    if (m->sp.world > 1) {
        int e = map_peers(m);
        if (e) return e;
    }
    /* one GPU: grid barriers between the phases (handing the vectors over
     * as exchange words there measured slower: 2.13 against 1.83 ms a token
     * for the 7B shape) */
    const int L = d->n_layers;
    tosk_step_layer_t *hl = (tosk_step_layer_t *)calloc((size_t)L, sizeof(*hl));
    if (!hl) return cudaErrorMemoryAllocation;
    size_t kv_layer = (size_t)d->max_seq * m->kv_dim * m->esz;
    for (int l = 0; l < L; l++) {
        const tosk_qmat_t *w[4] = {&m->wqkv[l], &m->wo[l], &m->wgu[l], &m->wdown[l]};
        for (int k = 0; k < 4; k++) {
            hl[l].qs[k] = w[k]->qs;
            hl[l].sc[k] = w[k]->sc;
        }
        hl[l].norm_att = m->norms + (size_t)(2 * l) * d->dim;
        hl[l].norm_ffn = m->norms + (size_t)(2 * l + 1) * d->dim;
        hl[l].k_cache = (char *)m->kc + kv_layer * l;
        hl[l].v_cache = (char *)m->vc + kv_layer * l;
    }
    int e = dmalloc(m, (void **)&m->step_layers, (size_t)L * sizeof(*hl));
    if (!e) e = cudaMemcpyAsync(m->step_layers, hl, (size_t)L * sizeof(*hl), cudaMemcpyHostToDevice, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);   /* hl is pageable and freed next */
    free(hl);
    if (!e) e = dmalloc(m, (void **)&m->step_sync, tosk_step_sync_bytes());
    if (!e) e = cudaMemsetAsync(m->step_sync, 0, tosk_step_sync_bytes(), m->st);
    if (e) return e;
    tosk_step_t *s = &m->step;
    memset(s, 0, sizeof(*s));
    s->layers = m->step_layers;
    s->n_layers = L;
    s->wtype = d->wtype;
    s->lm_type = m->lm.type;
    s->lm_qs = m->lm.qs;
    s->lm_sc = m->lm.sc;
    s->norm_out = m->norms + (size_t)2 * L * d->dim;
    s->embd = m->embd;
    s->embd_type = d->embd_type;
    s->x = m->x;
    s->q = m->q;
    s->att = m->att;
    s->h = m->h;
    s->logits = m->logits;
    s->attn_ws = m->ws;
    s->rope = m->rope;
    s->io = m->io;
    s->ring = m->ring;
    s->sync = m->step_sync;
    s->dim = d->dim;
    s->ff = d->ff_dim;
    s->n_heads = d->n_heads;
    s->n_kv = d->n_kv_heads;
    s->hd = m->hd;
    s->vocab = d->vocab_size;
    s->max_seq = d->max_seq;
    s->kv_type = d->kv_type;
    s->eps = d->norm_eps;
    s->vocab = m->sp.n_vocab;
    s->n_heads = m->sp.n_heads;
    s->n_kv = m->sp.n_kv_heads;
    if (m->sp.world > 1) {
        const tos_shard_plan_t *sp = &m->sp;
        s->world = sp->world;
        s->rank = sp->rank;
        s->n_rows = sp->n_rows;
        s->n_ff = sp->n_ff;
        s->q_full = d->n_heads * m->hd;
        s->q0 = sp->q_row0;
        s->row0 = sp->row0;
        s->ff0 = sp->ff0;
        s->vocab0 = sp->vocab0;
        for (int r = 0; r < sp->world; r++) s->peer_ll[r] = (unsigned long long *)m->peer_base[r];
    }
    /* shapes or devices the fused kernel does not cover keep the per-operator path */
    m->fused = tosk_step_check(s) == 0;
    cudaGetLastError();
    return 0;
}

static int create_impl(tos_model_t **out, const tos_model_desc_t *d, int world, int rank, const void *nccl_id)
{
    if (!out) return tos_set_status(TOS_EINVAL);
    *out = NULL;
    int rc = validate(d);
    if (rc) return tos_set_status(rc);
    if (world < 1 || rank < 0 || rank >= world || (world > 1 && !nccl_id)) return tos_set_status(TOS_EINVAL);
    rc = tos_ensure_init();
    if (rc) return tos_set_status(rc);
    tos_shard_plan_t sp;
    rc = tos_shard_plan(d, world, rank, &sp);
    if (rc) return tos_set_status(rc);
    tos_model_t *m = (tos_model_t *)calloc(1, sizeof(*m));
    if (!m) return tos_set_status(TOS_ENOMEM);
    m->d = *d;
    m->sp = sp;
    const int L = d->n_layers, dim = d->dim, ff = d->ff_dim;
    m->hd = dim / d->n_heads;
    m->q_dim = sp.n_q_rows;
    m->kv_dim = sp.n_kv_rows;
    m->esz = d->kv_type == TOS_TYPE_F16 ? 2 : 4;
    const int full_q = d->n_heads * m->hd;
    int e = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking);
    if (!e && world > 1) {
        rc = tos_nccl_comm_init(&m->comm, world, rank, nccl_id);
        if (rc) { tos_model_destroy(m); return tos_set_status(rc); }
    }
    m->wqkv = (tosk_qmat_t *)calloc((size_t)L, sizeof(tosk_qmat_t));
    m->wo = (tosk_qmat_t *)calloc((size_t)L, sizeof(tosk_qmat_t));
    m->wgu = (tosk_qmat_t *)calloc((size_t)L, sizeof(tosk_qmat_t));
    m->wdown = (tosk_qmat_t *)calloc((size_t)L, sizeof(tosk_qmat_t));
    if (!m->wqkv || !m->wo || !m->wgu || !m->wdown) { tos_model_destroy(m); return tos_set_status(TOS_ENOMEM); }

    const int wt = d->wtype;
    const void *head = d->output_weight ? d->output_weight : d->token_embd;
    const int ht = d->output_weight ? d->out_type : d->embd_type;
    /* staging holds the GGUF sources of one plane matrix, each 256-aligned */
#define AL256(v) (((v) + 255) & ~(size_t)255)
    size_t stage_b = 0, t;
    t = AL256(qrow_bytes(dim, wt) * (size_t)m->q_dim) + 2 * AL256(qrow_bytes(dim, wt) * (size_t)m->kv_dim);
    if (t > stage_b) stage_b = t;
    t = 2 * AL256(qrow_bytes(dim, wt) * (size_t)ff); if (t > stage_b) stage_b = t;
    t = AL256(qrow_bytes(ff, wt) * (size_t)dim); if (t > stage_b) stage_b = t;
    t = AL256(qrow_bytes(full_q, wt) * (size_t)dim); if (t > stage_b) stage_b = t;
    t = AL256(qrow_bytes(dim, ht) * (size_t)d->vocab_size); if (t > stage_b) stage_b = t;
#undef AL256
    void *stage = NULL;
    if (!e) e = cudaMalloc(&stage, stage_b);

    /* this rank's rows of each GGUF matrix (row-major: a row range is one
     * contiguous byte range) */
#define ROWS(p, r0, cols, type) ((const char *)(p) + (size_t)(r0) * qrow_bytes((cols), (type)))
    for (int l = 0; !e && l < L; l++) {
        const void *qkv[3] = {ROWS(d->wq[l], sp.q_row0, dim, wt), ROWS(d->wk[l], sp.kv_row0, dim, wt),
                              ROWS(d->wv[l], sp.kv_row0, dim, wt)};
        int rq[3] = {m->q_dim, m->kv_dim, m->kv_dim};
        e = upload_qmat(m, &m->wqkv[l], qkv, rq, 3, 0, wt, dim, stage);
        if (!e) { const void *s1[1] = {ROWS(d->wo[l], sp.row0, full_q, wt)}; int r1[1] = {sp.n_rows}; e = upload_qmat(m, &m->wo[l], s1, r1, 1, 0, wt, full_q, stage); }
        if (!e) { const void *gu[2] = {ROWS(d->wgate[l], sp.ff0, dim, wt), ROWS(d->wup[l], sp.ff0, dim, wt)}; int r2[2] = {sp.n_ff, sp.n_ff}; e = upload_qmat(m, &m->wgu[l], gu, r2, 2, 1, wt, dim, stage); }
        if (!e) { const void *s1[1] = {ROWS(d->wdown[l], sp.row0, ff, wt)}; int r1[1] = {sp.n_rows}; e = upload_qmat(m, &m->wdown[l], s1, r1, 1, 0, wt, ff, stage); }
    }
    if (!e) { const void *s1[1] = {ROWS(head, sp.vocab0, dim, ht)}; int r1[1] = {sp.n_vocab}; e = upload_qmat(m, &m->lm, s1, r1, 1, 0, ht, dim, stage); }
#undef ROWS
    if (stage) cudaFree(stage);

    /* Every device write of the set-up goes on the model's stream, which does
     * not synchronise with the legacy default stream (cudaStreamNonBlocking):
     * a plain cudaMemset or a pageable cudaMemcpy there could still be in
     * flight when the first step runs on m->st, and a late clear of the KV
     * cache or of io[] would then overwrite what that step wrote.  The host
     * sources are pageable and stay valid until the final synchronise. */
    size_t eb = embd_row_bytes(dim, d->embd_type) * (size_t)d->vocab_size;
    if (!e) e = dmalloc(m, &m->embd, eb);
    if (!e) e = cudaMemcpyAsync(m->embd, d->token_embd, eb, cudaMemcpyHostToDevice, m->st);
    size_t nb = ((size_t)L * 2 + 1) * (size_t)dim * 4;
    if (!e) e = dmalloc(m, (void **)&m->norms, nb);
    for (int l = 0; !e && l < L; l++) {
        e = cudaMemcpyAsync(m->norms + (size_t)(2 * l) * dim, d->attn_norm[l], (size_t)dim * 4,
                            cudaMemcpyHostToDevice, m->st);
        if (!e) e = cudaMemcpyAsync(m->norms + (size_t)(2 * l + 1) * dim, d->ffn_norm[l], (size_t)dim * 4,
                                    cudaMemcpyHostToDevice, m->st);
    }
    if (!e) e = cudaMemcpyAsync(m->norms + (size_t)2 * L * dim, d->output_norm, (size_t)dim * 4,
                                cudaMemcpyHostToDevice, m->st);

    size_t kvb = (size_t)L * d->max_seq * m->kv_dim * m->esz;
    if (!e) e = dmalloc(m, &m->kc, kvb);
    if (!e) e = dmalloc(m, &m->vc, kvb);
    if (!e) e = cudaMemsetAsync(m->kc, 0, kvb, m->st);
    if (!e) e = cudaMemsetAsync(m->vc, 0, kvb, m->st);
    int mx = dim > ff ? dim : ff;
    if (!e) e = dmalloc(m, (void **)&m->x, (size_t)dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->q, (size_t)mx * 4);
    if (!e) e = dmalloc(m, (void **)&m->att, (size_t)mx * 4);
    if (!e) e = dmalloc(m, (void **)&m->h, (size_t)ff * 4);
    if (!e) e = dmalloc(m, (void **)&m->logits, (size_t)sp.n_vocab * 4);
    if (!e && world > 1) e = dmalloc(m, (void **)&m->logits_full, (size_t)d->vocab_size * 4);
    if (!e && world > 1) e = dmalloc(m, (void **)&m->pairs, (size_t)world * 2 * sizeof(int));
    if (!e) e = dmalloc(m, (void **)&m->rope, (size_t)d->max_seq * (m->hd / 2) * sizeof(float2));
    if (!e) e = tosk_rope_table(m->rope, d->max_seq, m->hd, d->rope_base, m->st);
    m->ws_bytes = tosk_attention_ws_bytes(sp.n_heads, d->max_seq);
    if (!e) e = dmalloc(m, &m->ws, m->ws_bytes);
    /* the fused step's per-head counters live in it and start at zero */
    if (!e) e = cudaMemsetAsync(m->ws, 0, m->ws_bytes, m->st);
    if (!e) e = dmalloc(m, (void **)&m->io, 8 * sizeof(int));
    if (!e) e = cudaMemsetAsync(m->io, 0, 8 * sizeof(int), m->st);
    if (!e) e = dmalloc(m, (void **)&m->ring, (size_t)d->max_seq * sizeof(int));
    if (!e) e = cudaMallocHost((void **)&m->io_host, 8 * sizeof(int));
    if (!e) e = setup_step(m);
    if (!e) e = cudaStreamSynchronize(m->st);
    if (e) {
        tos_model_destroy(m);
        return tos_set_status(tos_from_cuda(e));
    }
    *out = m;
    return tos_set_status(TOS_OK);
}

int tos_model_create(tos_model_t **out, const tos_model_desc_t *d)
{
    return create_impl(out, d, 1, 0, NULL);
}

int tos_model_create_sharded(tos_model_t **out, const tos_model_desc_t *d, int rank, int world,
                             const void *nccl_id)
{
    return create_impl(out, d, world, rank, nccl_id);
}

size_t tos_model_device_bytes(const tos_model_t *m) { return m ? m->dev_bytes : 0; }
int tos_model_fused(const tos_model_t *m) { return m ? m->fused : 0; }
const float *tos_model_logits_dev(const tos_model_t *m)
{
    return m ? (m->sp.world > 1 ? m->logits_full : m->logits) : NULL;
}

int tos_model_reset(tos_model_t *m)
{
    if (!m) return tos_set_status(TOS_EINVAL);
    size_t kvb = (size_t)m->d.n_layers * m->d.max_seq * m->kv_dim * m->esz;
    int e = cudaMemsetAsync(m->kc, 0, kvb, m->st);
    if (!e) e = cudaMemsetAsync(m->vc, 0, kvb, m->st);
    if (!e && m->bd_cap) e = cudaMemsetAsync(m->bd_kc, 0, kvb * m->bd_cap, m->st);
    if (!e && m->bd_cap) e = cudaMemsetAsync(m->bd_vc, 0, kvb * m->bd_cap, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);
    return tos_set_status(tos_from_cuda(e));
}

static int enqueue_head(tos_model_t *m, int chained);

/* In-place all-gather: this rank's count floats sit at full + rank*count. */
static int gather(tos_model_t *m, float *full, int count)
{
    return tos_nccl_all_gather(full + (size_t)m->sp.rank * count, full, (size_t)count, 0, m->comm, m->st);
}

static int gather_to(tos_model_t *m, const float *mine, float *full, int count)
{
    return tos_nccl_all_gather(mine, full, (size_t)count, 0, m->comm, m->st);
}

/* Enqueue one token step; reads the token from io[0] (io[2] when chained:
 * the previous step's argmax) and the position from io[1], leaves the greedy
 * next token in io[2].  A chained step then records it and advances io[1]. */
static int enqueue_token(tos_model_t *m, int chained)
{
    if (m->fused) {
        m->step.chained = chained;
        int e = tosk_step_launch(&m->step, m->st);
        /* sharded: each rank holds its vocabulary rows; a plain step hands
         * out the whole logits vector */
        if (!e && m->sp.world > 1 && !chained) e = gather_to(m, m->logits, m->logits_full, m->sp.n_vocab);
        return e;
    }
    const tos_model_desc_t *d = &m->d;
    cudaStream_t st = m->st;
    int *err = m->io + 3;
    const int pdl = 1;
    const int dim = d->dim;
    const tos_shard_plan_t *sp = &m->sp;
    const int G = sp->world;
    size_t kv_layer = (size_t)d->max_seq * m->kv_dim * m->esz;
    int e = tosk_embed(m->x, m->embd, d->embd_type, dim, chained ? m->io + 2 : m->io, 0, pdl, st);
    for (int l = 0; !e && l < d->n_layers; l++) {
        tosk_norm_t n1 = {m->norms + (size_t)(2 * l) * dim, d->norm_eps};
        tosk_epi_t qkv;
        memset(&qkv, 0, sizeof(qkv));
        qkv.kind = TOSK_EPI_QKV;
        qkv.rope_cs = m->rope;
        qkv.pos = m->io + 1;
        qkv.hd = m->hd;
        qkv.q_rows = m->q_dim;
        qkv.kv_rows = m->kv_dim;
        qkv.kv_type = d->kv_type;
        qkv.k_cache = (char *)m->kc + kv_layer * l;
        qkv.v_cache = (char *)m->vc + kv_layer * l;
        e = tosk_gemv(&m->wqkv[l], m->x, &n1, m->q, &qkv, d->gemv_mode, err, pdl, st);
        float *att = m->att + sp->q_row0;   /* this rank's heads of the full output */
        if (!e) e = tosk_attention(att, m->q, qkv.k_cache, qkv.v_cache, d->kv_type, sp->n_heads,
                                   sp->n_kv_heads, m->hd, m->io + 1, 0, d->max_seq, d->attn_mode, m->ws,
                                   m->ws_bytes, err, pdl, st);
        if (!e && G > 1) e = gather(m, m->att, sp->n_q_rows);
        tosk_epi_t res;
        memset(&res, 0, sizeof(res));
        res.kind = TOSK_EPI_RESID;
        res.resid = m->x + sp->row0;
        if (!e) e = tosk_gemv(&m->wo[l], m->att, NULL, m->x + sp->row0, &res, d->gemv_mode, err, pdl, st);
        if (!e && G > 1) e = gather(m, m->x, sp->n_rows);
        tosk_norm_t n2 = {m->norms + (size_t)(2 * l + 1) * dim, d->norm_eps};
        tosk_epi_t sw;
        memset(&sw, 0, sizeof(sw));
        sw.kind = TOSK_EPI_SWIGLU;
        if (!e) e = tosk_gemv(&m->wgu[l], m->x, &n2, m->h + sp->ff0, &sw, d->gemv_mode, err, pdl, st);
        if (!e && G > 1) e = gather(m, m->h, sp->n_ff);
        if (!e) e = tosk_gemv(&m->wdown[l], m->h, NULL, m->x + sp->row0, &res, d->gemv_mode, err, pdl, st);
        if (!e && G > 1) e = gather(m, m->x, sp->n_rows);
    }
    if (!e) e = enqueue_head(m, chained);
    return e;
}

/* Final norm, LM head and greedy token (llm.c:737-742, 1129) from m->x. */
static int enqueue_head(tos_model_t *m, int chained)
{
    const tos_model_desc_t *d = &m->d;
    const tos_shard_plan_t *sp = &m->sp;
    const int G = sp->world, pdl = 1;
    cudaStream_t st = m->st;
    int *err = m->io + 3;
    int e = 0;
    tosk_norm_t no = {m->norms + (size_t)2 * d->n_layers * d->dim, d->norm_eps};
    if (!e) e = tosk_gemv(&m->lm, m->x, &no, m->logits, NULL, d->gemv_mode, err, pdl, st);
    if (G == 1) {
        if (!e) e = tosk_argmax(m->logits, d->vocab_size, m->io + 2, NULL, pdl, st);
    } else {
        int *mine = m->pairs + 2 * sp->rank;
        if (!e) e = tosk_argmax_slice(m->logits, sp->n_vocab, sp->vocab0, sp->rank == 0, mine, pdl, st);
        if (!e) e = tos_nccl_all_gather(mine, m->pairs, 2, 1, m->comm, st);
        if (!e) e = tosk_argmax_pairs(m->pairs, G, m->io + 2, pdl, st);
        if (!e && !chained) e = gather_to(m, m->logits, m->logits_full, sp->n_vocab);
    }
    if (!e && chained) e = tosk_decode_advance(m->io, m->ring, pdl, st);
    return e;
}

/* Captures the (plain or chained) token step into a graph. */
static int capture(tos_model_t *m, int chained, cudaGraphExec_t *out)
{
    cudaGraph_t g = NULL;
    int ok = 0;
    if (cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        int ce = enqueue_token(m, chained);
        int ee = cudaStreamEndCapture(m->st, &g);
        if (!ce && !ee && g && cudaGraphInstantiate(out, g, 0) == cudaSuccess) ok = 1;
        if (g) cudaGraphDestroy(g);
    }
    cudaGetLastError();
    return ok;
}

static int run_token(tos_model_t *m, int token, int pos)
{
    if (token < 0 || token >= m->d.vocab_size || pos < 0 || pos >= m->d.max_seq) return TOS_EINVAL;
    m->io_host[0] = token;
    m->io_host[1] = pos;
    int e = cudaMemcpyAsync(m->io, m->io_host, 2 * sizeof(int), cudaMemcpyHostToDevice, m->st);
    if (e) return tos_from_cuda(e);
    if (m->have_graph <= 0) {
        /* first step runs eagerly (sets kernel attributes), then capture;
         * without a graph every step stays eager */
        e = enqueue_token(m, 0);
        if (!e && m->have_graph == 0) {
            e = cudaStreamSynchronize(m->st);
            if (!e) m->have_graph = capture(m, 0, &m->gexec) ? 1 : -1;
        }
        if (e) return tos_from_cuda(e);
    } else {
        e = cudaGraphLaunch(m->gexec, m->st);
        if (e) return tos_from_cuda(e);
    }
    return TOS_OK;
}

/* After a bounded wait ran out: clear the error word and the fused step's
 * barrier counters (a step that stopped early leaves them mid-count). */
static void clear_error(tos_model_t *m)
{
    cudaMemsetAsync(m->io + 3, 0, sizeof(int), m->st);
    if (m->step_sync) cudaMemsetAsync(m->step_sync, 0, tosk_step_sync_bytes(), m->st);
    if (m->step_sync && m->ws) cudaMemsetAsync(m->ws, 0, m->ws_bytes, m->st);   /* attention counters */
    /* one GPU: the exchange words restart from a cleared area at epoch 0 (a
     * step that stopped early leaves words of its epochs behind).  A sharded
     * model cannot restart its peers' epochs from here: after a timeout it is
     * destroyed and created again on every rank. */
    if (m->xch && m->sp.world == 1) {
        cudaMemsetAsync(m->io + 5, 0, sizeof(int), m->st);
        cudaMemsetAsync(m->xch, 0, m->xch_bytes, m->st);
    }
    cudaStreamSynchronize(m->st);
}

static int finish(tos_model_t *m, float *logits, int *next)
{
    int e = cudaMemcpyAsync(m->io_host + 2, m->io + 2, 2 * sizeof(int), cudaMemcpyDeviceToHost, m->st);
    if (!e && logits)
        e = cudaMemcpyAsync(logits, m->sp.world > 1 ? m->logits_full : m->logits, (size_t)m->d.vocab_size * 4,
                            cudaMemcpyDeviceToHost, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);
    if (e) return tos_from_cuda(e);
    if (m->io_host[3] != 0) {
        clear_error(m);
        return TOS_ETIMEOUT;
    }
    if (next) *next = m->io_host[2];
    return TOS_OK;
}

int tos_model_forward_token(tos_model_t *m, float *logits, int token, int pos)
{
    if (!m) return tos_set_status(TOS_EINVAL);
    int rc = run_token(m, token, pos);
    if (!rc) rc = finish(m, logits, NULL);
    return tos_set_status(rc);
}

int tos_model_forward_argmax(tos_model_t *m, int token, int pos, int *next)
{
    if (!m || !next) return tos_set_status(TOS_EINVAL);
    int rc = run_token(m, token, pos);
    if (!rc) rc = finish(m, NULL, next);
    return tos_set_status(rc);
}

int tos_model_generate_greedy(tos_model_t *m, const int *prompt, int n_prompt, int n_gen, int *out)
{
    if (!m || n_prompt < 0 || n_gen < 0 || (n_prompt && !prompt) || (n_gen && !out))
        return tos_set_status(TOS_EINVAL);
    if (n_prompt == 0) return tos_set_status(TOS_EINVAL);
    int pos = 0, next = 0, rc = TOS_OK;
    for (int i = 0; i < n_prompt && !rc; i++) rc = tos_model_forward_argmax(m, prompt[i], pos++, &next);
    int g = 0;
    for (; !rc && g < n_gen && pos < m->d.max_seq; g++) {
        out[g] = next;
        rc = tos_model_forward_argmax(m, next, pos++, &next);
    }
    if (rc) return tos_set_status(rc);
    tos_set_status(TOS_OK);
    return g;
}

void *tos_model_stream(const tos_model_t *m) { return m ? (void *)m->st : NULL; }

int tos_model_decode(tos_model_t *m, int token, int pos, int n_steps, int *out_tokens)
{
    if (!m || n_steps < 0 || (n_steps && !out_tokens)) return tos_set_status(TOS_EINVAL);
    if (token < 0 || token >= m->d.vocab_size || pos < 0 || pos + n_steps > m->d.max_seq)
        return tos_set_status(TOS_EINVAL);
    if (n_steps == 0) return tos_set_status(TOS_OK);
    m->io_host[0] = token;
    m->io_host[1] = pos;
    m->io_host[2] = token;
    m->io_host[3] = 0;
    m->io_host[4] = 0;
    int e = cudaMemcpyAsync(m->io, m->io_host, 5 * sizeof(int), cudaMemcpyHostToDevice, m->st);
    int step = 0;
    if (!e && m->have_chain == 0) {
        /* one eager chained step (configures kernels), then capture */
        e = enqueue_token(m, 1);
        if (!e) e = cudaStreamSynchronize(m->st);
        step = 1;
        if (!e) m->have_chain = capture(m, 1, &m->gexec_chain) ? 1 : -1;
    }
    for (; !e && step < n_steps; step++)
        e = m->have_chain > 0 ? cudaGraphLaunch(m->gexec_chain, m->st) : enqueue_token(m, 1);
    if (!e) e = cudaMemcpyAsync(out_tokens, m->ring, (size_t)n_steps * sizeof(int), cudaMemcpyDeviceToHost, m->st);
    if (!e) e = cudaMemcpyAsync(m->io_host + 3, m->io + 3, sizeof(int), cudaMemcpyDeviceToHost, m->st);
    if (!e) e = cudaStreamSynchronize(m->st);
    if (e) return tos_set_status(tos_from_cuda(e));
    if (m->io_host[3] != 0) {
        clear_error(m);
        return tos_set_status(TOS_ETIMEOUT);
    }
    return tos_set_status(TOS_OK);
}

/* ---------------------------------------------------------------- prefill */

#define TOS_PF_CAP 128

static int pf_alloc(tos_model_t *m)
{
    if (m->pf_cap) return 0;
    const tos_model_desc_t *d = &m->d;
    const int C = TOS_PF_CAP, dim = d->dim, ff = d->ff_dim;
    const int nqkv = m->q_dim + 2 * m->kv_dim;
    int e = dmalloc(m, (void **)&m->pf_toks, (size_t)C * sizeof(int));
    if (!e) e = dmalloc(m, (void **)&m->pf_x, (size_t)C * dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->pf_qkv, (size_t)C * nqkv * 4);
    if (!e) e = dmalloc(m, (void **)&m->pf_q, (size_t)C * m->q_dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->pf_att, (size_t)C * m->q_dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->pf_h, (size_t)C * ff * 4);
    size_t ws = 0, t;
    t = tosk_gemm_ws_bytes(C, nqkv, dim); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, dim, m->q_dim); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, 2 * ff, dim); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, dim, ff); if (t > ws) ws = t;
    if (!e) e = dmalloc(m, &m->pf_ws, ws);
    if (e) return e;
    m->pf_ws_bytes = ws;
    m->pf_cap = C;
    return 0;
}

/* n <= TOS_PF_CAP tokens at positions pos0.. through every layer with the
 * projections as batched tensor-core GEMMs; leaves the last token's row in
 * m->x. */
static int pf_chunk(tos_model_t *m, const int *tokens, int n, int pos0)
{
    const tos_model_desc_t *d = &m->d;
    cudaStream_t st = m->st;
    int *err = m->io + 3;
    const int dim = d->dim, hd = m->hd;
    const int nqkv = m->q_dim + 2 * m->kv_dim;
    size_t kv_layer = (size_t)d->max_seq * m->kv_dim * m->esz;
    int e = cudaMemcpyAsync(m->pf_toks, tokens, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, st);
    if (!e) e = tosk_pf_embed(m->pf_x, m->embd, d->embd_type, dim, m->pf_toks, n, st);
    for (int l = 0; !e && l < d->n_layers; l++) {
        void *kc = (char *)m->kc + kv_layer * l, *vc = (char *)m->vc + kv_layer * l;
        e = tosk_gemm_q_norm(&m->wqkv[l], m->pf_x, m->norms + (size_t)(2 * l) * dim, d->norm_eps, n, m->pf_qkv,
                             m->pf_ws, m->pf_ws_bytes, err, 1, st);
        if (!e) e = tosk_pf_rope_store(m->pf_qkv, m->q_dim, m->kv_dim, hd, m->rope, pos0, m->pf_q, kc, vc,
                                       d->kv_type, n, st);
        if (!e) e = tosk_pf_attention(m->pf_q, kc, vc, d->kv_type, d->n_heads, d->n_kv_heads, hd, pos0, n,
                                      m->pf_att, st);
        /* the residual adds and SiLU*up run in the GEMMs' epilogues */
        if (!e) e = tosk_gemm_q_residual(&m->wo[l], m->pf_att, n, m->pf_x, m->pf_ws, m->pf_ws_bytes, err, 1,
                                         st);
        if (!e) e = tosk_gemm_q_norm_swiglu(&m->wgu[l], m->pf_x, m->norms + (size_t)(2 * l + 1) * dim,
                                            d->norm_eps, n, m->pf_h, m->pf_ws, m->pf_ws_bytes, err, 1, st);
        if (!e) e = tosk_gemm_q_residual(&m->wdown[l], m->pf_h, n, m->pf_x, m->pf_ws, m->pf_ws_bytes, err,
                                         1, st);
    }
    (void)nqkv;
    if (!e) e = cudaMemcpyAsync(m->x, m->pf_x + (size_t)(n - 1) * dim, (size_t)dim * 4, cudaMemcpyDeviceToDevice, st);
    return e;
}

int tos_model_prefill(tos_model_t *m, const int *tokens, int n, int pos0, float *logits, int *next)
{
    if (!m || !tokens || n <= 0 || pos0 < 0 || pos0 + n > m->d.max_seq) return tos_set_status(TOS_EINVAL);
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= m->d.vocab_size) return tos_set_status(TOS_EINVAL);
    /* batched GEMMs take K in 64-column chunks; one rank's model only */
    if (m->sp.world > 1 || m->d.dim % 64 || m->d.ff_dim % 64 || m->q_dim % 64) return tos_set_status(TOS_ENOTSUP);
    int e = pf_alloc(m);
    for (int c0 = 0; !e && c0 < n; c0 += TOS_PF_CAP) {
        const int nc = n - c0 < TOS_PF_CAP ? n - c0 : TOS_PF_CAP;
        e = pf_chunk(m, tokens + c0, nc, pos0 + c0);
        /* the host token buffer is read by the copy above: finish it before
         * the next chunk reuses the device token array */
        if (!e) e = cudaStreamSynchronize(m->st);
    }
    if (!e) e = enqueue_head(m, 0);
    if (e) return tos_set_status(tos_from_cuda(e));
    return tos_set_status(finish(m, logits, next));
}

/* --------------------------------------------------------- batched decode */

#define TOS_BATCH_CAP 16

static int bd_alloc(tos_model_t *m)
{
    if (m->bd_cap) return 0;
    const tos_model_desc_t *d = &m->d;
    const int C = TOS_BATCH_CAP, dim = d->dim, ff = d->ff_dim;
    const int nqkv = m->q_dim + 2 * m->kv_dim;
    const size_t kvb = (size_t)d->n_layers * C * d->max_seq * m->kv_dim * m->esz;
    int e = dmalloc(m, &m->bd_kc, kvb);
    if (!e) e = dmalloc(m, &m->bd_vc, kvb);
    if (!e) e = cudaMemsetAsync(m->bd_kc, 0, kvb, m->st);
    if (!e) e = cudaMemsetAsync(m->bd_vc, 0, kvb, m->st);
    if (!e) e = dmalloc(m, (void **)&m->bd_io, (size_t)4 * C * sizeof(int));
    if (!e) e = cudaMallocHost((void **)&m->bd_host, (size_t)4 * C * sizeof(int));
    if (!e) e = dmalloc(m, (void **)&m->bd_x, (size_t)C * dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->bd_qkv, (size_t)C * nqkv * 4);
    if (!e) e = dmalloc(m, (void **)&m->bd_q, (size_t)C * m->q_dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->bd_att, (size_t)C * m->q_dim * 4);
    if (!e) e = dmalloc(m, (void **)&m->bd_h, (size_t)C * ff * 4);
    if (!e) e = dmalloc(m, (void **)&m->bd_logits, (size_t)C * d->vocab_size * 4);
    size_t ws = 0, t;
    t = tosk_gemm_ws_bytes(C, nqkv, dim); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, dim, m->q_dim); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, 2 * ff, dim); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, dim, ff); if (t > ws) ws = t;
    t = tosk_gemm_ws_bytes(C, d->vocab_size, dim); if (t > ws) ws = t;
    if (!e) e = dmalloc(m, &m->bd_ws, ws);
    if (e) return e;
    m->bd_ws_bytes = ws;
    m->bd_cap = C;
    return 0;
}

/* One greedy step of n independent sequences: token[i] at position pos[i]
 * of the sequence in cache slot slot[i] (distinct slots).  The projections
 * are tensor-core GEMMs over the n tokens (tos_gemm_dev numerics), attention
 * is per sequence. */
int tos_model_decode_batch(tos_model_t *m, const int *slot, const int *tokens, const int *pos, int n,
                           float *logits, int *next)
{
    if (!m || !slot || !tokens || !pos || n <= 0 || n > TOS_BATCH_CAP) return tos_set_status(TOS_EINVAL);
    const tos_model_desc_t *d = &m->d;
    unsigned used = 0;
    for (int i = 0; i < n; i++) {
        if (tokens[i] < 0 || tokens[i] >= d->vocab_size || pos[i] < 0 || pos[i] >= d->max_seq ||
            slot[i] < 0 || slot[i] >= TOS_BATCH_CAP || (used >> slot[i] & 1u))
            return tos_set_status(TOS_EINVAL);
        used |= 1u << slot[i];
    }
    if (m->sp.world > 1 || d->dim % 64 || d->ff_dim % 64 || m->q_dim % 64) return tos_set_status(TOS_ENOTSUP);
    int e = bd_alloc(m);
    if (e) return tos_set_status(tos_from_cuda(e));
    cudaStream_t st = m->st;
    int *err = m->io + 3;
    const int C = m->bd_cap, dim = d->dim, hd = m->hd;
    const size_t cstride = (size_t)d->max_seq * m->kv_dim;           /* elements per sequence */
    const size_t kv_layer = cstride * C * m->esz;                    /* bytes per layer */
    memcpy(m->bd_host, tokens, (size_t)n * sizeof(int));
    memcpy(m->bd_host + C, pos, (size_t)n * sizeof(int));
    memcpy(m->bd_host + 3 * C, slot, (size_t)n * sizeof(int));
    e = cudaMemcpyAsync(m->bd_io, m->bd_host, (size_t)4 * C * sizeof(int), cudaMemcpyHostToDevice, st);
    if (!e) e = tosk_pf_embed(m->bd_x, m->embd, d->embd_type, dim, m->bd_io, n, st);
    for (int l = 0; !e && l < d->n_layers; l++) {
        void *kc = (char *)m->bd_kc + kv_layer * l, *vc = (char *)m->bd_vc + kv_layer * l;
        e = tosk_gemm_q_norm(&m->wqkv[l], m->bd_x, m->norms + (size_t)(2 * l) * dim, d->norm_eps, n, m->bd_qkv,
                             m->bd_ws, m->bd_ws_bytes, err, 1, st);
        if (!e) e = tosk_bd_rope_store(m->bd_qkv, m->q_dim, m->kv_dim, hd, m->rope, m->bd_io + C, m->bd_io + 3 * C,
                                       m->bd_q, kc, vc, cstride, d->kv_type, n, st);
        if (!e) e = tosk_bd_attention(m->bd_q, kc, vc, cstride, d->kv_type, d->n_heads, d->n_kv_heads, hd,
                                      m->bd_io + C, m->bd_io + 3 * C, d->max_seq, n, m->bd_att, st);
        /* the residual adds and SiLU*up run in the GEMMs' epilogues */
        if (!e) e = tosk_gemm_q_residual(&m->wo[l], m->bd_att, n, m->bd_x, m->bd_ws, m->bd_ws_bytes, err, 1,
                                         st);
        if (!e) e = tosk_gemm_q_norm_swiglu(&m->wgu[l], m->bd_x, m->norms + (size_t)(2 * l + 1) * dim,
                                            d->norm_eps, n, m->bd_h, m->bd_ws, m->bd_ws_bytes, err, 1, st);
        if (!e) e = tosk_gemm_q_residual(&m->wdown[l], m->bd_h, n, m->bd_x, m->bd_ws, m->bd_ws_bytes, err,
                                         1, st);
    }
    if (!e) e = tosk_gemm_q_norm(&m->lm, m->bd_x, m->norms + (size_t)2 * d->n_layers * dim, d->norm_eps, n,
                                 m->bd_logits, m->bd_ws, m->bd_ws_bytes, err, 1, st);
    if (!e) e = tosk_argmax_rows(m->bd_logits, d->vocab_size, n, m->bd_io + 2 * C, st);
    if (!e) e = cudaMemcpyAsync(m->bd_host + 2 * C, m->bd_io + 2 * C, (size_t)n * sizeof(int),
                                cudaMemcpyDeviceToHost, st);
    if (!e && logits)
        e = cudaMemcpyAsync(logits, m->bd_logits, (size_t)n * d->vocab_size * 4, cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaMemcpyAsync(m->io_host + 3, m->io + 3, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaStreamSynchronize(st);
    if (e) return tos_set_status(tos_from_cuda(e));
    if (m->io_host[3] != 0) {
        clear_error(m);
        return tos_set_status(TOS_ETIMEOUT);
    }
    if (next) memcpy(next, m->bd_host + 2 * C, (size_t)n * sizeof(int));
    return tos_set_status(TOS_OK);
}
