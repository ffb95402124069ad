/*
 * ref_llm_hosted.c - hosted build of the reference decode path (test infrastructure).
 *
 * This translation unit textually includes the UNMODIFIED reference source
 * runtime/nn/llm.c (TensorOS) so that its file-static operators can be called
 * from a hosted Linux process.  It is compiled only by oracle/Makefile into
 * oracle/_ref/libtos_ref.so and is used by the tests as the checker of the
 * restatement in oracle/tos_oracle.c; nothing in the product links it.
 *
 * Build notes:
 *  - llm.c:864 calls llm_build_hash_table, which is defined static later
 *    (llm.c:893); gcc rejects the implicit declaration, so it is declared here.
 *  - The limits in llm.h:29-37 are raised so that the Llama-2-7B shape
 *    (dim 4096, ff 11008, ctx > 2048) fits the static scratch buffers
 *    (llm.c:48-65).  The KV cache is supplied by the harness (llm.h:100-101),
 *    so LLM_KV_FLOATS stays small.
 *  - runtime/jit/x86_jit.c is replaced by a stub returning NULL, so Q8_0 takes
 *    the portable C path of llm_gemv (llm.c:343-348): the JIT is x86-only
 *    code generation, and the GPU path follows the portable C path.
 */
#define _GNU_SOURCE   /* ucontext register names for the timestamp trap below */
#include "runtime/nn/llm.h"

#undef LLM_MAX_DIM
#define LLM_MAX_DIM 11008
#undef LLM_MAX_FF
#define LLM_MAX_FF 11008
#undef LLM_MAX_SEQ
#define LLM_MAX_SEQ 8192
#undef LLM_KV_FLOATS
#define LLM_KV_FLOATS 1024

static void llm_build_hash_table(const llm_model_t *m);

#include "runtime/nn/llm.c"

#include <stdlib.h>
#include <string.h>

/* ---- exported wrappers around the static operators ---- */

float ref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }
float ref_expf(float x) { return llm_expf(x); }
float ref_sqrtf(float x) { return llm_sqrtf(x); }

float ref_q4_0_dot32(const void *block, const float *x)
{ return q4_0_dot32((const ggml_q4_0_t *)block, x); }

float ref_q8_0_dot32(const void *block, const float *x)
{ return q8_0_dot32((const ggml_q8_0_t *)block, x); }

float ref_vec_dot(const void *w, const float *x, int n, int type)
{ return llm_vec_dot(w, x, n, (ggml_type_t)type); }

void ref_gemv(float *out, const void *w, const float *x, int out_dim, int in_dim, int type)
{ llm_gemv(out, w, x, out_dim, in_dim, (ggml_type_t)type); }

void ref_rmsnorm(float *out, const float *x, const void *w, int dim, int wtype)
{ llm_rmsnorm(out, x, w, dim, (ggml_type_t)wtype); }

void ref_rope(float *vec, int pos, int head_dim, float base)
{ llm_rope(vec, pos, head_dim, base); }

void ref_softmax(float *x, int n) { llm_softmax(x, n); }
void ref_silu(float *x, int n) { llm_silu(x, n); }
float ref_dot_f32(const float *a, const float *b, int n) { return llm_dot_f32(a, b, n); }
void ref_axpy_f32(float *dst, float s, const float *src, int n) { llm_axpy_f32(dst, s, src, n); }
void ref_vadd_f32(float *dst, const float *src, int n) { llm_vadd_f32(dst, src, n); }
void ref_vmul_f32(float *dst, const float *src, int n) { llm_vmul_f32(dst, src, n); }
int ref_argmax(const float *logits, int n) { return llm_argmax(logits, n); }

void ref_embed(float *out, const void *embd, int embd_type, int dim, int token)
{
    llm_model_t *m = (llm_model_t *)calloc(1, sizeof(llm_model_t));
    m->dim = dim;
    m->token_embd = embd;
    m->token_embd_type = (ggml_type_t)embd_type;
    llm_embed(out, m, token);
    free(m);
}

/* ---- whole-model harness: llm_model_t built from flat weight pointers ---- */

typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, ff_dim, vocab_size, max_seq;
    float rope_base;
    int wtype;                  /* ggml type of every projection matrix */
    int embd_type;              /* ggml type of token_embd */
    int out_type;               /* ggml type of output.weight */
    const void *token_embd;
    const void *output_weight;  /* NULL = tied to token_embd */
    const float *output_norm;   /* F32 [dim] */
    /* per layer, n_layers entries each */
    const float *const *attn_norm;
    const float *const *ffn_norm;
    const void *const *wq, *const *wk, *const *wv, *const *wo;
    const void *const *wgate, *const *wup, *const *wdown;
} ref_model_desc_t;

void *ref_model_create(const ref_model_desc_t *d)
{
    if (d->n_layers > LLM_MAX_LAYERS || d->dim > LLM_MAX_DIM ||
        d->ff_dim > LLM_MAX_FF || d->max_seq > LLM_MAX_SEQ)
        return NULL;
    llm_model_t *m = (llm_model_t *)calloc(1, sizeof(llm_model_t));
    m->dim = d->dim;
    m->n_layers = d->n_layers;
    m->n_heads = d->n_heads;
    m->n_kv_heads = d->n_kv_heads;
    m->head_dim = d->dim / d->n_heads;         /* llm.c:1541 */
    m->ff_dim = d->ff_dim;
    m->vocab_size = d->vocab_size;
    m->max_seq = d->max_seq;
    m->rope_base = d->rope_base;
    for (int L = 0; L < d->n_layers; L++) {
        llm_layer_t *ly = &m->layers[L];
        ly->attn_norm = d->attn_norm[L];
        ly->ffn_norm = d->ffn_norm[L];
        ly->attn_norm_type = GGML_TYPE_F32;
        ly->ffn_norm_type = GGML_TYPE_F32;
        ly->q_weight = d->wq[L]; ly->k_weight = d->wk[L];
        ly->v_weight = d->wv[L]; ly->o_weight = d->wo[L];
        ly->ffn_gate = d->wgate[L]; ly->ffn_up = d->wup[L]; ly->ffn_down = d->wdown[L];
        ly->q_type = ly->k_type = ly->v_type = ly->o_type = (ggml_type_t)d->wtype;
        ly->gate_type = ly->up_type = ly->down_type = (ggml_type_t)d->wtype;
    }
    m->token_embd = d->token_embd;
    m->token_embd_type = (ggml_type_t)d->embd_type;
    m->output_norm = d->output_norm;
    m->output_norm_type = GGML_TYPE_F32;
    m->output_weight = d->output_weight;
    m->output_type = (ggml_type_t)d->out_type;
    size_t kv = (size_t)d->n_layers * d->max_seq * d->n_kv_heads * m->head_dim;
    m->k_cache = (float *)calloc(kv, sizeof(float));
    m->v_cache = (float *)calloc(kv, sizeof(float));
    if (!m->k_cache || !m->v_cache) {
        free(m->k_cache); free(m->v_cache); free(m);
        return NULL;
    }
    return m;
}

void ref_model_free(void *p)
{
    llm_model_t *m = (llm_model_t *)p;
    if (!m) return;
    free(m->k_cache);
    free(m->v_cache);
    free(m);
}

void ref_forward_token(void *p, float *logits, int token, int pos)
{ llm_forward_token((llm_model_t *)p, logits, token, pos); }

/* Greedy continuation exactly as llm_generate does it with temperature 0
 * (llm.c:1279-1288, 1290-1347) minus the text-based stop heuristics:
 * prefill token by token, then argmax / forward for n_gen tokens. */
int ref_generate_greedy(void *p, const int *prompt, int n_prompt, int n_gen, int *out)
{
    llm_model_t *m = (llm_model_t *)p;
    float *logits = (float *)malloc(sizeof(float) * (size_t)m->vocab_size);
    if (!logits) return -1;
    int pos = 0;
    for (int i = 0; i < n_prompt; i++)
        llm_forward_token(m, logits, prompt[i], pos++);
    int next = llm_argmax(logits, m->vocab_size);
    int g = 0;
    for (; g < n_gen && pos < m->max_seq; g++) {
        out[g] = next;
        llm_forward_token(m, logits, next, pos++);
        next = llm_argmax(logits, m->vocab_size);
    }
    free(logits);
    return g;
}

/* ---- llm_sample with a chosen timestamp ----
 *
 * llm_sample (llm.c:1177-1246) draws from the CPU timestamp (rdtsc,
 * llm.c:1228-1230).  To pin the whole sampler, the draw included, the
 * harness makes rdtsc trap for the calling thread (prctl PR_SET_TSC,
 * PR_TSC_SIGSEGV), answers the trap with the chosen value in EDX:EAX and
 * steps over the two-byte instruction, then restores both.  The reference
 * code runs unmodified; only its timestamp source is scripted. */
#if defined(__x86_64__) && defined(__linux__)
#include <signal.h>
#include <sys/prctl.h>
#include <ucontext.h>

static volatile uint32_t g_tsc_lo;
static volatile int g_tsc_used;

static void tsc_trap(int sig, siginfo_t *si, void *ctx)
{
    (void)si;
    ucontext_t *uc = (ucontext_t *)ctx;
    const unsigned char *ip = (const unsigned char *)uc->uc_mcontext.gregs[REG_RIP];
    if (ip[0] == 0x0F && ip[1] == 0x31) {   /* rdtsc */
        uc->uc_mcontext.gregs[REG_RAX] = g_tsc_lo;
        uc->uc_mcontext.gregs[REG_RDX] = 0;
        uc->uc_mcontext.gregs[REG_RIP] += 2;
        g_tsc_used++;
        return;
    }
    /* any other fault: restore the default action and let it happen again */
    signal(sig, SIG_DFL);
}

/* llm_sample(logits, n, temperature) with rdtsc returning tsc_lo.  Returns
 * the reference's token, -1 when the timestamp cannot be scripted here (no
 * PR_SET_TSC), or -2 when the reference did not read the timestamp (the
 * greedy limit). */
int ref_sample_at(const float *logits, int n, float temperature, uint32_t tsc_lo)
{
    struct sigaction sa, old;
    memset(&sa, 0, sizeof(sa));
    sa.sa_sigaction = tsc_trap;
    sa.sa_flags = SA_SIGINFO;
    sigemptyset(&sa.sa_mask);
    if (sigaction(SIGSEGV, &sa, &old) != 0) return -1;
    g_tsc_lo = tsc_lo;
    g_tsc_used = 0;
    if (prctl(PR_SET_TSC, PR_TSC_SIGSEGV, 0, 0, 0) != 0) {
        sigaction(SIGSEGV, &old, NULL);
        return -1;
    }
    int tok = llm_sample(logits, n, temperature);
    prctl(PR_SET_TSC, PR_TSC_ENABLE, 0, 0, 0);
    sigaction(SIGSEGV, &old, NULL);
    return g_tsc_used ? tok : (temperature <= 0.001f ? tok : -2);
}
#else
int ref_sample_at(const float *logits, int n, float temperature, uint32_t tsc_lo)
{
    (void)logits; (void)n; (void)temperature; (void)tsc_lo;
    return -1;
}
#endif
