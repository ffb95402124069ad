/*
 * tos_oracle.h - CPU restatement of TensorOS runtime/nn's decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the GPU path is compared
 * against; it is never linked into, loaded by, or called from the product
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg use it.
 *
 * Every function restates the arithmetic of the reference operator named in
 * its comment (file:line inside the TensorOS tree), in the same order of
 * IEEE fp32 operations, so that with gcc -O2 -msse2 -mno-fma
 * -ffp-contract=off it reproduces the reference bit for bit.  Parity of this
 * restatement with the reference itself is pinned by tests that run the
 * reference sources (oracle/_ref) and by the committed golden vectors under
 * tests/golden/.
 */
#ifndef TOS_ORACLE_H
#define TOS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define ORC_TYPE_F32 0
#define ORC_TYPE_F16 1
#define ORC_TYPE_Q4_0 2
#define ORC_TYPE_Q8_0 8

float orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);
float orc_expf(float x);
float orc_sqrtf(float x);

float orc_q4_0_dot32(const void *block, const float *x);
float orc_q8_0_dot32(const void *block, const float *x);
float orc_vec_dot(const void *w, const float *x, int n, int type);
void orc_gemv(float *out, const void *w, const float *x, int out_dim, int in_dim, int type);
void orc_gemv_threads(float *out, const void *w, const float *x, int out_dim, int in_dim,
                      int type, int n_threads);
size_t orc_row_bytes(int in_dim, int type);

void orc_embed(float *out, const void *embd, int type, int dim, int token);
void orc_rmsnorm(float *out, const float *x, const void *w, int wtype, int dim, float eps);
void orc_rope_cs(int pos, int i, int head_dim, float base, float *cos_out, float *sin_out);
void orc_rope(float *vec, int pos, int head_dim, float base);
void orc_rope_rows(float *rows, int n_rows, int row_len, int hd, const int *pos, float base);
void orc_softmax(float *x, int n);
void orc_silu(float *x, int n);
float orc_dot_f32(const float *a, const float *b, int n);
void orc_axpy_f32(float *dst, float s, const float *src, int n);
void orc_vadd_f32(float *dst, const float *src, int n);
void orc_vmul_f32(float *dst, const float *src, int n);
int orc_argmax(const float *x, int n);
int orc_sample(const float *logits, int n, float temperature, uint32_t entropy);

/* Single-query attention over a KV cache laid out [pos][n_kv*hd]
 * (kv_type ORC_TYPE_F32 or ORC_TYPE_F16). */
void orc_attention(float *out, const float *q, const void *k_cache, const void *v_cache,
                   int kv_type, int n_heads, int n_kv, int hd, int pos);

/* quantize4.c's fp32-scale Q4 (20-byte block) */
float orc_q4f_dot_block(const void *block20, const float *x);
void orc_q4f_gemv(float *out, const void *blocks, const float *x, int out_dim, int in_dim);

/* Whole model (llm_forward_token) */
typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, ff_dim, vocab_size, max_seq;
    float rope_base;
    float norm_eps;             /* the reference hard-codes 1e-6f */
    int wtype, embd_type, out_type;
    int kv_type;                /* ORC_TYPE_F32 (reference) or ORC_TYPE_F16 */
    const void *token_embd;
    const void *output_weight;  /* NULL = tied */
    const float *output_norm;
    const float *const *attn_norm;
    const float *const *ffn_norm;
    const void *const *wq, *const *wk, *const *wv, *const *wo;
    const void *const *wgate, *const *wup, *const *wdown;
} orc_model_desc_t;

void *orc_model_create(const orc_model_desc_t *d);
void orc_model_free(void *m);
void orc_forward_token(void *m, float *logits, int token, int pos);
int orc_generate_greedy(void *m, const int *prompt, int n_prompt, int n_gen, int *out);
/* Access to the model's KV cache (for checks): returns base of layer L */
const void *orc_model_kcache(void *m, int layer);
const void *orc_model_vcache(void *m, int layer);
/* The last step's RMS-normalised final hidden state (dim floats): the LM
 * head's input, llm.c:737-742 (for per-element error scales in checks) */
const float *orc_model_hidden(void *m);

#endif
