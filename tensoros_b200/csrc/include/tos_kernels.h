/*
 * tos_kernels.h - internal C-callable launchers for the sm_100a kernels.
 *
 * The C11 host runtime (csrc/host) calls only these functions; each
 * enqueues work on the given stream and returns a cudaError_t value (0 = ok).
 * Nothing here allocates device memory except tosk_qmat_alloc.
 */
#ifndef TOS_KERNELS_H
#define TOS_KERNELS_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type_t values, runtime/nn/gguf.h:38-58 */
#define TOSK_F32 0
#define TOSK_F16 1
#define TOSK_Q4_0 2
#define TOSK_Q8_0 8

/* Device-resident quantised matrix in "plane" layout: the per-block fp16
 * scales and the packed quants of the GGUF blocks (llm.c:142-146) are split
 * so that every row's quants are 16-byte aligned for bulk copies. */
typedef struct {
    int type;        /* TOSK_Q4_0 or TOSK_Q8_0 */
    int rows, cols;  /* out_dim, in_dim (cols a multiple of 32) */
    int nb;          /* blocks per row = cols/32 */
    int nbp;         /* scale row stride in halves = nb rounded up to 8 */
    int qb;          /* quant bytes per block: 16 (Q4_0) or 32 (Q8_0) */
    uint8_t *qs;     /* [rows][nb][qb] */
    uint16_t *sc;    /* [rows][nbp] fp16 bit patterns */
    float *rws;      /* [rows] power-of-two row scales of the tensor-core path */
    size_t bytes;    /* device bytes held by qs + sc + rws */
} tosk_qmat_t;

/* ---- weight planes ---- */
/* allocates the planes and clears the scale padding on stream st (the
 * stream of the repack that fills them) */
int tosk_qmat_alloc(tosk_qmat_t *m, int type, int rows, int cols, cudaStream_t st);
void tosk_qmat_free(tosk_qmat_t *m);
/* Repack GGUF blocks already on the device into m (row-concatenation of
 * n_src sources, or row interleave when interleave != 0: dst row
 * n_src*i + s <- source s row i). */
int tosk_qmat_repack(tosk_qmat_t *m, const void *const *src_dev, const int *src_rows,
                     int n_src, int interleave, cudaStream_t st);

/* ---- GEMV epilogues ---- */
enum {
    TOSK_EPI_STORE = 0,   /* out[r] = y */
    TOSK_EPI_RESID = 1,   /* out[r] = resid[r] + y   (llm_vadd_f32) */
    TOSK_EPI_QKV = 2,     /* RoPE q/k rows, q -> out, k/v -> KV cache at *pos */
    TOSK_EPI_SWIGLU = 3   /* rows (2i, 2i+1) = (gate_i, up_i): out[i] = silu(g)*u */
};

typedef struct {
    int kind;
    const float *resid;        /* RESID */
    /* QKV */
    const float2 *rope_cs;     /* [max_seq][hd/2] (cos, sin) */
    const int *pos;            /* device int: current position */
    int hd;                    /* head dim */
    int q_rows;                /* n_heads*hd */
    int kv_rows;               /* n_kv*hd */
    int kv_type;               /* TOSK_F32 or TOSK_F16 */
    void *k_cache;             /* this layer's [max_seq][kv_rows] */
    void *v_cache;
} tosk_epi_t;

typedef struct {
    const float *norm_w;       /* non-NULL: fuse RMSNorm of x (F32 weights) */
    float eps;
} tosk_norm_t;

/* y = W * x.  TOSK_GEMV_EXACT: the reference's per-block lane tree and
 * serial block order (llm.c:148-237), bit for bit.  TOSK_GEMV_FAST: integer
 * dot products on 24-bit fixed-point x and tree row sums (and a tree sum of
 * squares for a fused RMSNorm); normwise error ~1e-7.  x (length cols) is
 * device memory. */
enum { TOSK_GEMV_EXACT = 0, TOSK_GEMV_FAST = 1 };
int tosk_gemv(const tosk_qmat_t *w, const float *x, const tosk_norm_t *norm,
              float *out, const tosk_epi_t *epi, int mode, int *err, int pdl, cudaStream_t st);

/* Y[M][N] = X[M][K] W^T on the tcgen05 tensor cores (fp16 hi/lo split of
 * dequantised weights and scaled activations, fp32 accumulation; ~1e-6
 * normwise vs the fp32 GEMV).  X, Y row-major fp32 device memory; ws of
 * tosk_gemm_ws_bytes(M, N, K) bytes, 256-byte aligned. */
size_t tosk_gemm_ws_bytes(int M, int N, int K);
/* batched prompt pass (prefill.cu): n tokens, row-major [n][...] */
int tosk_pf_embed(float *x, const void *embd, int type, int dim, const int *toks, int n, cudaStream_t st);
int tosk_pf_rope_store(const float *qkv, int q_rows, int kv_rows, int hd, const float2 *cs, int pos0,
                       float *q_out, void *kc, void *vc, int kv_type, int n, cudaStream_t st);
int tosk_pf_attention(const float *q, const void *kc, const void *vc, int kv_type, int n_heads, int n_kv,
                      int hd, int pos0, int n, float *out, cudaStream_t st);
/* batched decode: n tokens of n sequences, token t of sequence slot[t] at
 * position pos[t] (device arrays); slot s's cache at kc/vc + s*cstride elements */
int tosk_bd_rope_store(const float *qkv, int q_rows, int kv_rows, int hd, const float2 *cs, const int *pos,
                       const int *slot, float *q_out, void *kc, void *vc, size_t cstride, int kv_type, int n,
                       cudaStream_t st);
int tosk_bd_attention(const float *q, const void *kc, const void *vc, size_t cstride, int kv_type, int n_heads,
                      int n_kv, int hd, const int *pos, const int *slot, int max_ctx, int n, float *out,
                      cudaStream_t st);
/* m->rws from m->sc (run after the planes are filled) */
int tosk_qmat_row_scales(tosk_qmat_t *m, cudaStream_t st);
int tosk_gemm_q(const tosk_qmat_t *w, const float *x, int M, float *y, void *ws, size_t ws_bytes,
                int *err, int pdl, cudaStream_t st);
/* the same with each row of x RMS-normalised by norm_w first (llm_rmsnorm,
 * llm.c:416-452, tree sum of squares): the norm runs inside the GEMM's
 * activation prep */
int tosk_gemm_q_norm(const tosk_qmat_t *w, const float *x, const float *norm_w, float eps, int M, float *y,
                     void *ws, size_t ws_bytes, int *err, int pdl, cudaStream_t st);
/* res[M][N] += x . W^T (the residual add of llm.c:717-718, 732-733 in the
 * GEMM's epilogue) */
int tosk_gemm_q_residual(const tosk_qmat_t *w, const float *x, int M, float *res, void *ws, size_t ws_bytes,
                         int *err, int pdl, cudaStream_t st);
/* h[M][N/2] = SiLU(g) * u of the normalised GEMM's interleaved gate|up rows
 * (llm.c:723-729) in its epilogue */
int tosk_gemm_q_norm_swiglu(const tosk_qmat_t *w, const float *x, const float *norm_w, float eps, int M,
                            float *h, void *ws, size_t ws_bytes, int *err, int pdl, cudaStream_t st);

/* per-block exact partials: blocks in GGUF layout, n_blocks consecutive,
 * x of length 32*n_blocks, out[n_blocks] (q4_0_dot32 / q8_0_dot32) */
int tosk_block_dots(const void *blocks, int type, const float *x, int n_blocks, float *out,
                    cudaStream_t st);
/* fp32-scale 20-byte Q4 (quantize4.c:122-198) */
int tosk_q4f_gemv(const void *blocks, const float *x, float *out, int rows, int cols,
                  cudaStream_t st);
/* F16/F32 weight rows (llm.c:239-284) */
int tosk_gemv_float(const void *w, int type, const float *x, float *out, int rows, int cols,
                    cudaStream_t st);

/* ---- elementwise / small ops (exact) ---- */
int tosk_rmsnorm(float *out, const float *x, const void *w, int wtype, int dim, float eps,
                 int pdl, cudaStream_t st);
int tosk_rope_table(float2 *cs, int max_seq, int hd, float base, cudaStream_t st);
int tosk_rope(float *vec, int n_vec, const int *pos_dev, int pos, int hd, float base,
              cudaStream_t st);
int tosk_softmax(float *x, int n, cudaStream_t st);
int tosk_silu(float *x, int n, cudaStream_t st);
int tosk_vadd(float *dst, const float *src, int n, cudaStream_t st);
int tosk_vmul(float *dst, const float *src, int n, cudaStream_t st);
int tosk_axpy(float *dst, float s, const float *src, int n, cudaStream_t st);
int tosk_dot(const float *a, const float *b, int n, float *out, cudaStream_t st);
int tosk_embed(float *out, const void *embd, int type, int dim, const int *tok_dev, int tok,
               int pdl, cudaStream_t st);
int tosk_argmax(const float *x, int n, int *out_idx, float *out_val, int pdl, cudaStream_t st);
/* one rank's slice of a row-sharded vector: pair = {value bits, index+offset
 * or -1}; first_rule for the slice that starts the vector (rank 0) */
int tosk_argmax_slice(const float *x, int n, int offset, int first_rule, int *pair, int pdl, cudaStream_t st);
/* llm_sample (llm.c:1177-1246) with the timestamp replaced by `entropy` */
int tosk_sample(const float *x, int n, float temperature, uint32_t entropy, int *out_idx, cudaStream_t st);
/* llm_argmax of each of `rows` consecutive rows of n (batched decode) */
int tosk_argmax_rows(const float *x, int n, int rows, int *out_idx, cudaStream_t st);
/* reduce world pairs (rank order) to the reference's argmax */
int tosk_argmax_pairs(const int *pairs, int world, int *out_idx, int pdl, cudaStream_t st);
/* io[2] -> ring[io[4]]; io[4] += 1; io[1] += 1 (device-side greedy chaining) */
int tosk_decode_advance(int *io, int *ring, int pdl, cudaStream_t st);

/* ---- decode attention ---- */
enum { TOSK_ATTN_EXACT = 0, TOSK_ATTN_FAST = 1 };
size_t tosk_attention_ws_bytes(int n_heads, int max_ctx);
int tosk_attention(float *out, const float *q, const void *k_cache, const void *v_cache,
                   int kv_type, int n_heads, int n_kv, int hd, const int *pos_dev, int pos,
                   int max_ctx, int mode, void *ws, size_t ws_bytes, int *err, int pdl,
                   cudaStream_t st);

int tosk_num_sms(void);

/* ---- tensor-engine operators (tensor_ops.cu; runtime/tensor/tensor_cpu.c) ---- */
int tosk_teng_matmul(float *C, const float *A, const float *B, int M, int N, int K, cudaStream_t st);
int tosk_teng_softmax_rows(float *out, const float *x, int rows, int n, cudaStream_t st);
int tosk_teng_layernorm_rows(float *out, const float *x, const float *gamma, const float *beta, int rows, int n,
                             float eps, cudaStream_t st);
int tosk_teng_elementwise(float *out, const float *a, const float *b, size_t n, int op, cudaStream_t st);
/* S[i][j] = dot(Q_i, K_j) * scale, Q and K [seq][hd] */
int tosk_teng_scores(float *S, const float *Q, const float *K, int seq, int hd, float scale, cudaStream_t st);

/* ---- fp32 transformer engine (tf_engine.cu; runtime/nn/transformer.c) ---- */
/* y = W x, W rows x cols row-major; chunk_order 1: sum += ((p0+p1)+p2)+p3
 * over groups of four, 0: sum += w*x in order */
int tosk_tf_matvec(const float *W, const float *x, float *y, int rows, int cols, int chunk_order, cudaStream_t st);
int tosk_tf_rmsnorm(float *out, const float *x, const float *w, int dim, cudaStream_t st);
int tosk_tf_silu_mul(float *g, const float *u, int n, cudaStream_t st);
int tosk_tf_add(float *x, const float *y, int n, cudaStream_t st);
/* tf_cached_attention for heads [h0, h0+nh) of one layer: head i's q/k/v at
 * q/k/v + i*qstride, output at out + i*ostride; cache [layers][n_heads][max_seq][hd] */
int tosk_tf_attention(float *out, int ostride, const float *q, const float *k, const float *v, int qstride,
                      float *kc, float *vc, int layer, int h0, int nh, int n_heads, int hd, int max_seq,
                      int pos, cudaStream_t st);

/* ---- fused decode step (decode_step.cu): one cooperative kernel per token
 * runs every layer, the LM head and the greedy argmax with FAST arithmetic
 * (tosk_gemv FAST block values, FAST attention) ---- */
typedef struct {
    const uint8_t *qs[4];      /* planes of q|k|v, o, gate|up (interleaved), down */
    const uint16_t *sc[4];
    const float *norm_att, *norm_ffn;
    void *k_cache, *v_cache;   /* this layer's [max_seq][kv_dim] */
} tosk_step_layer_t;

/* most GPUs a fused step is sharded over (one node) */
#define TOSK_MAX_WORLD 8

typedef struct {
    const tosk_step_layer_t *layers;  /* device array [n_layers] */
    int n_layers;
    int wtype;                        /* TOSK_Q4_0 / TOSK_Q8_0: every projection */
    int lm_type;                      /* LM head */
    const uint8_t *lm_qs;
    const uint16_t *lm_sc;
    const float *norm_out;
    const void *embd;
    int embd_type;                    /* TOSK_Q4_0 / TOSK_Q8_0 / TOSK_F16 / TOSK_F32 */
    float *x, *q, *att, *h, *logits;  /* residual [dim], q [q_dim], attention out [q_dim], [ff], [vocab] */
    void *attn_ws;                    /* tosk_attention_ws_bytes(n_heads, max_seq) bytes */
    const float2 *rope;               /* [max_seq][hd/2] */
    int *io;                          /* token, pos, next, err, ring count */
    int *ring;
    int chained;                      /* token from io[2]; then ring[io[4]++] = next, io[1] += 1 */
    unsigned *sync;                   /* tosk_step_sync_bytes(), zero before the first launch */
    int dim, ff, n_heads, n_kv, hd, vocab, max_seq, kv_type;
    float eps;
    /* Row sharding over `world` GPUs of one node (world 1: everything here).
     * n_heads / n_kv / vocab above are this rank's heads and logit rows;
     * dim and ff are the full vector lengths (the projections' columns).
     * This rank computes residual rows [row0, row0 + n_rows), SwiGLU rows
     * [ff0, ff0 + n_ff), attention-output elements [q0, q0 + n_heads*hd) of
     * q_full, and vocabulary rows [vocab0, vocab0 + vocab); x holds the
     * residual rows it computes.  The vectors the ranks exchange (attention
     * output, residual after o, SwiGLU output, residual after down, argmax
     * pairs) travel as 8-byte words {value, epoch}: its epilogues store each
     * produced element into every rank's exchange area (peer_ll[r]: rank r's
     * area as mapped here, [rank] the local one), and the phase that reads a
     * vector waits on the epochs of its words (tosk_step_ll_words long).
     * On one GPU peer_ll[0] may name a local area (the phases then hand
     * their vectors over the same way instead of at grid barriers) or be
     * NULL.  io[5] holds the epoch base (0 on a fresh model). */
    int world, rank;
    int n_rows, n_ff, q_full;
    int q0, row0, ff0, vocab0;
    unsigned long long *peer_ll[TOSK_MAX_WORLD];
} tosk_step_t;

/* 8-byte words of one rank's exchange area for a sharded step */
size_t tosk_step_ll_words(int q_full, int dim, int ff);

size_t tosk_step_sync_bytes(void);
/* 0 when the fused step supports this configuration on this device */
int tosk_step_check(const tosk_step_t *s);
int tosk_step_launch(const tosk_step_t *s, cudaStream_t st);

#ifdef __cplusplus
}
#endif
#endif
