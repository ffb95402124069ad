/*
 * tensoros_nn_gpu.h - B200 (sm_100a) drop-in for TensorOS runtime/nn's GGUF
 * decode path.
 *
 * Every operator the reference keeps file-static in runtime/nn/llm.c has a
 * host-pointer twin here with the same arguments and the same results (bit
 * for bit): a hosted llm.c links against these names instead of its static
 * functions.  Behind them the work runs on the GPU through hand-written
 * sm_100a kernels; there is no CPU fallback: without a usable GPU every call
 * fails with TOS_ENODEV and the void drop-ins leave their zero-filled result.
 *
 * Ownership: the caller owns every buffer.  Weights passed by host pointer
 * are uploaded and repacked once and cached by (pointer, shape, type), as the
 * reference uses GGUF tensors in place (runtime/nn/gguf.c:301-313); call
 * tos_weight_cache_clear() after changing such memory.  Device-pointer
 * variants (*_dev) are asynchronous on the given CUDA stream (NULL = the
 * library's stream) and never synchronise.
 *
 * Errors: functions returning int return a tos_status_t.  The void / float
 * drop-ins mirror the reference's void signatures; their status is kept in a
 * thread-local slot read by tos_last_status().  As in the reference
 * (llm.c:285-287, 359-360, 406-408), an unsupported ggml type yields zeros.
 *
 * Threading: calls are serialised per library instance on one stream; a model
 * (tos_model_t) must be used by one host thread at a time.
 */
#ifndef TENSOROS_NN_GPU_H
#define TENSOROS_NN_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
typedef enum {
    TOS_OK = 0,
    TOS_EINVAL = -1,    /* bad argument (shape, type, pointer) */
    TOS_ENOMEM = -2,    /* device or host allocation failed */
    TOS_ECUDA = -3,     /* CUDA runtime error */
    TOS_ENCCL = -4,     /* collective error */
    TOS_ETIMEOUT = -5,  /* a bounded device-side wait ran out */
    TOS_ENOTSUP = -6,   /* valid but unsupported configuration */
    TOS_ENODEV = -7     /* no usable CUDA device */
} tos_status_t;

/* ggml_type_t numeric values, verbatim from runtime/nn/gguf.h:38-58 */
enum {
    TOS_TYPE_F32 = 0,
    TOS_TYPE_F16 = 1,
    TOS_TYPE_Q4_0 = 2,
    TOS_TYPE_Q8_0 = 8
};

/* attention numerics */
enum {
    TOS_ATTN_EXACT = 0, /* reference order, bit-identical */
    TOS_ATTN_FAST = 1   /* split-position partial sums; max rel. error 1e-4 */
};

/* GEMV arithmetic (with the RMSNorm fused into it) */
enum {
    TOS_GEMV_EXACT = 0, /* reference lane tree and serial row chain, bit-identical */
    TOS_GEMV_FAST = 1   /* integer dot products on 24-bit fixed-point x, tree sums;
                           normwise error ~1e-7, bound 1e-4 */
};

const char *tos_status_string(int status);
int tos_last_status(void);

/* ------------------------------------------------------------ library */
/* Select the device and create the library stream (idempotent). */
int tos_init(int device);
int tos_shutdown(void);
int tos_device_count(void);
int tos_synchronize(void);
/* The library's CUDA stream (cudaStream_t as void*). */
void *tos_stream(void);

/* ------------------------------------------------- registered weights */
/* A quantised matrix [out_dim][in_dim/32 blocks] (Q4_0 or Q8_0) held on the
 * device in plane layout.  Replaces the zero-copy GGUF pointer of llm.c. */
typedef struct tos_weight tos_weight_t;
int tos_weight_create(tos_weight_t **w, const void *host_blocks, int out_dim, int in_dim, int type);
int tos_weight_create_dev(tos_weight_t **w, const void *dev_blocks, int out_dim, int in_dim,
                          int type, void *stream);
void tos_weight_destroy(tos_weight_t *w);
size_t tos_weight_device_bytes(const tos_weight_t *w);
void tos_weight_cache_clear(void);

/* ---------------------------------------- device-pointer operators */
/* out = W x  (llm_gemv, llm.c:329-349), x/out device pointers */
int tos_gemv_dev(const tos_weight_t *w, const float *x, float *out, void *stream);
/* out = W rmsnorm(x, norm_w, eps): fused llm_rmsnorm + llm_gemv */
int tos_gemv_norm_dev(const tos_weight_t *w, const float *x, const float *norm_w, float eps,
                      float *out, void *stream);
/* either of the two above (norm_w NULL: no norm) in TOS_GEMV_EXACT or
 * TOS_GEMV_FAST arithmetic; the EXACT form is tos_gemv_dev/tos_gemv_norm_dev */
int tos_gemv_mode_dev(const tos_weight_t *w, const float *x, const float *norm_w, float eps,
                      float *out, int mode, void *stream);
/* Batched GEMM for prefill and batched decode: y[m][out_dim] = x[m][in_dim]
 * W^T for m rows of activations (row-major, device memory), i.e. m calls of
 * llm_gemv (llm.c:329-349) at once.  No counterpart in the reference (which
 * runs tokens one by one).  Runs on the tcgen05 tensor cores with an exact
 * fp16 hi/lo split of the dequantised weights and a 22-bit split of the
 * activations, fp32 accumulation; Q4_0 at m <= 16 with in_dim a multiple of
 * 128 instead as exact integer block products (the FAST GEMV's 22-bit
 * fixed-point activations, 8-bit tensor-core MMAs) scaled and summed in
 * fp32.  Normwise error ~1e-6 against the fp32 GEMV either way.  in_dim a
 * multiple of 64; ws: tos_gemm_workspace_bytes bytes,
 * 256-byte aligned.  tos_gemm_workspace_bytes(m, ...) covers every call with
 * at most m rows, so one workspace sized for the longest batch serves the
 * shorter ones.  Results are bit-identical run to run. */
size_t tos_gemm_workspace_bytes(int m, int out_dim, int in_dim);
int tos_gemm_dev(const tos_weight_t *w, const float *x, int m, float *y, void *ws, size_t ws_bytes,
                 void *stream);
/* per-block values q4_0_dot32 / q8_0_dot32 (llm.c:148-216) for n_blocks
 * consecutive GGUF blocks against x[32*n_blocks] */
int tos_block_dots_dev(const void *blocks, int type, const float *x, int n_blocks, float *out,
                       void *stream);
int tos_rmsnorm_dev(float *out, const float *x, const void *w, int wtype, int dim, float eps,
                    void *stream);
int tos_rope_dev(float *vec, int n_vec, int pos, int head_dim, float base, void *stream);
int tos_softmax_dev(float *x, int n, void *stream);
int tos_silu_dev(float *x, int n, void *stream);
int tos_vadd_dev(float *dst, const float *src, int n, void *stream);
int tos_vmul_dev(float *dst, const float *src, int n, void *stream);
int tos_axpy_dev(float *dst, float s, const float *src, int n, void *stream);
int tos_dot_dev(const float *a, const float *b, int n, float *out, void *stream);
int tos_embed_dev(float *out, const void *embd, int type, int dim, int token, void *stream);
int tos_argmax_dev(const float *x, int n, int *out_index, void *stream);
/* llm_sample (llm.c:1177-1246) on device logits; see tos_sample */
int tos_sample_dev(const float *logits, int n, float temperature, uint32_t entropy, int *out_index,
                   void *stream);
/* The distributed argmax of a row-sharded model, on one device: x is cut into
 * `world` equal slices, each slice gives a (value, index) pair and the pairs
 * reduce with llm_argmax's rule (llm.c:1129-1140); same kernels as a sharded
 * model's last step.  No counterpart in the reference. */
int tos_argmax_sharded_dev(const float *x, int n, int world, int *out_index, void *stream);

/* Single-query attention over a KV cache [ctx][n_kv*head_dim] (kv_type F32 or
 * F16) for query heads q[n_heads*head_dim] at position pos (attends t<=pos),
 * llm.c:683-714.  workspace: tos_attention_workspace_bytes(n_heads, max_ctx)
 * bytes of device memory. */
size_t tos_attention_workspace_bytes(int n_heads, int max_ctx);
int tos_attention_dev(float *out, const float *q, const void *k_cache, const void *v_cache,
                      int kv_type, int n_heads, int n_kv, int head_dim, int pos, int max_ctx,
                      int mode, void *workspace, size_t workspace_bytes, void *stream);

/* Allocation-free variant of tos_attention_dev (this entry point has no
 * counterpart in the reference).  For callers that cannot allocate device
 * memory while they run a step, as the reference's own static-scratch decode
 * loop never does: the workspace is a 4 MiB device array inside the library
 * (held on every GPU that loads it until exit) instead of caller memory.
 * Returns TOS_ENOMEM, queueing nothing, when
 * tos_attention_workspace_bytes(n_heads, max_ctx) exceeds 4 MiB.  The first
 * call on a device resolves the array's address (make it before any stream
 * capture).  All calls share the array: calls that overlap on the GPU race
 * and must be serialised by the caller.  Nothing needs to start at zero.
 * A cudaDeviceReset invalidates the resolved address along with every other
 * device object of the library: call tos_shutdown before a reset.
 * stream: the caller's CUDA stream (NULL = the legacy default stream). */
int tos_attention_noalloc_dev(float *out, const float *q, const void *k_cache, const void *v_cache,
                              int kv_type, int n_heads, int n_kv, int head_dim, int pos, int max_ctx,
                              int mode, void *stream);

/* --------------------- host-pointer drop-ins for runtime/nn/llm.c statics */
void tos_gemv(float *out, const void *weight, const float *x, int out_dim, int in_dim, int type); /* llm.c:329 */
float tos_vec_dot(const void *weight, const float *x, int n, int type);                           /* llm.c:221 */
float tos_q4_0_dot32(const void *block, const float *x);                                          /* llm.c:148 */
float tos_q8_0_dot32(const void *block, const float *x);                                          /* llm.c:187 */
void tos_embed(float *out, const void *embd, int type, int dim, int token);                       /* llm.c:365 */
void tos_rmsnorm(float *out, const float *x, const void *w, int dim, int wtype);                  /* llm.c:416 */
void tos_rope(float *vec, int pos, int head_dim, float base);                                     /* llm.c:460 */
void tos_softmax(float *x, int n);                                                                /* llm.c:506 */
void tos_silu(float *x, int n);                                                                   /* llm.c:538 */
float tos_dot_f32(const float *a, const float *b, int n);                                         /* llm.c:551 */
void tos_axpy_f32(float *dst, float scale, const float *src, int n);                              /* llm.c:580 */
void tos_vadd_f32(float *dst, const float *src, int n);                                           /* llm.c:599 */
void tos_vmul_f32(float *dst, const float *src, int n);                                           /* llm.c:617 */
int tos_argmax(const float *logits, int n);                                                       /* llm.c:1129 */
/* llm_sample (llm.c:1177-1246): top-40, temperature, nucleus 0.9, one draw.
 * The reference draws from the CPU timestamp; here the caller passes the
 * 32-bit word (mixed and reduced to r in [0,1) exactly as the reference
 * mixes its timestamp).  temperature <= 0.001: llm_argmax.  Finite logits. */
int tos_sample(const float *logits, int n, float temperature, uint32_t entropy);
/* quantize4.h:64-67: fp32-scale 20-byte Q4 blocks */
float tos_q4_dot_block(const void *block20, const float *x);
void tos_q4_gemv(float *out, const void *blocks20, const float *x, int out_dim, int in_dim);

/* ------------------------------------------------------------- model */
/* Mirrors llm_model_t (llm.h:44-115): architecture parameters and the GGUF
 * tensor pointers (host memory, GGUF block layout).  Layer arrays hold
 * n_layers pointers each.  Norm weights are F32 [dim]. */
typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, ff_dim, vocab_size, max_seq;
    float rope_base;
    float norm_eps;          /* the reference hard-codes 1e-6f (llm.c:431) */
    int kv_type;             /* TOS_TYPE_F32 (reference) or TOS_TYPE_F16 */
    int attn_mode;           /* TOS_ATTN_EXACT or TOS_ATTN_FAST */
    int wtype;               /* type of every projection matrix: Q4_0 / Q8_0 */
    int embd_type;           /* token_embd type: Q4_0 / Q8_0 / F16 / F32 */
    int out_type;            /* output.weight type (Q4_0 / Q8_0) */
    const void *token_embd;
    const void *output_weight;   /* NULL: tied to token_embd (llm.c:740-742) */
    const float *output_norm;
    const float *const *attn_norm;
    const float *const *ffn_norm;
    const void *const *wq;
    const void *const *wk;
    const void *const *wv;
    const void *const *wo;
    const void *const *wgate;
    const void *const *wup;
    const void *const *wdown;
    int gemv_mode;           /* TOS_GEMV_EXACT (default) or TOS_GEMV_FAST */
    int fused_step;          /* 1: with FAST arithmetic on one GPU each token runs as one fused
                                persistent kernel; 0 (default): one kernel per operator */
} tos_model_desc_t;

typedef struct tos_model tos_model_t;

int tos_model_create(tos_model_t **m, const tos_model_desc_t *desc);
void tos_model_destroy(tos_model_t *m);
/* llm_reset_cache (llm.c:2042-2053): zero the KV cache */
int tos_model_reset(tos_model_t *m);
/* llm_forward_token (llm.c:641-743): logits (host, vocab_size floats) may be
 * NULL to skip the copy-out. */
int tos_model_forward_token(tos_model_t *m, float *logits, int token, int pos);
/* forward + llm_argmax on the device; *next receives the greedy token */
int tos_model_forward_argmax(tos_model_t *m, int token, int pos, int *next);
/* llm_generate with temperature 0 and no text stops (llm.c:1279-1347):
 * prefill the prompt token by token, then n_gen greedy tokens into out.
 * Returns the number generated or a negative status. */
int tos_model_generate_greedy(tos_model_t *m, const int *prompt, int n_prompt, int n_gen, int *out);
/* Greedy decode of n_steps tokens kept on the device: step i consumes the
 * previous token (token for i = 0) at position pos+i and its argmax becomes
 * out_tokens[i] (host, copied once at the end).  Same tokens as n_steps
 * calls of tos_model_forward_argmax, without a host round trip per step. */
int tos_model_decode(tos_model_t *m, int token, int pos, int n_steps, int *out_tokens);
/* Batched prompt pass (no counterpart in the reference, which runs the
 * prompt token by token, llm.c:1279-1281): tokens[0..n) at positions
 * pos0.. go through every layer together, the projections as tensor-core
 * GEMMs (tos_gemm_dev numerics) and attention causal per token; the KV cache
 * is filled for those positions.  logits (may be NULL) and *next (may be
 * NULL) get the last token's logits and greedy next token.  Needs dim and
 * ff_dim multiples of 64; not for sharded models (TOS_ENOTSUP). */
int tos_model_prefill(tos_model_t *m, const int *tokens, int n, int pos0, float *logits, int *next);
/* Batched decode (no counterpart in the reference, which decodes one
 * sequence): one greedy step of n <= 16 independent sequences: token[i] at
 * position pos[i] of the sequence held in KV-cache slot slot[i] (distinct
 * slots in [0, 16); the caches are allocated on first use and zeroed by
 * tos_model_reset).  The projections run as tensor-core GEMMs over the n
 * tokens (tos_gemm_dev numerics, FAST attention).  logits (n x vocab_size,
 * may be NULL) and next[n] are host buffers.  Needs dim and ff_dim
 * multiples of 64; one GPU (TOS_ENOTSUP). */
int tos_model_decode_batch(tos_model_t *m, const int *slot, const int *tokens, const int *pos, int n,
                           float *logits, int *next);
/* the model's CUDA stream (cudaStream_t as void*) */
void *tos_model_stream(const tos_model_t *m);
/* device pointer of the last logits (vocab_size floats) */
const float *tos_model_logits_dev(const tos_model_t *m);
size_t tos_model_device_bytes(const tos_model_t *m);
/* 1 when each token runs as the one fused kernel (see fused_step) */
int tos_model_fused(const tos_model_t *m);

/* ---------------------------------------------- fp32 transformer engine
 * The reference's other decoder, runtime/nn/transformer.c (fp32 weights,
 * KV cache [layer][head][seq][head_dim], eps 1e-5, the activations of
 * runtime/tensor/tensor_cpu.c), on the GPU with its results bit for bit. */
void tos_tf_rmsnorm(float *out, const float *x, const float *w, int dim);                   /* transformer.c:92 */
void tos_tf_swiglu_ffn(float *out, const float *x, const float *w1, const float *w2,
                       const float *w3, int dim, int ff_dim);                             /* transformer.c:121 */
/* Mirrors tf_model_t / tf_block_weights_t (transformer.h): host fp32 arrays,
 * per-layer pointer arrays of num_layers entries; wq/wk/wv/wo [dim][dim],
 * w1/w3 [ff_dim][dim], w2 [dim][ff_dim], tok_embed [vocab_size][dim]. */
typedef struct {
    int dim, num_heads, ff_dim, num_layers, vocab_size, max_seq;
    const float *const *wq, *const *wk, *const *wv, *const *wo;
    const float *const *w1, *const *w2, *const *w3;
    const float *const *rms_att, *const *rms_ffn;
    const float *tok_embed, *rms_final;
} tos_tf_desc_t;
typedef struct tos_tf_model tos_tf_model_t;
int tos_tf_model_create(tos_tf_model_t **m, const tos_tf_desc_t *desc);           /* kv_cache_init, transformer.c:46 */
void tos_tf_model_destroy(tos_tf_model_t *m);
int tos_tf_reset(tos_tf_model_t *m);                                               /* kv_cache_reset, transformer.c:67 */
int tos_tf_cached_attention(tos_tf_model_t *m, float *out, const float *q, const float *k, const float *v,
                            int layer, int head, int pos);                         /* transformer.c:193 */
int tos_tf_forward_token(tos_tf_model_t *m, float *logits, const float *tok_embed, int pos); /* transformer.c:255 */

/* ------------------------------------- GPU dispatch of the tensor engine
 * The reference's intended GPU entry points (kernel/drivers/gpu/gpu.h:80-96,
 * stubs in gpu.c:155-225 that compute nothing) and the engine's routing
 * rule (runtime/tensor/tensor_engine.c:28-67), backed here by kernels that
 * give the engine's CPU operators' results bit for bit
 * (runtime/tensor/tensor_cpu.c: tensor_cpu_matmul, _softmax, _layernorm,
 * element-wise ops, tensor_cpu_attention).  Tensors are F32, contiguous
 * row-major; data_virt is host memory when device_id is 0 and device memory
 * of the library's GPU otherwise.  Each returns 0, or -1 for what the
 * reference rejects (a gpu_id it has no GPU for, mismatched shapes) and for
 * what is not supported here; tos_last_status() gives the reason. */
typedef struct {                 /* tensor_desc_t, kernel/core/kernel.h:30-40 */
    uint32_t ndim;
    uint64_t shape[8];
    uint64_t strides[8];         /* bytes (not read: contiguous tensors only) */
    int32_t dtype;               /* TENSOR_DTYPE_*: 0 = F32 */
    uint64_t data_phys;
    uint64_t data_virt;
    uint64_t size_bytes;
    uint32_t device_id;          /* 0 = host memory, 1+ = this GPU */
    uint32_t flags;
} tos_tensor_desc_t;

/* tir_opcode_t values the routing rule looks at (runtime/pseudocode/pseudocode_jit.h:186-217) */
enum {
    TOS_TIR_MATMUL = 4, TOS_TIR_CONV2D = 5, TOS_TIR_ATTENTION = 6, TOS_TIR_SOFTMAX = 7,
    TOS_TIR_LAYERNORM = 8, TOS_TIR_RELU = 9, TOS_TIR_GELU = 10, TOS_TIR_ADD = 12, TOS_TIR_MUL = 13,
    TOS_TIR_EMBEDDING = 23
};
enum { TOS_BACKEND_CPU = 0, TOS_BACKEND_GPU = 1 };   /* engine_backend_t, tensor_engine.h:23-28 */

/* select_backend (tensor_engine.c:28-67): which backend the engine sends an
 * operation to, given the tensors' sizes and how many GPUs it has */
int tos_tensor_select_backend(int op, const tos_tensor_desc_t *tensors, uint32_t count, uint32_t gpu_count);
/* C[M][N] = A[M][K] B[K][N]; sets C's ndim, shape, dtype, size_bytes as
 * tensor_matmul does (tensor_engine.c:83-88) */
int tos_gpu_tensor_matmul(uint32_t gpu_id, tos_tensor_desc_t *C, const tos_tensor_desc_t *A,
                          const tos_tensor_desc_t *B);                                          /* gpu.c:155 */
/* out[seq][d] = softmax(Q K^T * scale) V for Q, K, V [seq][d] (no mask), as
 * tensor_cpu_attention (which uses scale 1/sqrt(d): pass scale <= 0) */
int tos_gpu_tensor_attention(uint32_t gpu_id, tos_tensor_desc_t *output, const tos_tensor_desc_t *Q,
                             const tos_tensor_desc_t *K, const tos_tensor_desc_t *V, float scale); /* gpu.c:178 */
/* softmax along the last axis (axis = ndim-1 or -1), tensor_cpu_softmax per row */
int tos_gpu_tensor_softmax(uint32_t gpu_id, tos_tensor_desc_t *output, const tos_tensor_desc_t *input,
                           int axis);                                                           /* gpu.c:195 */
/* layer norm along the last axis (tensor_cpu_layernorm per row), then
 * * gamma + beta per element when those are given (data_virt != 0) */
int tos_gpu_tensor_layernorm(uint32_t gpu_id, tos_tensor_desc_t *output, const tos_tensor_desc_t *input,
                             const tos_tensor_desc_t *gamma, const tos_tensor_desc_t *beta,
                             float epsilon);                                                   /* gpu.c:202 */
/* output = a op b, op 0 add, 1 mul, 2 sub, 3 div (gpu.h:94) */
int tos_gpu_tensor_elementwise(uint32_t gpu_id, tos_tensor_desc_t *output, const tos_tensor_desc_t *a,
                               const tos_tensor_desc_t *b, int op);                            /* gpu.c:211 */

/* ------------------------------------------------------------ GGUF files
 * The container of runtime/nn (gguf.c:204-423): v2/v3 headers, metadata,
 * tensor infos; tensor data is used in place (the caller's buffer, or a
 * read-only mapping of the file).  tos_gguf_model_desc maps a llama-family
 * file onto tos_model_desc_t (llm.c:1374-1448, 1521-1545): architecture
 * from "<general.architecture>.*" keys, tensors blk.N.attn_q.weight etc.,
 * output.weight tied to token_embd when absent; max_seq = the file's
 * context length, kv_type F16, EXACT arithmetic (the caller may change
 * them).  The descriptor's pointers stay valid until tos_gguf_close. */
typedef struct tos_gguf tos_gguf_t;
int tos_gguf_open(tos_gguf_t **g, const void *data, uint64_t size);
int tos_gguf_open_file(tos_gguf_t **g, const char *path);
void tos_gguf_close(tos_gguf_t *g);
uint32_t tos_gguf_version(const tos_gguf_t *g);
int64_t tos_gguf_n_tensors(const tos_gguf_t *g);
int64_t tos_gguf_n_kv(const tos_gguf_t *g);
int64_t tos_gguf_find_tensor(const tos_gguf_t *g, const char *name);   /* index or -1 */
/* dims[d] = ne[d] (fastest first; 1 beyond n_dims); bytes 0 for a type
 * whose block size is unknown */
int tos_gguf_tensor_info(const tos_gguf_t *g, int64_t i, const char **name, int *type, int *n_dims,
                         uint64_t dims[4], const void **data, uint64_t *bytes);
int tos_gguf_get_u32(const tos_gguf_t *g, const char *key, uint32_t *out);   /* any integer type */
int tos_gguf_get_f32(const tos_gguf_t *g, const char *key, float *out);
int tos_gguf_get_str(const tos_gguf_t *g, const char *key, const char **str, uint64_t *len);
int tos_gguf_model_desc(tos_gguf_t *g, tos_model_desc_t *desc);

/* ------------------------------------------ multi-GPU (one node, NCCL)
 * No counterpart in the reference (a single-CPU decoder).  A model is
 * row-sharded over `world` ranks, one process and one GPU per rank: rank r
 * keeps heads, residual rows, FFN rows and vocabulary rows
 * [r*n/world, (r+1)*n/world) of each projection and its heads' KV cache;
 * the slices produced by each GEMV are all-gathered, and the greedy token is
 * a distributed argmax.  Rows are computed exactly as on one GPU, so every
 * rank's logits and tokens equal the one-GPU model's (bit-identical in EXACT
 * mode).  Every rank passes the full host weights (the GGUF tensors of the
 * one-GPU descriptor) and uploads only its rows. */
typedef struct {
    int world, rank;
    int head0, n_heads;            /* query heads */
    int kv_head0, n_kv_heads;      /* key/value heads (and KV cache) */
    int q_row0, n_q_rows;          /* rows of wq = heads * head_dim */
    int kv_row0, n_kv_rows;        /* rows of wk / wv */
    int row0, n_rows;              /* rows of wo and wdown (residual stream) */
    int ff0, n_ff;                 /* rows of wgate / wup */
    int vocab0, n_vocab;           /* LM-head rows */
} tos_shard_plan_t;

/* [begin, begin+count) of `total` for `rank`: equal slices of whole `unit`s;
 * TOS_ENOTSUP when total is not a multiple of unit*world */
int tos_shard_range(int total, int unit, int world, int rank, int *begin, int *count);
/* the rows rank `rank` of `world` keeps (heads whole, other slices in
 * multiples of 32 rows) */
int tos_shard_plan(const tos_model_desc_t *desc, int world, int rank, tos_shard_plan_t *plan);
/* NCCL unique id (NCCL_UNIQUE_ID_BYTES = 128) for tos_model_create_sharded:
 * made by one rank and handed to all (NCCL is loaded at run time) */
int tos_nccl_unique_id(void *id, size_t bytes);
/* Collective: every rank calls it with the same descriptor and id, on its
 * own current device (tos_init(local_gpu) first).  world == 1 is
 * tos_model_create. */
int tos_model_create_sharded(tos_model_t **m, const tos_model_desc_t *desc, int rank, int world,
                             const void *nccl_id);

#ifdef __cplusplus
}
#endif
#endif
