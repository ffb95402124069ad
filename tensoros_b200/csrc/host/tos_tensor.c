/*
 * tos_tensor.c - the reference's GPU dispatch point for its tensor engine
 * (kernel/drivers/gpu/gpu.c:155-225, gpu.h:80-96) and the engine's routing
 * rule (runtime/tensor/tensor_engine.c:28-67), backed by tensor_ops.cu.
 *
 * The reference's gpu_tensor_* are stubs that validate and return 0 without
 * computing; the operations they stand for are the engine's CPU operators
 * (runtime/tensor/tensor_cpu.c), whose results these give bit for bit.
 * Tensors whose device_id is 0 live in host memory and travel through the
 * library's scratch; others are device memory used in place.
 */
#include <stdlib.h>
#include <string.h>

#include "tos_internal.h"

/* tensor_engine.c:28-67, restated: no GPU -> CPU; under 4 KiB in all -> CPU;
 * matmul / conv2d / attention / softmax / embedding -> GPU; add, mul, relu,
 * gelu -> GPU above 64 KiB; layernorm -> GPU above 32 KiB; else CPU. */
int tos_tensor_select_backend(int op, const tos_tensor_desc_t *t, uint32_t count, uint32_t gpu_count)
{
    if (gpu_count == 0) return TOS_BACKEND_CPU;
    uint64_t total = 0;
    for (uint32_t i = 0; t && i < count; i++) total += t[i].size_bytes;
    if (total < 4096) return TOS_BACKEND_CPU;
    switch (op) {
    case TOS_TIR_MATMUL:
    case TOS_TIR_CONV2D:
    case TOS_TIR_ATTENTION:
    case TOS_TIR_SOFTMAX:
    case TOS_TIR_EMBEDDING:
        return TOS_BACKEND_GPU;
    case TOS_TIR_ADD:
    case TOS_TIR_MUL:
    case TOS_TIR_RELU:
    case TOS_TIR_GELU:
        return total > 65536 ? TOS_BACKEND_GPU : TOS_BACKEND_CPU;
    case TOS_TIR_LAYERNORM:
        return total > 32768 ? TOS_BACKEND_GPU : TOS_BACKEND_CPU;
    default:
        return TOS_BACKEND_CPU;
    }
}

/* ---- operand staging ---- */

typedef struct {
    const tos_tensor_desc_t *d;
    size_t n;          /* floats */
    float *dev;        /* where the kernel reads / writes it */
    int host;          /* staged through scratch */
} operand_t;

static size_t elems(const tos_tensor_desc_t *d)
{
    if (!d || d->ndim == 0 || d->ndim > 8) return 0;
    size_t n = 1;
    for (uint32_t i = 0; i < d->ndim; i++) {
        if (d->shape[i] == 0 || n > ((size_t)1 << 40) / d->shape[i]) return 0;
        n *= (size_t)d->shape[i];
    }
    return n;
}

static int f32_operand(const tos_tensor_desc_t *d)
{
    return d && d->dtype == 0 && d->data_virt && elems(d) > 0;
}

/* Places every operand: device tensors in place, host tensors in the library
 * scratch (inputs copied in); returns a cudaError_t / tos status value. */
static int stage(operand_t *ops, int n_ops, int n_inputs, cudaStream_t st)
{
    size_t off = 0;
    for (int i = 0; i < n_ops; i++)
        if (ops[i].d && ops[i].d->device_id == 0) off += (ops[i].n * 4 + 255) & ~(size_t)255;
    if (off && !tos_scratch(off)) return TOS_ENOMEM;
    off = 0;
    for (int i = 0; i < n_ops; i++) {
        if (!ops[i].d) continue;
        if (ops[i].d->device_id == 0) {
            ops[i].dev = (float *)((char *)tos_g.scratch + off);
            ops[i].host = 1;
            off += (ops[i].n * 4 + 255) & ~(size_t)255;
            if (i < n_inputs) {
                int e = cudaMemcpyAsync(ops[i].dev, (const void *)(uintptr_t)ops[i].d->data_virt, ops[i].n * 4,
                                        cudaMemcpyHostToDevice, st);
                if (e) return e;
            }
        } else {
            ops[i].dev = (float *)(uintptr_t)ops[i].d->data_virt;
        }
    }
    return 0;
}

/* Copies the output back when it is host memory and waits. */
static int finish_out(const operand_t *out, cudaStream_t st)
{
    int e = 0;
    if (out->host)
        e = cudaMemcpyAsync((void *)(uintptr_t)out->d->data_virt, out->dev, out->n * 4, cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaStreamSynchronize(st);
    return e;
}

static int ret(int st) { return tos_set_status(st) == TOS_OK ? 0 : -1; }

static int gpu_ok(uint32_t gpu_id)
{
    /* one library instance drives one GPU: id 0 is it (gpu.c:160 rejects
     * ids beyond the GPUs found) */
    if (tos_ensure_init()) return TOS_ENODEV;
    return gpu_id == 0 ? TOS_OK : TOS_EINVAL;
}

int tos_gpu_tensor_matmul(uint32_t gpu_id, tos_tensor_desc_t *C, const tos_tensor_desc_t *A,
                          const tos_tensor_desc_t *B)
{
    int rc = gpu_ok(gpu_id);
    if (rc) return ret(rc);
    if (!C || !A || !B || A->ndim < 2 || B->ndim < 2) return ret(TOS_EINVAL);
    if (A->shape[A->ndim - 1] != B->shape[B->ndim - 2]) return ret(TOS_EINVAL);   /* gpu.c:161-162 */
    if (A->ndim != 2 || B->ndim != 2 || !f32_operand(A) || !f32_operand(B) || !C->data_virt) return ret(TOS_ENOTSUP);
    const uint64_t M = A->shape[0], K = A->shape[1], N = B->shape[1];
    if (M > (1u << 30) || N > (1u << 30) || K > (1u << 30)) return ret(TOS_ENOTSUP);
    /* tensor_engine.c:83-88: the output's shape */
    C->ndim = 2;
    C->shape[0] = M;
    C->shape[1] = N;
    C->dtype = A->dtype;
    C->size_bytes = M * N * sizeof(float);
    operand_t o[3] = {{A, (size_t)(M * K), NULL, 0}, {B, (size_t)(K * N), NULL, 0}, {C, (size_t)(M * N), NULL, 0}};
    cudaStream_t st = tos_g.stream;
    int e = stage(o, 3, 2, st);
    if (!e) e = tosk_teng_matmul(o[2].dev, o[0].dev, o[1].dev, (int)M, (int)N, (int)K, st);
    if (!e) e = finish_out(&o[2], st);
    return ret(tos_from_cuda(e));
}

int tos_gpu_tensor_softmax(uint32_t gpu_id, tos_tensor_desc_t *out, const tos_tensor_desc_t *in, int axis)
{
    int rc = gpu_ok(gpu_id);
    if (rc) return ret(rc);
    if (!out || !f32_operand(in) || !out->data_virt) return ret(TOS_EINVAL);
    if (axis != -1 && axis != (int)in->ndim - 1) return ret(TOS_ENOTSUP);   /* rows only */
    const size_t n = (size_t)in->shape[in->ndim - 1], total = elems(in);
    if (n > (1u << 30) || total / n > (1u << 30)) return ret(TOS_ENOTSUP);
    operand_t o[2] = {{in, total, NULL, 0}, {out, total, NULL, 0}};
    cudaStream_t st = tos_g.stream;
    int e = stage(o, 2, 1, st);
    if (!e) e = tosk_teng_softmax_rows(o[1].dev, o[0].dev, (int)(total / n), (int)n, st);
    if (!e) e = finish_out(&o[1], st);
    return ret(tos_from_cuda(e));
}

int tos_gpu_tensor_layernorm(uint32_t gpu_id, tos_tensor_desc_t *out, const tos_tensor_desc_t *in,
                             const tos_tensor_desc_t *gamma, const tos_tensor_desc_t *beta, float eps)
{
    int rc = gpu_ok(gpu_id);
    if (rc) return ret(rc);
    if (!out || !f32_operand(in) || !out->data_virt) return ret(TOS_EINVAL);
    const size_t n = (size_t)in->shape[in->ndim - 1], total = elems(in);
    if (n > (1u << 30) || total / n > (1u << 30)) return ret(TOS_ENOTSUP);
    const tos_tensor_desc_t *g = gamma && gamma->data_virt ? gamma : NULL;
    const tos_tensor_desc_t *b = beta && beta->data_virt ? beta : NULL;
    if ((g && (!f32_operand(g) || elems(g) != n)) || (b && (!f32_operand(b) || elems(b) != n))) return ret(TOS_EINVAL);
    operand_t o[4] = {{in, total, NULL, 0}, {g, n, NULL, 0}, {b, n, NULL, 0}, {out, total, NULL, 0}};
    cudaStream_t st = tos_g.stream;
    int e = stage(o, 4, 3, st);
    if (!e) e = tosk_teng_layernorm_rows(o[3].dev, o[0].dev, g ? o[1].dev : NULL, b ? o[2].dev : NULL,
                                         (int)(total / n), (int)n, eps, st);
    if (!e) e = finish_out(&o[3], st);
    return ret(tos_from_cuda(e));
}

int tos_gpu_tensor_elementwise(uint32_t gpu_id, tos_tensor_desc_t *out, const tos_tensor_desc_t *a,
                               const tos_tensor_desc_t *b, int op)
{
    int rc = gpu_ok(gpu_id);
    if (rc) return ret(rc);
    if (!out || !f32_operand(a) || !f32_operand(b) || !out->data_virt || op < 0 || op > 3) return ret(TOS_EINVAL);
    const size_t n = elems(a);
    if (elems(b) != n) return ret(TOS_EINVAL);
    operand_t o[3] = {{a, n, NULL, 0}, {b, n, NULL, 0}, {out, n, NULL, 0}};
    cudaStream_t st = tos_g.stream;
    int e = stage(o, 3, 2, st);
    if (!e) e = tosk_teng_elementwise(o[2].dev, o[0].dev, o[1].dev, n, op, st);
    if (!e) e = finish_out(&o[2], st);
    return ret(tos_from_cuda(e));
}

int tos_gpu_tensor_attention(uint32_t gpu_id, tos_tensor_desc_t *out, const tos_tensor_desc_t *Q,
                             const tos_tensor_desc_t *K, const tos_tensor_desc_t *V, float scale)
{
    int rc = gpu_ok(gpu_id);
    if (rc) return ret(rc);
    if (!out || !f32_operand(Q) || !f32_operand(K) || !f32_operand(V) || !out->data_virt) return ret(TOS_EINVAL);
    if (Q->ndim != 2 || K->ndim != 2 || V->ndim != 2) return ret(TOS_ENOTSUP);
    const uint64_t seq = Q->shape[0], hd = Q->shape[1];
    if (K->shape[0] != seq || K->shape[1] != hd || V->shape[0] != seq || V->shape[1] != hd) return ret(TOS_EINVAL);
    if (seq > 65535 || hd > (1u << 20)) return ret(TOS_ENOTSUP);
    /* tensor_cpu.c:1170: 1 / sqrt(head_dim) when no scale is given */
    const float sc = scale > 0.0f ? scale : 1.0f / __builtin_sqrtf((float)hd);   /* IEEE sqrt and divide */
    operand_t o[4] = {{Q, (size_t)(seq * hd), NULL, 0}, {K, (size_t)(seq * hd), NULL, 0},
                      {V, (size_t)(seq * hd), NULL, 0}, {out, (size_t)(seq * hd), NULL, 0}};
    cudaStream_t st = tos_g.stream;
    int e = stage(o, 4, 3, st);
    float *S = NULL;
    if (!e) e = cudaMallocAsync((void **)&S, (size_t)(seq * seq) * 4, st);
    /* tensor_cpu.c:1172-1187: scores, row softmax, scores x V */
    if (!e) e = tosk_teng_scores(S, o[0].dev, o[1].dev, (int)seq, (int)hd, sc, st);
    if (!e) e = tosk_teng_softmax_rows(S, S, (int)seq, (int)seq, st);
    if (!e) e = tosk_teng_matmul(o[3].dev, S, o[2].dev, (int)seq, (int)hd, (int)seq, st);
    if (!e) e = finish_out(&o[3], st);
    if (S) cudaFreeAsync(S, st);
    cudaStreamSynchronize(st);
    return ret(tos_from_cuda(e));
}
