/*
 * ref_engine_hosted.c - hosted build of the reference's tensor engine
 * dispatch (test infrastructure, oracle/_ref only).
 *
 * Textually includes the UNMODIFIED runtime/tensor/tensor_engine.c so that
 * its file-static routing rule, select_backend (tensor_engine.c:28-67), can
 * be called with chosen tensors and GPU counts.  The kernel state it reads
 * (kstate.gpu_count, kernel/core/kernel.h:142-156) and the GPU driver's
 * entry points it calls (kernel/drivers/gpu/gpu.h:80-96) are supplied here:
 * the entry points record which one was called, as the reference's own
 * stubs compute nothing either.
 */
#include <stdlib.h>

#include "runtime/tensor/tensor_engine.c"

struct kernel_state kstate;

void *kmalloc(size_t n) { return malloc(n); }
void kfree(void *p) { free(p); }

static int g_gpu_called;   /* 1 matmul, 2 attention, 3 softmax, 4 layernorm, 5 elementwise */

int gpu_tensor_matmul(uint32_t g, tensor_desc_t *C, const tensor_desc_t *A, const tensor_desc_t *B)
{ (void)g; (void)C; (void)A; (void)B; g_gpu_called = 1; return 0; }
int gpu_tensor_attention(uint32_t g, tensor_desc_t *o, const tensor_desc_t *q, const tensor_desc_t *k,
                         const tensor_desc_t *v, float s)
{ (void)g; (void)o; (void)q; (void)k; (void)v; (void)s; g_gpu_called = 2; return 0; }
int gpu_tensor_softmax(uint32_t g, tensor_desc_t *o, const tensor_desc_t *i, int a)
{ (void)g; (void)o; (void)i; (void)a; g_gpu_called = 3; return 0; }
int gpu_tensor_layernorm(uint32_t g, tensor_desc_t *o, const tensor_desc_t *i, const tensor_desc_t *ga,
                         const tensor_desc_t *b, float e)
{ (void)g; (void)o; (void)i; (void)ga; (void)b; (void)e; g_gpu_called = 4; return 0; }
int gpu_tensor_elementwise(uint32_t g, tensor_desc_t *o, const tensor_desc_t *a, const tensor_desc_t *b, int op)
{ (void)g; (void)o; (void)a; (void)b; (void)op; g_gpu_called = 5; return 0; }

/* select_backend for count tensors of the given byte sizes with gpu_count GPUs */
int ref_select_backend(int op, const uint64_t *sizes, int count, int gpu_count)
{
    tensor_desc_t t[8];
    if (count > 8) return -1;
    for (int i = 0; i < count; i++) {
        memset(&t[i], 0, sizeof(t[i]));
        t[i].size_bytes = sizes[i];
    }
    kstate.gpu_count = (uint32_t)gpu_count;
    return (int)select_backend((tir_opcode_t)op, t, (uint32_t)count);
}
