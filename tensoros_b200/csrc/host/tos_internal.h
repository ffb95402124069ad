/*
 * tos_internal.h - shared state of the C11 host runtime (not installed).
 */
#ifndef TOS_INTERNAL_H
#define TOS_INTERNAL_H

#include <cuda_runtime_api.h>
#include <stddef.h>

#include "tensoros_nn_gpu.h"
#include "tos_kernels.h"

struct tos_weight {
    tosk_qmat_t m;
};

typedef struct {
    int inited;
    int device;
    cudaStream_t stream;
    int *err_dev;           /* device-side error word of bounded waits */
    void *scratch;          /* device scratch for the host-pointer drop-ins */
    size_t scratch_bytes;
} tos_lib_t;

extern tos_lib_t tos_g;

int tos_set_status(int st);
int tos_from_cuda(int cuda_err);
int tos_ensure_init(void);
void *tos_scratch(size_t bytes);
int tos_check_device_error(void);
cudaStream_t tos_pick_stream(void *s);

/* RoPE arguments the reference's range reduction (llm.c:468-482) can finish
 * on: a finite base and positions below 2^20. */
#define TOS_MAX_POS (1 << 20)
int tos_rope_args_ok(int pos, float base);

/* NCCL plumbing (tos_shard.c) */
int tos_nccl_comm_init(void **comm, int world, int rank, const void *id);
void tos_nccl_comm_destroy(void *comm);
int tos_nccl_all_gather(const void *send, void *recv, size_t count, int is_int, void *comm, cudaStream_t st);

#endif
