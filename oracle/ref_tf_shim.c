/*
 * ref_tf_shim.c - hosted stand-ins for the kernel services that the
 * reference's runtime/tensor/tensor_cpu.c links against (test
 * infrastructure, oracle/_ref only): one CPU (kernel/core/smp.h:43-102 with
 * no application processors started, work run inline) and the tensor heap
 * (runtime/tensor/tensor_cpu.h:19-20) as malloc/free.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "kernel/core/smp.h"

smp_state_t smp;

int smp_dispatch(uint32_t cpu_id, smp_work_fn_t fn, void *arg)
{
    (void)cpu_id;
    fn(arg);
    return 0;
}

void smp_wait_all(void) {}

void *tensor_alloc(uint64_t size) { return malloc((size_t)size); }
void tensor_free(void *ptr) { free(ptr); }
