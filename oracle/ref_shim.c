/*
 * ref_shim.c - hosted stand-ins for the freestanding kernel services that
 * runtime/nn/llm.c and runtime/nn/gguf.c link against (test infrastructure,
 * built only into oracle/_ref/libtos_ref.so).
 *
 * kprintf, kmemset/kmemcpy and kstrlen/kstrcpy follow kernel/core/kernel.h:183-245;
 * the perf helpers follow kernel/core/perf.h:53-62; the virtio_blk calls follow
 * kernel/drivers/blk/virtio_blk.h:84-94 and report "no disk"; the x86 JIT entry
 * jit_compile_q8_gemv (runtime/jit/x86_jit.h) returns NULL so that llm_gemv
 * takes its portable C path (llm.c:343-348).
 */
#include <stdarg.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

int kprintf(const char *fmt, ...)
{
    (void)fmt;
    return 0;
}

int kprintf_debug(const char *fmt, ...)
{
    (void)fmt;
    return 0;
}

int kprintf_to_buf(char *buf, int buflen, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    int n = vsnprintf(buf, (size_t)buflen, fmt, ap);
    va_end(ap);
    return n;
}

void *kmemset(void *s, int c, size_t n) { return memset(s, c, n); }
void *kmemcpy(void *d, const void *s, size_t n) { return memcpy(d, s, n); }
int kstrcmp(const char *a, const char *b) { return strcmp(a, b); }
int kstrncmp(const char *a, const char *b, size_t n) { return strncmp(a, b, n); }
size_t kstrlen(const char *s) { return strlen(s); }
char *kstrcpy(char *d, const char *s) { return strcpy(d, s); }
char *kstrncpy(char *d, const char *s, size_t n) { return strncpy(d, s, n); }

uint64_t perf_tsc_mhz(void) { return 1000; }
uint64_t perf_cycles_to_ns(uint64_t c) { return c; }
uint64_t perf_cycles_to_us(uint64_t c) { return c / 1000; }
void perf_calibrate(void) {}

uint64_t virtio_blk_capacity(void) { return 0; }
int virtio_blk_read(uint64_t sector, uint32_t count, void *buf)
{
    (void)sector; (void)count; (void)buf;
    return -1;
}

char __model_cache_start[16];
char __model_cache_end[1];

void *jit_compile_q8_gemv(int rows, int cols)
{
    (void)rows; (void)cols;
    return NULL;
}
