/*
 * tos_synth.h - seeded synthetic inputs for the TensorOS decode-path workloads.
 *
 * Every value is a pure function of (seed, stream, index): a splitmix64-style
 * counter hash, so results do not depend on how many threads generate them.
 * Normals use Box-Muller in double precision.  The layouts are the GGUF ones
 * the reference reads in place (runtime/nn/llm.c:142-146):
 *   Q4_0 block = {u16 fp16 scale; u8 qs[16]}  (18 bytes, element 2j = low
 *                nibble of qs[j], 2j+1 = high nibble, value (nibble-8)*scale)
 *   Q8_0 block = {u16 fp16 scale; i8 qs[32]}  (34 bytes)
 * Scales are fp16_rne(|N(0, scale_std)|); Q4_0 nibbles are uniform 0..15;
 * Q8_0 values are uniform in [-127, 127].
 *
 * This library (libtos_synth.so) is host C11 with no CUDA dependency.
 */
#ifndef TOS_SYNTH_H
#define TOS_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint64_t tos_synth_u64(uint64_t seed, uint64_t stream, uint64_t index);
/* IEEE fp32 -> fp16 round-to-nearest-even (bit pattern) */
uint16_t tos_synth_f32_to_f16(float f);

void tos_synth_normal_f32(float *out, size_t n, uint64_t seed, uint64_t stream,
                          float mean, float std, int n_threads);
void tos_synth_normal_f16(uint16_t *out, size_t n, uint64_t seed, uint64_t stream,
                          float mean, float std, int n_threads);
void tos_synth_q4_0(void *out, size_t n_blocks, uint64_t seed, uint64_t stream,
                    float scale_std, int n_threads);
void tos_synth_q8_0(void *out, size_t n_blocks, uint64_t seed, uint64_t stream,
                    float scale_std, int n_threads);
/* quantize4.c's 20-byte fp32-scale Q4 block (runtime/nn/quantize4.h:30-33):
 * scale = |N(0, scale_std)| as fp32, nibbles uniform 0..15 */
void tos_synth_q4f(void *out, size_t n_blocks, uint64_t seed, uint64_t stream,
                   float scale_std, int n_threads);
void tos_synth_tokens(int32_t *out, size_t n, int32_t vocab, uint64_t seed, uint64_t stream);

#ifdef __cplusplus
}
#endif
#endif
