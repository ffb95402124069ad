/*
 * ref_q4_shim.c - link stubs for the demo-only dependencies of the reference's
 * runtime/nn/quantize4.c (test infrastructure, oracle/_ref only).
 *
 * quantize4.c's q4_run_demos (quantize4.c:322-555) references the fp32 MLP,
 * INT16 quantizer (the tensor_cpu helpers are the reference's own
 * runtime/tensor/tensor_cpu.c, linked for the fp32 engine); the oracle calls only q4_dot_block
 * and q4_gemv (quantize4.c:122-198), so these symbols exist only to satisfy
 * the linker and abort if ever reached.
 */
#include <stdlib.h>

void nn_forward(void) { abort(); }
void nn_model_init(void) { abort(); }
void nn_qforward(void) { abort(); }
void nn_quant_reset_pool(void) { abort(); }
void nn_quantize_model(void) { abort(); }
