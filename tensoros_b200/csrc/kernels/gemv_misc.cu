// gemv_misc.cu - the reference's less common GEMV row formats, exact:
//   F16 / F32 weight rows (runtime/nn/llm.c:239-284) and the fp32-scale
//   20-byte Q4 blocks of runtime/nn/quantize4.c:122-198.
// One thread per output row keeps the reference's serial order; these formats
// are off the Q4_0/Q8_0 hot path.
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

// llm.c:239-259 (F16): one 4-lane accumulator over i step 4, horizontal sum
// added to the row sum, then the scalar tail.
// llm.c:260-284 (F32): two 4-lane accumulators over i step 8, acc0+acc1,
// horizontal sum added to the row sum, then the scalar tail.
__global__ void gemv_float_kernel(const uint8_t* __restrict__ w, int type, const float* __restrict__ x,
                                  float* __restrict__ out, int rows, int n) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float sum = 0.0f;
  if (type == TOSK_F16) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(w) + (size_t)r * n;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int i = 0;
    for (; i + 4 <= n; i += 4)
      for (int l = 0; l < 4; ++l) acc[l] = __fadd_rn(acc[l], __fmul_rn(h2f(h[i + l]), x[i + l]));
    sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), acc[2]), acc[3]));
    for (; i < n; ++i) sum = __fadd_rn(sum, __fmul_rn(h2f(h[i]), x[i]));
  } else {
    const float* f = reinterpret_cast<const float*>(w) + (size_t)r * n;
    float a0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, a1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int i = 0;
    for (; i + 8 <= n; i += 8)
      for (int l = 0; l < 4; ++l) {
        a0[l] = __fadd_rn(a0[l], __fmul_rn(f[i + l], x[i + l]));
        a1[l] = __fadd_rn(a1[l], __fmul_rn(f[i + 4 + l], x[i + 4 + l]));
      }
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = __fadd_rn(a0[l], a1[l]);
    sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), t[2]), t[3]));
    for (; i < n; ++i) sum = __fadd_rn(sum, __fmul_rn(f[i], x[i]));
  }
  out[r] = sum;
}

// quantize4.c:122-198: block {float scale; u8 data[16]}, lane tree as Q4_0,
// block value scale * hsum, row sum serial over blocks from 0.
__global__ void q4f_gemv_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                float* __restrict__ out, int rows, int nb) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float sum = 0.0f;
  for (int b = 0; b < nb; ++b) {
    const uint8_t* blk = w + ((size_t)r * nb + b) * 20;
    const float scale = *reinterpret_cast<const float*>(blk);
    const float* xb = x + 32 * b;
    float ch[8];
    for (int c = 0; c < 8; ++c) ch[c] = 0.0f;
    for (int k = 0; k < 4; ++k)
      for (int c = 0; c < 8; ++c) {
        const int e = 8 * k + c;
        const uint8_t byte = blk[4 + (e >> 1)];
        const int nib = (e & 1) ? (byte >> 4) : (byte & 0x0F);
        ch[c] = __fadd_rn(ch[c], __fmul_rn((float)(nib - 8), xb[e]));
      }
    const float t0 = __fadd_rn(ch[0], ch[4]), t1 = __fadd_rn(ch[1], ch[5]);
    const float t2 = __fadd_rn(ch[2], ch[6]), t3 = __fadd_rn(ch[3], ch[7]);
    sum = __fadd_rn(sum, __fmul_rn(scale, __fadd_rn(__fadd_rn(__fadd_rn(t0, t1), t2), t3)));
  }
  out[r] = sum;
}

}  // namespace tos

extern "C" int tosk_gemv_float(const void* w, int type, const float* x, float* out, int rows, int cols,
                               cudaStream_t st) {
  if (type != TOSK_F16 && type != TOSK_F32) return (int)cudaErrorInvalidValue;
  if (rows <= 0) return 0;
  tos::gemv_float_kernel<<<(rows + 127) / 128, 128, 0, st>>>((const uint8_t*)w, type, x, out, rows, cols);
  return (int)cudaGetLastError();
}

extern "C" int tosk_q4f_gemv(const void* blocks, const float* x, float* out, int rows, int cols,
                             cudaStream_t st) {
  if (rows <= 0) return 0;
  if (cols % 32) return (int)cudaErrorInvalidValue;
  tos::q4f_gemv_kernel<<<(rows + 127) / 128, 128, 0, st>>>((const uint8_t*)blocks, x, out, rows, cols / 32);
  return (int)cudaGetLastError();
}
