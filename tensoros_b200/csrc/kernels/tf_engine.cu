// tf_engine.cu - the fp32 transformer engine of TensorOS runtime/nn
// (runtime/nn/transformer.c:92-366) on sm_100a, bit-identical to it.
//
// The engine is the reference's other decoder: fp32 weights (no
// quantisation), a KV cache laid out [layer][head][seq][head_dim]
// (transformer.c:67-81), RMSNorm with eps 1e-5 and a single serial sum of
// squares (transformer.c:92-113), and its activations from
// runtime/tensor/tensor_cpu.c (fast_expf's range-reduced polynomial, SiLU,
// the three-pass softmax).  Every rounding of those C loops is kept: IEEE
// round-to-nearest intrinsics, no FMA contraction (-fmad=false), the
// reference's summation orders:
//   * "chunk" rows (tf_swiglu_ffn, the o projection, the logits;
//     transformer.c:130-183, 328-340, 355-365): sum += ((p0 + p1) + p2) + p3
//     over groups of four products, then the scalar tail;
//   * "scalar" rows (q, k, v; transformer.c:290-301): sum += w * x in order;
//   * attention (transformer.c:193-247): chunk dot products times
//     1/sqrt(head_dim), tensor_cpu_softmax (serial max and sum,
//     tensor_cpu.c:318-335), out = out + p * v in position order.
// These are serial chains per output element, so the kernels give each
// element one thread and run the elements of a vector in parallel; the
// engine is a small demo model (dims up to a few hundred), latency-bound.
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {
namespace tf {

// runtime/tensor/tensor_cpu.c:108-133: exp(x) = 2^n * p(r), n = (int)(x*log2e
// +- 0.5) (truncating conversion), r = (x - n*ln2_hi) - n*ln2_lo, p a degree-5
// polynomial in Horner form, 2^n built from its exponent bits.  The
// reference's own function, restated operation by operation.
__device__ __forceinline__ float fast_expf(float x) {
  if (x > 88.72f) return 3.4028235e+38f;
  if (x < -87.33f) return 0.0f;
  const float kLog2e = 1.44269504089f, kLn2Hi = 0.693359375f, kLn2Lo = -2.12194440e-4f;
  const float n = __fmul_rn(x, kLog2e);
  const int ni = __float2int_rz(__fadd_rn(n, n > 0.0f ? 0.5f : -0.5f));
  const float nf = __int2float_rn(ni);
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(nf, kLn2Hi)), __fmul_rn(nf, kLn2Lo));
  float p = __fadd_rn(0.041666668f, __fmul_rn(r, 0.008333334f));
  p = __fadd_rn(0.166666667f, __fmul_rn(r, p));
  p = __fadd_rn(0.5f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  const float scale = __uint_as_float((uint32_t)(ni + 127) << 23);
  return __fmul_rn(p, scale);
}

// tensor_cpu.c:307-311: x / (1 + exp(-x))
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, fast_expf(-x))); }

// One row of y = W x in the engine's orders (row: cols consecutive floats).
template <bool kChunk>
__device__ __forceinline__ float row_dot(const float* __restrict__ row, const float* __restrict__ x, int cols) {
  float sum = 0.0f;
  int j = 0;
  if constexpr (kChunk) {
    for (; j + 4 <= cols; j += 4) {
      const float p0 = __fmul_rn(row[j], x[j]), p1 = __fmul_rn(row[j + 1], x[j + 1]);
      const float p2 = __fmul_rn(row[j + 2], x[j + 2]), p3 = __fmul_rn(row[j + 3], x[j + 3]);
      sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(__fadd_rn(p0, p1), p2), p3));
    }
  }
  for (; j < cols; ++j) sum = __fadd_rn(sum, __fmul_rn(row[j], x[j]));
  return sum;
}

// y[i] = row i of W (rows x cols, row-major) . x; x staged in shared memory.
template <bool kChunk>
__global__ void __launch_bounds__(128) matvec_kernel(const float* __restrict__ W, const float* __restrict__ x,
                                                     float* __restrict__ y, int rows, int cols) {
  extern __shared__ float xs[];
  for (int j = threadIdx.x; j < cols; j += blockDim.x) xs[j] = x[j];
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) y[i] = row_dot<kChunk>(W + (size_t)i * cols, xs, cols);
}

// transformer.c:92-113: serial sum of squares, ss / dim + 1e-5, 1 / sqrt,
// out = (x * inv) * w.  One CTA.
__global__ void __launch_bounds__(256) rmsnorm_kernel(float* __restrict__ out, const float* __restrict__ x,
                                                      const float* __restrict__ w, int dim) {
  __shared__ float inv;
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int i = 0; i < dim; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
    ss = __fadd_rn(__fdiv_rn(ss, (float)dim), 1e-5f);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(ss));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// transformer.c:183-184 (tensor_cpu_silu, then tensor_cpu_mul): g = silu(g) * u
__global__ void silu_mul_kernel(float* __restrict__ g, const float* __restrict__ u, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) g[i] = __fmul_rn(silu(g[i]), u[i]);
}

// x += y (transformer.c:343-344, 352-353)
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}

// tf_cached_attention (transformer.c:193-247) for heads [h0, h0 + gridDim.x)
// of one layer: q, k, v of head h at q + h * qstride etc.; the cache rows of
// (layer, head) start at kc + ((layer * n_heads + head) * max_seq) * hd.
// scores: shared memory of max_seq floats.
__global__ void __launch_bounds__(128) attention_kernel(float* __restrict__ out, int ostride,
                                                        const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, int qstride,
                                                        float* __restrict__ kc, float* __restrict__ vc, int layer,
                                                        int h0, int n_heads, int hd, int max_seq, int pos) {
  extern __shared__ float sh[];
  float* sc = sh;                  // [pos + 1] scores, then probabilities
  float* red = sh + max_seq;       // [2]: max, then 1/sum (or 0: no scaling)
  const int h = h0 + blockIdx.x;
  const float* qh = q + (size_t)blockIdx.x * qstride;
  float* kbase = kc + ((size_t)layer * n_heads + h) * max_seq * hd;
  float* vbase = vc + ((size_t)layer * n_heads + h) * max_seq * hd;
  const int n = pos + 1;
  // append k, v (transformer.c:200-205)
  for (int i = threadIdx.x; i < hd; i += blockDim.x) {
    kbase[(size_t)pos * hd + i] = k[(size_t)blockIdx.x * qstride + i];
    vbase[(size_t)pos * hd + i] = v[(size_t)blockIdx.x * qstride + i];
  }
  __syncthreads();
  // scores (transformer.c:208-223): chunk dot products times the scale
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = __fmul_rn(row_dot<true>(kbase + (size_t)j * hd, qh, hd), scale);
  __syncthreads();
  // tensor_cpu_softmax (tensor_cpu.c:318-335): max from x[0] (strict >),
  // e = fast_expf(x - max), serial sum, then x * (1 / sum) if the sum > 0
  if (threadIdx.x == 0) {
    float m = sc[0];
    for (int j = 1; j < n; ++j)
      if (sc[j] > m) m = sc[j];
    red[0] = m;
  }
  __syncthreads();
  const float m = red[0];
  for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = fast_expf(__fsub_rn(sc[j], m));
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int j = 0; j < n; ++j) s = __fadd_rn(s, sc[j]);
    red[1] = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
  }
  __syncthreads();
  if (red[1] != 0.0f)
    for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = __fmul_rn(sc[j], red[1]);
  __syncthreads();
  // out = sum_j p_j v_j, position order (transformer.c:233-246)
  for (int i = threadIdx.x; i < hd; i += blockDim.x) {
    float o = 0.0f;
    for (int j = 0; j < n; ++j) o = __fadd_rn(o, __fmul_rn(sc[j], vbase[(size_t)j * hd + i]));
    out[(size_t)blockIdx.x * ostride + i] = o;
  }
}

}  // namespace tf
}  // namespace tos

using namespace tos::tf;

static int check_launch() { return (int)cudaGetLastError(); }

extern "C" int tosk_tf_matvec(const float* W, const float* x, float* y, int rows, int cols, int chunk_order,
                              cudaStream_t st) {
  if (rows <= 0 || cols <= 0 || (size_t)cols * 4 > 200 * 1024) return (int)cudaErrorInvalidValue;
  const size_t smem = (size_t)cols * 4;
  const int grid = (rows + 127) / 128;
  if (chunk_order) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(matvec_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    matvec_kernel<true><<<grid, 128, smem, st>>>(W, x, y, rows, cols);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(matvec_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    matvec_kernel<false><<<grid, 128, smem, st>>>(W, x, y, rows, cols);
  }
  return check_launch();
}

extern "C" int tosk_tf_rmsnorm(float* out, const float* x, const float* w, int dim, cudaStream_t st) {
  if (dim <= 0) return (int)cudaErrorInvalidValue;
  rmsnorm_kernel<<<1, 256, 0, st>>>(out, x, w, dim);
  return check_launch();
}

extern "C" int tosk_tf_silu_mul(float* g, const float* u, int n, cudaStream_t st) {
  if (n <= 0) return 0;
  silu_mul_kernel<<<(n + 255) / 256, 256, 0, st>>>(g, u, n);
  return check_launch();
}

extern "C" int tosk_tf_add(float* x, const float* y, int n, cudaStream_t st) {
  if (n <= 0) return 0;
  add_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, y, n);
  return check_launch();
}

extern "C" int tosk_tf_attention(float* out, int ostride, const float* q, const float* k, const float* v, int qstride,
                                 float* kc, float* vc, int layer, int h0, int nh, int n_heads, int hd, int max_seq,
                                 int pos, cudaStream_t st) {
  if (nh <= 0 || hd <= 0 || pos < 0 || pos >= max_seq || h0 < 0 || h0 + nh > n_heads) return (int)cudaErrorInvalidValue;
  const size_t smem = ((size_t)max_seq + 2) * 4;
  if (smem > 200 * 1024) return (int)cudaErrorInvalidValue;
  if (smem > 48 * 1024) cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  attention_kernel<<<nh, 128, smem, st>>>(out, ostride, q, k, v, qstride, kc, vc, layer, h0, n_heads, hd, max_seq, pos);
  return check_launch();
}
