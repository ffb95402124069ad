// tensor_ops.cu - the operators behind the reference's GPU dispatch point
// (kernel/drivers/gpu/gpu.c:155-225, routed by runtime/tensor/
// tensor_engine.c:28-104), with the results of the engine's CPU operators
// (runtime/tensor/tensor_cpu.c), bit for bit:
//   * matmul: tensor_cpu_matmul (tensor_cpu.c:575-631).  Its BLIS-style
//     blocking does not change its arithmetic: every C element starts at 0
//     and gets c = c + a*b for k in order (the 4x4 micro-kernel keeps the
//     element in a lane, the edge path adds in place; tensor_cpu.c:453-573).
//     Here a tiled SIMT GEMM gives each thread whole elements and the same
//     serial k chain (no FMA: -fmad=false, explicit _rn ops).
//   * softmax over rows: tensor_cpu_softmax (tensor_cpu.c:318-335).
//   * layer norm over rows: tensor_cpu_layernorm (tensor_cpu.c:344-368:
//     tensor_cpu_reduce_sum's four lane sums, the serial variance).
//   * element-wise add / mul / sub / div (gpu.h:94 op codes).
//   * attention: tensor_cpu_attention (tensor_cpu.c:1167-1188): Q K^T with
//     tensor_cpu_dot's four lane sums, times the scale, row softmax, then
//     the matmul above.
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {
namespace teng {

// tensor_cpu.c:108-133 (the engine's exponential; also in tf_engine.cu)
__device__ __forceinline__ float fast_expf(float x) {
  if (x > 88.72f) return 3.4028235e+38f;
  if (x < -87.33f) return 0.0f;
  const float n = __fmul_rn(x, 1.44269504089f);
  const int ni = __float2int_rz(__fadd_rn(n, n > 0.0f ? 0.5f : -0.5f));
  const float nf = __int2float_rn(ni);
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(nf, 0.693359375f)), __fmul_rn(nf, -2.12194440e-4f));
  float p = __fadd_rn(0.041666668f, __fmul_rn(r, 0.008333334f));
  p = __fadd_rn(0.166666667f, __fmul_rn(r, p));
  p = __fadd_rn(0.5f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
}

// C[M][N] = A[M][K] B[K][N]: 64x64 tiles of C per CTA, 16x16 threads with
// 4x4 elements each, K staged 16 at a time; element (i, j) is the serial
// chain c = c + A[i][k] * B[k][j], k = 0, 1, ...
constexpr int kTile = 64, kKt = 16;
__global__ void __launch_bounds__(256) matmul_kernel(float* __restrict__ C, const float* __restrict__ A,
                                                     const float* __restrict__ B, int M, int N, int K) {
  __shared__ float As[kKt][kTile + 1];
  __shared__ float Bs[kKt][kTile + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int i0 = blockIdx.y * kTile, j0 = blockIdx.x * kTile;
  float c[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) c[a][b] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += kKt) {
    for (int e = threadIdx.x; e < kKt * kTile; e += 256) {
      const int kk = e / kTile, ii = e % kTile;
      const int gi = i0 + ii, gk = k0 + kk;
      As[kk][ii] = (gi < M && gk < K) ? A[(size_t)gi * K + gk] : 0.0f;
      const int gj = j0 + ii;
      Bs[kk][ii] = (gk < K && gj < N) ? B[(size_t)gk * N + gj] : 0.0f;
    }
    __syncthreads();
    const int kn = min(kKt, K - k0);
    for (int kk = 0; kk < kn; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        a[t] = As[kk][ty + 16 * t];
        b[t] = Bs[kk][tx + 16 * t];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) c[u][v] = __fadd_rn(c[u][v], __fmul_rn(a[u], b[v]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int gi = i0 + ty + 16 * u, gj = j0 + tx + 16 * v;
      if (gi < M && gj < N) C[(size_t)gi * N + gj] = c[u][v];
    }
}

// tensor_cpu_softmax of each row of n (in place allowed): max from x[0]
// (strict >, so a NaN x[0] stays and later NaNs never win), e = fast_expf(x -
// max), serial sum, x * (1/sum) when sum > 0.  One CTA per row.
__global__ void __launch_bounds__(256) softmax_rows_kernel(float* __restrict__ out, const float* __restrict__ x,
                                                           int n) {
  __shared__ float red[8];
  __shared__ float s_max, s_inv;
  const float* xr = x + (size_t)blockIdx.x * n;
  float* orow = out + (size_t)blockIdx.x * n;
  // the maximum over the non-NaN elements; x[0] NaN -> NaN (the serial rule)
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, xr[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
    // every element NaN: fmaxf gives NaN only through x[0]; keep the serial result
    s_max = (xr[0] != xr[0]) ? xr[0] : (mm == -INFINITY ? xr[0] : mm);
  }
  __syncthreads();
  const float mx = s_max;
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = fast_expf(__fsub_rn(xr[i], mx));
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s = __fadd_rn(s, orow[i]);
    s_inv = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
  }
  __syncthreads();
  if (s_inv != 0.0f)
    for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = __fmul_rn(orow[i], s_inv);
}

// tensor_cpu_layernorm of each row of n, then out * gamma + beta when given
// (per element of the row).  sum: four lane sums over i = 0, 4, 8, ...,
// ((l0 + l1) + l2) + l3, then the scalar tail; mean = sum / n; variance
// sum of (x - mean)^2 serially; inv = 1 / sqrt(var / n + eps); (x - mean) * inv.
__global__ void __launch_bounds__(128) layernorm_rows_kernel(float* __restrict__ out, const float* __restrict__ x,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ beta, int n, float eps) {
  __shared__ float lane[4];
  __shared__ float s_mean, s_inv;
  const float* xr = x + (size_t)blockIdx.x * n;
  float* orow = out + (size_t)blockIdx.x * n;
  const int n4 = n & ~3;
  if (threadIdx.x < 4) {
    float a = 0.0f;
    for (int i = threadIdx.x; i < n4; i += 4) a = __fadd_rn(a, xr[i]);
    lane[threadIdx.x] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = __fadd_rn(__fadd_rn(__fadd_rn(lane[0], lane[1]), lane[2]), lane[3]);
    for (int i = n4; i < n; ++i) s = __fadd_rn(s, xr[i]);
    const float mean = __fdiv_rn(s, (float)n);
    float v = 0.0f;
    for (int i = 0; i < n; ++i) {
      const float d = __fsub_rn(xr[i], mean);
      v = __fadd_rn(v, __fmul_rn(d, d));
    }
    s_mean = mean;
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)n), eps)));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float y = __fmul_rn(__fsub_rn(xr[i], s_mean), s_inv);
    if (gamma) y = __fmul_rn(y, gamma[i]);
    if (beta) y = __fadd_rn(y, beta[i]);
    orow[i] = y;
  }
}

// out = a op b element-wise (gpu.h:94: 0 add, 1 mul, 2 sub, 3 div)
__global__ void elementwise_kernel(float* __restrict__ out, const float* __restrict__ a,
                                   const float* __restrict__ b, size_t n, int op) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float x = a[i], y = b[i];
    out[i] = op == 0 ? __fadd_rn(x, y) : op == 1 ? __fmul_rn(x, y) : op == 2 ? __fsub_rn(x, y) : __fdiv_rn(x, y);
  }
}

// S[i][j] = tensor_cpu_dot(Q_i, K_j) * scale: four lane sums (lane l takes
// d = 4t + l), ((l0 + l1) + l2) + l3, then the scalar tail.
__global__ void scores_kernel(float* __restrict__ S, const float* __restrict__ Q, const float* __restrict__ Kt,
                              int seq, int hd, float scale) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
  if (j >= seq) return;
  const float* q = Q + (size_t)i * hd;
  const float* k = Kt + (size_t)j * hd;
  const int h4 = hd & ~3;
  float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f;
  for (int d = 0; d < h4; d += 4) {
    l0 = __fadd_rn(l0, __fmul_rn(q[d], k[d]));
    l1 = __fadd_rn(l1, __fmul_rn(q[d + 1], k[d + 1]));
    l2 = __fadd_rn(l2, __fmul_rn(q[d + 2], k[d + 2]));
    l3 = __fadd_rn(l3, __fmul_rn(q[d + 3], k[d + 3]));
  }
  float s = __fadd_rn(__fadd_rn(__fadd_rn(l0, l1), l2), l3);
  for (int d = h4; d < hd; ++d) s = __fadd_rn(s, __fmul_rn(q[d], k[d]));
  S[(size_t)i * seq + j] = __fmul_rn(s, scale);
}

}  // namespace teng
}  // namespace tos

using namespace tos::teng;

extern "C" int tosk_teng_matmul(float* C, const float* A, const float* B, int M, int N, int K, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return (int)cudaErrorInvalidValue;
  dim3 grid((N + kTile - 1) / kTile, (M + kTile - 1) / kTile);
  if (grid.y > 65535) return (int)cudaErrorInvalidValue;
  matmul_kernel<<<grid, 256, 0, st>>>(C, A, B, M, N, K);
  return (int)cudaGetLastError();
}

extern "C" int tosk_teng_softmax_rows(float* out, const float* x, int rows, int n, cudaStream_t st) {
  if (rows <= 0 || n <= 0) return (int)cudaErrorInvalidValue;
  softmax_rows_kernel<<<rows, 256, 0, st>>>(out, x, n);
  return (int)cudaGetLastError();
}

extern "C" int tosk_teng_layernorm_rows(float* out, const float* x, const float* gamma, const float* beta, int rows,
                                        int n, float eps, cudaStream_t st) {
  if (rows <= 0 || n <= 0) return (int)cudaErrorInvalidValue;
  layernorm_rows_kernel<<<rows, 128, 0, st>>>(out, x, gamma, beta, n, eps);
  return (int)cudaGetLastError();
}

extern "C" int tosk_teng_elementwise(float* out, const float* a, const float* b, size_t n, int op, cudaStream_t st) {
  if (op < 0 || op > 3) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  size_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  elementwise_kernel<<<(unsigned)blocks, 256, 0, st>>>(out, a, b, n, op);
  return (int)cudaGetLastError();
}

extern "C" int tosk_teng_scores(float* S, const float* Q, const float* K, int seq, int hd, float scale,
                                cudaStream_t st) {
  if (seq <= 0 || hd <= 0 || seq > 65535) return (int)cudaErrorInvalidValue;
  scores_kernel<<<dim3((seq + 127) / 128, seq), 128, 0, st>>>(S, Q, K, seq, hd, scale);
  return (int)cudaGetLastError();
}
