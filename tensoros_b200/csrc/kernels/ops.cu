// ops.cu - exact device versions of runtime/nn/llm.c's small operators.
//
// Each kernel reproduces the fp32 operation order of the reference operator
// named beside it, using IEEE round-to-nearest intrinsics only.  Serial
// reference chains (the RMSNorm lane sums, the softmax sum) stay serial: they
// are short (dim/4, n) and run in one thread while the other threads do the
// element-parallel parts.
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

// llm.c:352-362 llm_get_f: F32 / F16 read, any other type reads 0
__device__ __forceinline__ float get_f(const void* w, int i, int type) {
  if (type == TOSK_F32) return reinterpret_cast<const float*>(w)[i];
  if (type == TOSK_F16) return h2f(reinterpret_cast<const uint16_t*>(w)[i]);
  return 0.0f;
}

// llm.c:416-442 (single CTA).  Lane l of warp 0 (l < 4) sums x[4i+l]^2
// serially; thread 0 combines ((s0+s1)+s2)+s3, adds the scalar tail, and
// forms 1/sqrt(ss/dim + eps); every thread then writes (x*ss)*w.
__global__ void rmsnorm_kernel(float* __restrict__ out, const float* __restrict__ x,
                               const void* __restrict__ w, int wtype, int dim, float eps) {
  __shared__ float lanes[4];
  __shared__ float s_ss;
  pdl_wait();
  if (threadIdx.x < 4) {
    float acc = 0.0f;
    for (int i0 = 0; i0 + 4 <= dim; i0 += 4) {
      const float v = x[i0 + threadIdx.x];
      acc = __fadd_rn(acc, __fmul_rn(v, v));
    }
    lanes[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ss = __fadd_rn(__fadd_rn(__fadd_rn(lanes[0], lanes[1]), lanes[2]), lanes[3]);
    for (int i = dim & ~3; i < dim; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
    s_ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
  }
  __syncthreads();
  pdl_trigger();
  const float ss = s_ss;
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    out[i] = __fmul_rn(__fmul_rn(x[i], ss), get_f(w, i, wtype));
}

// llm.c:460-487: cos/sin for element pair i of a head at position pos.
__device__ __forceinline__ float2 rope_cs(int pos, int i, int hd, float base) {
  const float exponent = __fdiv_rn(-(float)i, (float)hd);
  // The host rejects a non-finite base and positions >= 2^20, where these
  // reduction loops of the reference would not terminate; the iteration
  // bounds below are a second guard.
  float b = base;
  int k = 0;
  while (b > 2.0f && k < 256) {
    b = __fmul_rn(b, 0.5f);
    ++k;
  }
  const float m1 = __fsub_rn(b, 1.0f);
  const float inner = __fsub_rn(1.0f, __fmul_rn(m1, __fsub_rn(0.5f, __fmul_rn(m1, 0.3333f))));
  const float log_base = __fadd_rn(__fmul_rn((float)k, 0.6931472f), __fmul_rn(m1, inner));
  const float freq = ref_expf(__fmul_rn(exponent, log_base));
  float theta = __fmul_rn((float)pos, freq);
  const float pi = 3.14159265f;
  const float two_pi = 2.0f * pi;
  for (int it = 0; theta > pi && it < (1 << 20); ++it) theta = __fsub_rn(theta, two_pi);
  for (int it = 0; theta < -pi && it < (1 << 20); ++it) theta = __fadd_rn(theta, two_pi);
  const float t2 = __fmul_rn(theta, theta);
  const float c = __fsub_rn(
      1.0f, __fmul_rn(t2, __fsub_rn(0.5f, __fmul_rn(t2, __fsub_rn(0.04166667f, __fmul_rn(t2, 0.001388889f))))));
  const float s = __fmul_rn(
      theta,
      __fsub_rn(1.0f, __fmul_rn(t2, __fsub_rn(0.1666667f,
                                              __fmul_rn(t2, __fsub_rn(0.008333333f, __fmul_rn(t2, 0.000198413f)))))));
  return make_float2(c, s);
}

__global__ void rope_table_kernel(float2* __restrict__ cs, int max_seq, int hd, float base) {
  const int half = hd >> 1;
  const long long total = (long long)max_seq * half;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int pos = (int)(idx / half);
    const int j = (int)(idx % half);
    cs[idx] = rope_cs(pos, 2 * j, hd, base);
  }
}

// llm.c:488-492 applied to n_vec consecutive heads of hd elements
__global__ void rope_kernel(float* __restrict__ vec, int n_vec, const int* __restrict__ pos_dev,
                            int pos_arg, int hd, float base) {
  const int half = hd >> 1;
  const int pos = pos_dev ? *pos_dev : pos_arg;
  const int total = n_vec * half;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int h = idx / half, j = idx % half;
    const float2 cs = rope_cs(pos, 2 * j, hd, base);
    float* v = vec + (size_t)h * hd + 2 * j;
    const float v0 = v[0], v1 = v[1];
    v[0] = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
    v[1] = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
  }
}

// llm.c:506-532 (single CTA): max (first pass, strict >), e = exp(x-max) in
// parallel, serial sum by thread 0, inv = 1/(sum+1e-10), x *= inv.
__global__ void softmax_kernel(float* __restrict__ x, int n) {
  __shared__ float s_max, s_inv;
  if (threadIdx.x == 0) {
    float m = x[0];
    for (int i = 1; i < n; ++i)
      if (x[i] > m) m = x[i];
    s_max = m;
  }
  __syncthreads();
  const float m = s_max;
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = ref_expf(__fsub_rn(x[i], m));
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, x[i]);
    s_inv = __fdiv_rn(1.0f, __fadd_rn(sum, 1e-10f));
  }
  __syncthreads();
  const float inv = s_inv;
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fmul_rn(x[i], inv);
}

enum { EW_SILU = 0, EW_VADD = 1, EW_VMUL = 2, EW_AXPY = 3 };

__global__ void elementwise_kernel(int op, float* __restrict__ dst, const float* __restrict__ src,
                                   float s, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    switch (op) {
      case EW_SILU: dst[i] = ref_silu(dst[i]); break;                            // llm.c:538-544
      case EW_VADD: dst[i] = __fadd_rn(dst[i], src[i]); break;                   // llm.c:599-614
      case EW_VMUL: dst[i] = __fmul_rn(dst[i], src[i]); break;                   // llm.c:617-632
      case EW_AXPY: dst[i] = __fadd_rn(dst[i], __fmul_rn(s, src[i])); break;     // llm.c:580-596
    }
  }
}

// llm.c:551-577: chain c (0..7) over elements 8m+c; t_l = c_l + c_{l+4};
// ((t0+t1)+t2)+t3; scalar tail.  One warp.
__global__ void dot_kernel(const float* __restrict__ a, const float* __restrict__ b, int n,
                           float* __restrict__ out) {
  const int lane = threadIdx.x;
  const int n8 = n & ~7;
  float acc = 0.0f;
  if (lane < 8)
    for (int i = 0; i < n8; i += 8) acc = __fadd_rn(acc, __fmul_rn(a[i + lane], b[i + lane]));
  const float hi = __shfl_down_sync(0xffffffffu, acc, 4);
  const float t = __fadd_rn(acc, hi);  // lanes 0..3: t_l
  const float t1 = __shfl_sync(0xffffffffu, t, 1);
  const float t2 = __shfl_sync(0xffffffffu, t, 2);
  const float t3 = __shfl_sync(0xffffffffu, t, 3);
  if (lane == 0) {
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(t, t1), t2), t3);
    for (int i = n8; i < n; ++i) sum = __fadd_rn(sum, __fmul_rn(a[i], b[i]));
    *out = sum;
  }
}

// llm.c:365-410: dequantise the embedding row of one token
__global__ void embed_kernel(float* __restrict__ out, const uint8_t* __restrict__ embd, int type,
                             int dim, const int* __restrict__ tok_dev, int tok_arg) {
  pdl_wait();
  const int tok = tok_dev ? *tok_dev : tok_arg;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (type == TOSK_Q4_0) {
      const uint8_t* blk = embd + ((size_t)tok * (dim / 32) + i / 32) * 18;
      const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
      const int j = i & 31;
      const uint8_t byte = blk[2 + (j >> 1)];
      const int nib = (j & 1) ? (byte >> 4) : (byte & 0x0F);
      v = __fmul_rn((float)(nib - 8), d);
    } else if (type == TOSK_Q8_0) {
      const uint8_t* blk = embd + ((size_t)tok * (dim / 32) + i / 32) * 34;
      const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
      v = __fmul_rn((float)(int8_t)blk[2 + (i & 31)], d);
    } else if (type == TOSK_F16) {
      v = h2f(reinterpret_cast<const uint16_t*>(embd)[(size_t)tok * dim + i]);
    } else if (type == TOSK_F32) {
      v = reinterpret_cast<const float*>(embd)[(size_t)tok * dim + i];
    }
    out[i] = v;
  }
  pdl_trigger();
}

// llm.c:1129-1140.  The serial scan returns the first strict maximum and
// never lets a NaN win except x[0]; the parallel form reduces candidates by
// (larger value, then lower index), skipping NaNs, and returns 0 when x[0]
// is NaN.  One CTA of 1024 threads.
__device__ __forceinline__ void arg_combine(float& v, int& i, float v2, int i2) {
  if (i2 < 0) return;
  if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// first_rule: the reference's rule for a whole vector (x[0] wins when it is
// NaN or nothing beats it).  Without it (a later slice of a row-sharded
// vector) the result is the first non-NaN maximum, or index -1.  Indices are
// reported plus `offset`.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int n,
                                                      int* __restrict__ out_idx,
                                                      float* __restrict__ out_val, int first_rule,
                                                      int offset) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  // one row per CTA (a grid of several CTAs reduces consecutive rows of n)
  x += (size_t)blockIdx.x * n;
  out_idx += blockIdx.x;
  if (out_val) out_val += blockIdx.x;
  float v = 0.0f;
  int idx = -1;
  // each thread scans 4 consecutive elements per step (vector loads when x
  // is 16-byte aligned), four steps in flight; in-thread order stays
  // increasing so the first maximum wins
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  const int n4 = vec ? (n & ~3) : 0;
  for (int base = 4 * threadIdx.x; base < n4; base += 16 * blockDim.x) {
    float4 c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + 4 * u * blockDim.x;
      c[u] = i < n4 ? *reinterpret_cast<const float4*>(x + i) : make_float4(NAN, NAN, NAN, NAN);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + 4 * u * blockDim.x;
      const float e[4] = {c[u].x, c[u].y, c[u].z, c[u].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (!(e[j] != e[j]) && (idx < 0 || e[j] > v || (e[j] == v && i + j < idx))) {
          v = e[j];
          idx = i + j;
        }
    }
  }
  for (int i = n4 + threadIdx.x; i < n; i += blockDim.x) {
    const float xi = x[i];
    if (!(xi != xi) && (idx < 0 || xi > v || (xi == v && i < idx))) {
      v = xi;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_down_sync(0xffffffffu, v, o);
    const int i2 = __shfl_down_sync(0xffffffffu, idx, o);
    arg_combine(v, idx, v2, i2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    v = lane < nw ? sv[lane] : 0.0f;
    idx = lane < nw ? si[lane] : -1;
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_down_sync(0xffffffffu, v, o);
      const int i2 = __shfl_down_sync(0xffffffffu, idx, o);
      arg_combine(v, idx, v2, i2);
    }
    if (lane == 0) {
      if (first_rule) {
        const float x0 = x[0];
        if (x0 != x0 || idx < 0) {
          idx = 0;
          v = x0;
        }
      }
      *out_idx = idx < 0 ? -1 : idx + offset;
      if (out_val) *out_val = v;
    }
  }
  pdl_trigger();
}

// Distributed argmax: (value bits, index) pairs of the ranks' vocabulary
// slices in rank order (rank 0 applied the whole-vector rule); a later slice
// wins only with a strictly larger value, as in llm.c:1129-1140.
__global__ void argmax_pairs_kernel(const int* __restrict__ pairs, int world, int* __restrict__ out_idx) {
  pdl_wait();
  if (threadIdx.x == 0) {
    float bv = __int_as_float(pairs[0]);
    int bi = pairs[1];
    for (int r = 1; r < world; ++r) {
      const float v = __int_as_float(pairs[2 * r]);
      const int i = pairs[2 * r + 1];
      if (i >= 0 && v > bv) {
        bv = v;
        bi = i;
      }
    }
    *out_idx = bi;
  }
  pdl_trigger();
}

// llm_sample (llm.c:1143-1246) on the device, one CTA of 1024 threads.
// The reference keeps the 40 largest logits ordered by (value descending,
// index ascending) - its insertion-based partial sort resolves equal values
// that way - then runs a short serial recipe.  Here the 40th largest value
// is found by a 4-pass radix select on order-preserving keys (-0.0 counted
// as +0.0, as float comparison does), the 40 candidates are gathered (for
// equal values at the threshold the lowest indices, by a prefix count in
// index order) and sorted, and thread 0 runs the reference's serial steps in
// its rounding order: softmax of (l - max)/T with llm_expf, nucleus 0.9,
// renormalisation, and the inverse-CDF draw with r from the entropy word
// mixed as the reference mixes its timestamp.  Finite logits.
constexpr int kSampleK = 40;

__device__ __forceinline__ uint32_t order_key(float v) {
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0;   // -0.0 == +0.0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(1024) sample_kernel(const float* __restrict__ x, int n, float temperature,
                                                      uint32_t entropy, int* __restrict__ out) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_prefix, s_need;
  __shared__ unsigned wsum[32];
  __shared__ int s_cnt;
  __shared__ float cv[kSampleK];
  __shared__ int ci[kSampleK];
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = n < kSampleK ? n : kSampleK;
  if (tid == 0) {
    s_prefix = 0;
    s_need = (unsigned)k;
    s_cnt = 0;
  }
  unsigned pmask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const unsigned prefix = s_prefix;
    for (int i = tid; i < n; i += blockDim.x) {
      const uint32_t kk = order_key(x[i]);
      if ((kk & pmask) == prefix) atomicAdd(&hist[(kk >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned need = s_need, cum = 0;
      for (int bin = 255; bin >= 0; --bin) {
        if (cum + hist[bin] >= need) {
          s_prefix = prefix | ((unsigned)bin << shift);
          s_need = need - cum;
          break;
        }
        cum += hist[bin];
      }
    }
    pmask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const unsigned need = s_need;   // elements equal to the threshold to keep (lowest indices)
  // keys above the threshold: all kept; equal ones: rank in index order
  const int chunk = (n + blockDim.x - 1) / blockDim.x;
  const int i0 = tid * chunk, i1 = min(n, i0 + chunk);
  unsigned eq = 0;
  for (int i = i0; i < i1; ++i) eq += order_key(x[i]) == T;
  unsigned incl = eq;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    unsigned w = lane < nw ? wsum[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    if (lane < nw) wsum[lane] = w;   // inclusive per-warp totals
  }
  __syncthreads();
  unsigned rank = (warp > 0 ? wsum[warp - 1] : 0u) + incl - eq;   // equal keys before this chunk
  for (int i = i0; i < i1; ++i) {
    const uint32_t kk = order_key(x[i]);
    bool take = kk > T;
    if (kk == T) {
      take = rank < need;
      ++rank;
    }
    if (take) {
      const int slot = atomicAdd(&s_cnt, 1);
      if (slot < kSampleK) {
        cv[slot] = x[i];
        ci[slot] = i;
      }
    }
  }
  __syncthreads();
  if (tid != 0) return;
  const int m = min(s_cnt, kSampleK);
  // (value descending, index ascending)
  for (int a = 1; a < m; ++a) {
    const float v = cv[a];
    const int ix = ci[a];
    int j = a - 1;
    while (j >= 0 && (cv[j] < v || (cv[j] == v && ci[j] > ix))) {
      cv[j + 1] = cv[j];
      ci[j + 1] = ci[j];
      --j;
    }
    cv[j + 1] = v;
    ci[j + 1] = ix;
  }
  float pr[kSampleK];
  const float mx = cv[0];
  float sum = 0.0f;
  for (int a = 0; a < m; ++a) {
    pr[a] = ref_expf(__fdiv_rn(__fsub_rn(cv[a], mx), temperature));
    sum = __fadd_rn(sum, pr[a]);
  }
  float inv = __fdiv_rn(1.0f, __fadd_rn(sum, 1e-10f));
  for (int a = 0; a < m; ++a) pr[a] = __fmul_rn(pr[a], inv);
  float cum = 0.0f;
  int cut = m;
  for (int a = 0; a < m; ++a) {
    cum = __fadd_rn(cum, pr[a]);
    if (cum >= 0.9f) {
      cut = a + 1;
      break;
    }
  }
  if (cut < m) {
    sum = 0.0f;
    for (int a = 0; a < cut; ++a) sum = __fadd_rn(sum, pr[a]);
    inv = __fdiv_rn(1.0f, __fadd_rn(sum, 1e-10f));
    for (int a = 0; a < cut; ++a) pr[a] = __fmul_rn(pr[a], inv);
  }
  uint32_t lo = entropy;
  lo = lo ^ (lo >> 16);
  lo = lo * 0x45d9f3bU;
  const float r = __fdiv_rn((float)(lo % 10000u), 10000.0f);
  float cdf = 0.0f;
  int pick = ci[cut - 1];
  for (int a = 0; a < cut; ++a) {
    cdf = __fadd_rn(cdf, pr[a]);
    if (cdf >= r) {
      pick = ci[a];
      break;
    }
  }
  *out = pick;
}

// Greedy decode on the device: record the token the last argmax produced
// (io[2]) in ring[io[4]], then advance the position io[1] and the counter.
__global__ void decode_advance_kernel(int* __restrict__ io, int* __restrict__ ring) {
  pdl_wait();
  const int k = io[4];
  ring[k] = io[2];
  io[4] = k + 1;
  io[1] = io[1] + 1;
  pdl_trigger();
}

}  // namespace tos

using namespace tos;

static int launch_pdl(const void* func, dim3 grid, dim3 block, void** args, int pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return (int)cudaLaunchKernelExC(&cfg, func, args);
}

extern "C" int tosk_rmsnorm(float* out, const float* x, const void* w, int wtype, int dim, float eps,
                            int pdl, cudaStream_t st) {
  if (dim <= 0) return 0;
  void* args[] = {&out, &x, &w, &wtype, &dim, &eps};
  return launch_pdl((const void*)rmsnorm_kernel, dim3(1), dim3(1024), args, pdl, st);
}

extern "C" int tosk_rope_table(float2* cs, int max_seq, int hd, float base, cudaStream_t st) {
  const long long total = (long long)max_seq * (hd / 2);
  int grid = (int)((total + 255) / 256);
  if (grid > 4096) grid = 4096;
  if (grid < 1) grid = 1;
  rope_table_kernel<<<grid, 256, 0, st>>>(cs, max_seq, hd, base);
  return (int)cudaGetLastError();
}

extern "C" int tosk_rope(float* vec, int n_vec, const int* pos_dev, int pos, int hd, float base,
                         cudaStream_t st) {
  const int total = n_vec * (hd / 2);
  if (total <= 0) return 0;
  rope_kernel<<<(total + 255) / 256, 256, 0, st>>>(vec, n_vec, pos_dev, pos, hd, base);
  return (int)cudaGetLastError();
}

extern "C" int tosk_softmax(float* x, int n, cudaStream_t st) {
  if (n <= 0) return 0;
  softmax_kernel<<<1, 1024, 0, st>>>(x, n);
  return (int)cudaGetLastError();
}

static int ew(int op, float* dst, const float* src, float s, int n, cudaStream_t st) {
  if (n <= 0) return 0;
  int grid = (n + 255) / 256;
  if (grid > 1184) grid = 1184;
  elementwise_kernel<<<grid, 256, 0, st>>>(op, dst, src, s, n);
  return (int)cudaGetLastError();
}

extern "C" int tosk_silu(float* x, int n, cudaStream_t st) { return ew(EW_SILU, x, nullptr, 0.0f, n, st); }
extern "C" int tosk_vadd(float* d, const float* s, int n, cudaStream_t st) { return ew(EW_VADD, d, s, 0.0f, n, st); }
extern "C" int tosk_vmul(float* d, const float* s, int n, cudaStream_t st) { return ew(EW_VMUL, d, s, 0.0f, n, st); }
extern "C" int tosk_axpy(float* d, float sc, const float* s, int n, cudaStream_t st) {
  return ew(EW_AXPY, d, s, sc, n, st);
}

extern "C" int tosk_dot(const float* a, const float* b, int n, float* out, cudaStream_t st) {
  dot_kernel<<<1, 32, 0, st>>>(a, b, n, out);
  return (int)cudaGetLastError();
}

extern "C" int tosk_embed(float* out, const void* embd, int type, int dim, const int* tok_dev, int tok,
                          int pdl, cudaStream_t st) {
  if (dim <= 0) return 0;
  int grid = (dim + 255) / 256;
  void* args[] = {&out, &embd, &type, &dim, &tok_dev, &tok};
  return launch_pdl((const void*)embed_kernel, dim3(grid), dim3(256), args, pdl, st);
}

extern "C" int tosk_argmax(const float* x, int n, int* out_idx, float* out_val, int pdl, cudaStream_t st) {
  if (n <= 0) return (int)cudaErrorInvalidValue;
  int first_rule = 1, offset = 0;
  void* args[] = {&x, &n, &out_idx, &out_val, &first_rule, &offset};
  return launch_pdl((const void*)argmax_kernel, dim3(1), dim3(1024), args, pdl, st);
}

extern "C" int tosk_sample(const float* x, int n, float temperature, uint32_t entropy, int* out_idx,
                           cudaStream_t st) {
  if (n <= 0 || !x || !out_idx) return (int)cudaErrorInvalidValue;
  if (temperature <= 0.001f) return tosk_argmax(x, n, out_idx, nullptr, 0, st);   // llm.c:1179-1180
  void* args[] = {&x, &n, &temperature, &entropy, &out_idx};
  return launch_pdl((const void*)sample_kernel, dim3(1), dim3(1024), args, 0, st);
}

extern "C" int tosk_argmax_rows(const float* x, int n, int rows, int* out_idx, cudaStream_t st) {
  if (n <= 0 || rows <= 0) return (int)cudaErrorInvalidValue;
  int first_rule = 1, offset = 0;
  float* out_val = nullptr;
  void* args[] = {&x, &n, &out_idx, &out_val, &first_rule, &offset};
  return launch_pdl((const void*)argmax_kernel, dim3(rows), dim3(1024), args, 1, st);
}

extern "C" int tosk_argmax_slice(const float* x, int n, int offset, int first_rule, int* pair, int pdl,
                                 cudaStream_t st) {
  if (n <= 0 || !pair) return (int)cudaErrorInvalidValue;
  int* out_idx = pair + 1;
  float* out_val = reinterpret_cast<float*>(pair);
  void* args[] = {&x, &n, &out_idx, &out_val, &first_rule, &offset};
  return launch_pdl((const void*)argmax_kernel, dim3(1), dim3(1024), args, pdl, st);
}

extern "C" int tosk_argmax_pairs(const int* pairs, int world, int* out_idx, int pdl, cudaStream_t st) {
  if (world <= 0) return (int)cudaErrorInvalidValue;
  void* args[] = {&pairs, &world, &out_idx};
  return launch_pdl((const void*)argmax_pairs_kernel, dim3(1), dim3(32), args, pdl, st);
}

extern "C" int tosk_decode_advance(int* io, int* ring, int pdl, cudaStream_t st) {
  void* args[] = {&io, &ring};
  return launch_pdl((const void*)decode_advance_kernel, dim3(1), dim3(1), args, pdl, st);
}
