// attention.cu - single-query decode attention over the KV cache
// (runtime/nn/llm.c:683-714), fp32 or fp16 cache laid out [pos][n_kv*hd].
//
// Reference order, per query head h (kv head kvh = h / (n_heads/n_kv)):
//   score[t] = llm_dot_f32(q_h, K[t][kvh]) * (1/sqrt(hd))      t = 0..pos
//   llm_softmax(score, pos+1): max, e_t = llm_expf(s_t - max), serial sum,
//     inv = 1/(sum + 1e-10), p_t = e_t * inv
//   head[d] = 0; for t: head[d] = head[d] + p_t * V[t][kvh][d]   (serial in t)
//
// EXACT mode keeps every reference rounding:
//   scores_kernel  - persistent CTAs over (kv head, 128-position tile); the K
//                    tile is staged in shared memory (padded rows) and each
//                    thread forms one exact 8-chain dot per query head of the
//                    group.  Fully parallel, HBM-bound.
//   softmax_pv_kernel - one warp per (head, 64-wide slice of d): max over the
//                    scores, e_t in parallel, the serial sum in lane 0, p_t in
//                    parallel, then the serial PV chain with each lane owning
//                    two d (packed f32x2).  V rows stream through a cp.async
//                    ring.  The chains are the bound: ~4-5 cycles per position.
// FAST mode is a split-K flash-decoding pass in two kernels over 64-position
// chunks: fast_scores_kernel (a warp per 16 positions with all 16 rows in
// flight, lanes across d, one shuffle reduce-scatter per 16 dots) writes the
// scores and per-chunk maxima; fast_pv_kernel forms e_t = llm_expf(s_t - global max) (the
// reference's exponential of the same argument), the chunk's e-sum and
// sum_t e_t v_t, and the last chunk of each head to finish (a counter per
// head) adds the chunks in order and divides.  Only summation order and
// the place of the 1/sum differ from the reference (tolerance 1e-4).
#include <cuda_runtime.h>

#include <mutex>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

constexpr int kScoreTile = 128;
constexpr int kPvRows = 64;     // rows per V stage
constexpr int kPvStages = 4;
constexpr int kFChunk = 64;     // positions per FAST chunk
constexpr int kFThreads = 128;  // FAST CTAs: 4 warps x 16 positions
constexpr int kFMaxHd = 256;

template <int ESZ>
__device__ __forceinline__ void load8(const uint8_t* p, float2 (&v)[4]) {
  if constexpr (ESZ == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    v[0] = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    v[1] = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[2] = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
    v[3] = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
  } else {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 16);
    v[0] = make_float2(a.x, a.y);
    v[1] = make_float2(a.z, a.w);
    v[2] = make_float2(b.x, b.y);
    v[3] = make_float2(b.z, b.w);
  }
}

template <int ESZ>
__device__ __forceinline__ float load1(const uint8_t* p) {
  if constexpr (ESZ == 2) return h2f(*reinterpret_cast<const uint16_t*>(p));
  return *reinterpret_cast<const float*>(p);
}

// ---------------------------------------------------------------------------
// scores
// ---------------------------------------------------------------------------
template <int ESZ>
__global__ void __launch_bounds__(kScoreTile) scores_kernel(const float* __restrict__ q,
                                                            const uint8_t* __restrict__ kc,
                                                            int n_heads, int n_kv, int hd,
                                                            const int* __restrict__ pos_dev,
                                                            int pos_arg, float* __restrict__ S,
                                                            int max_ctx) {
  extern __shared__ __align__(16) uint8_t sm[];
  pdl_wait();
  pdl_trigger();
  const int n = (pos_dev ? *pos_dev : pos_arg) + 1;
  const int group = n_heads / n_kv;
  const int kv_dim = n_kv * hd;
  const int rowb = hd * ESZ;           // bytes of one K row slice
  const int strideb = rowb + 16;       // padded to spread banks
  float* qs = reinterpret_cast<float*>(sm);
  uint8_t* ks = sm + ((group * hd * 4 + 15) & ~15);
  const int ntile = (n + kScoreTile - 1) / kScoreTile;
  const int items = n_kv * ntile;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const int hd8 = hd & ~7;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int kvh = item / ntile;
    const int t0 = (item % ntile) * kScoreTile;
    const int rows = min(kScoreTile, n - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < group * hd; i += blockDim.x) qs[i] = q[(size_t)kvh * group * hd + i];
    const int cpr = rowb / 16;  // 16-byte chunks per row (hd*ESZ is a multiple of 16)
    for (int c = threadIdx.x; c < rows * cpr; c += blockDim.x) {
      const int r = c / cpr, k = c % cpr;
      const uint4 v =
          *reinterpret_cast<const uint4*>(kc + ((size_t)(t0 + r) * kv_dim + (size_t)kvh * hd) * ESZ + k * 16);
      *reinterpret_cast<uint4*>(ks + r * strideb + k * 16) = v;
    }
    __syncthreads();
    const int r = threadIdx.x;
    if (r < rows) {
      const uint8_t* kr = ks + r * strideb;
      for (int g = 0; g < group; ++g) {
        const float* qh = qs + g * hd;
        float2 acc[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[p] = make_float2(0.0f, 0.0f);
        for (int m = 0; m < hd8; m += 8) {
          float2 kv[4];
          load8<ESZ>(kr + m * ESZ, kv);
#pragma unroll
          for (int p = 0; p < 4; ++p)
            acc[p] = __fadd2_rn(acc[p], mul2_rn(make_float2(qh[m + 2 * p], qh[m + 2 * p + 1]), kv[p]));
        }
        const float2 t01 = __fadd2_rn(acc[0], acc[2]);
        const float2 t23 = __fadd2_rn(acc[1], acc[3]);
        float sum = __fadd_rn(__fadd_rn(__fadd_rn(t01.x, t01.y), t23.x), t23.y);
        for (int i = hd8; i < hd; ++i) sum = __fadd_rn(sum, __fmul_rn(qh[i], load1<ESZ>(kr + i * ESZ)));
        S[(size_t)(kvh * group + g) * max_ctx + t0 + r] = __fmul_rn(sum, scale);
      }
    }
  }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streams V rows [t_begin, t_end) of this warp's slice through the ring and
// accumulates acc += p_t * v_t (serial in t).  P holds p indexed by t.
template <int ESZ>
__device__ __forceinline__ float2 pv_chain(const uint8_t* __restrict__ vbase, size_t row_stride_b,
                                           int slice_b, const float* __restrict__ P, int p_off,
                                           int t_begin, int t_end, uint8_t* ring, int lane, bool active,
                                           float2 acc) {
  const int cpr = slice_b / 16;
  const int stage_b = kPvRows * slice_b;
  const int nrows = t_end - t_begin;
  const int nst = (nrows + kPvRows - 1) / kPvRows;
  auto issue = [&](int s) {
    if (s < nst) {
      const int r0 = t_begin + s * kPvRows;
      const int rows = min(kPvRows, t_end - r0);
      uint8_t* dst = ring + (s % kPvStages) * stage_b;
      for (int c = lane; c < rows * cpr; c += 32) {
        const int r = c / cpr, k = c % cpr;
        cp_async16(dst + r * slice_b + k * 16, vbase + (size_t)(r0 + r) * row_stride_b + k * 16);
      }
    }
    cp_commit();
  };
#pragma unroll
  for (int s = 0; s < kPvStages - 1; ++s) issue(s);
  for (int s = 0; s < nst; ++s) {
    issue(s + kPvStages - 1);
    cp_wait<kPvStages - 1>();
    __syncwarp();
    const uint8_t* buf = ring + (s % kPvStages) * stage_b;
    const int r0 = t_begin + s * kPvRows;
    const int rows = min(kPvRows, t_end - r0);
    if (active) {
      for (int r = 0; r < rows; ++r) {
        const float p = P[r0 + r - p_off];
        float2 v;
        if constexpr (ESZ == 2)
          v = __half22float2(*reinterpret_cast<const __half2*>(buf + r * slice_b + lane * 4));
        else
          v = *reinterpret_cast<const float2*>(buf + r * slice_b + lane * 8);
        acc = __fadd2_rn(acc, mul2_rn(make_float2(p, p), v));   // llm.c:586-588
      }
    }
    __syncwarp();
  }
  cp_wait<0>();
  return acc;
}

template <int ESZ>
__global__ void __launch_bounds__(32) softmax_pv_kernel(const float* __restrict__ S,
                                                        const uint8_t* __restrict__ vc, int n_heads,
                                                        int n_kv, int hd, const int* __restrict__ pos_dev,
                                                        int pos_arg, int max_ctx, float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t sm[];
  float* P = reinterpret_cast<float*>(sm);
  uint8_t* ring = sm + (((size_t)max_ctx * 4 + 15) & ~(size_t)15);
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x;
  const int ngr = (hd + 63) / 64;
  const int h = blockIdx.x / ngr, g = blockIdx.x % ngr;
  const int kvh = h / (n_heads / n_kv);
  const int n = (pos_dev ? *pos_dev : pos_arg) + 1;
  const float* Sh = S + (size_t)h * max_ctx;
  // llm.c:509-511: max
  float m = -INFINITY;
  for (int t = lane; t < n; t += 32) m = fmaxf(m, Sh[t]);
  m = warp_max(m);
  // llm.c:514-517: e_t (parallel), then the serial sum in lane 0
  for (int t = lane; t < n; t += 32) P[t] = ref_expf(__fsub_rn(Sh[t], m));
  __syncwarp();
  float inv = 0.0f;
  if (lane == 0) {
    float sum = 0.0f;
    int t = 0;
    for (; t + 4 <= n; t += 4) {
      const float4 e = *reinterpret_cast<const float4*>(P + t);
      sum = __fadd_rn(sum, e.x);
      sum = __fadd_rn(sum, e.y);
      sum = __fadd_rn(sum, e.z);
      sum = __fadd_rn(sum, e.w);
    }
    for (; t < n; ++t) sum = __fadd_rn(sum, P[t]);
    inv = __fdiv_rn(1.0f, __fadd_rn(sum, 1e-10f));
  }
  inv = __shfl_sync(0xffffffffu, inv, 0);
  for (int t = lane; t < n; t += 32) P[t] = __fmul_rn(P[t], inv);
  __syncwarp();
  // llm.c:703-709: serial PV chain
  const int d0 = 64 * g;
  const int slice = min(64, hd - d0);
  const bool active = 2 * lane < slice;
  const int kv_dim = n_kv * hd;
  const uint8_t* vbase = vc + ((size_t)kvh * hd + d0) * ESZ;
  float2 acc = pv_chain<ESZ>(vbase, (size_t)kv_dim * ESZ, slice * ESZ, P, 0, 0, n, ring, lane, active,
                             make_float2(0.0f, 0.0f));
  if (active) {
    out[(size_t)h * hd + d0 + 2 * lane] = acc.x;
    out[(size_t)h * hd + d0 + 2 * lane + 1] = acc.y;
  }
}

// ---------------------------------------------------------------------------
// FAST mode.  Workspace: S[n_heads][max_ctx] | cmax[n_heads][maxc] |
// lsum[n_heads][maxc] | opart[n_heads][maxc][kFMaxHd] | cnt[n_heads] (int).
// ---------------------------------------------------------------------------
// Four consecutive cache elements (8 bytes of fp16 or 16 of fp32) as floats.
template <int ESZ>
__device__ __forceinline__ float4 load4(const uint8_t* p) {
  if constexpr (ESZ == 2) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  } else {
    return *reinterpret_cast<const float4*>(p);
  }
}

// Four cache elements as loaded (fp16: two packed words, half the registers
// of four floats, so more rows stay in flight per SM) and as floats.
template <int ESZ> struct RawT { using type = float4; };
template <> struct RawT<2> { using type = uint2; };
template <int ESZ>
__device__ __forceinline__ typename RawT<ESZ>::type ldraw(const uint8_t* p) {
  return *reinterpret_cast<const typename RawT<ESZ>::type*>(p);
}
template <int ESZ>
__device__ __forceinline__ float4 unraw(typename RawT<ESZ>::type r) {
  if constexpr (ESZ == 2) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  } else {
    return r;
  }
}

// Lane l covers d = 128 s + 4 l .. +3 for slabs s < ceil(hd / 128).
constexpr int kFSlabs = kFMaxHd / 128;

template <int ESZ>
__global__ void __launch_bounds__(kFThreads, 8) fast_scores_kernel(
    const float* __restrict__ q, const uint8_t* __restrict__ kc, int n_heads, int n_kv, int hd,
    const int* __restrict__ pos_dev, int pos_arg, float* __restrict__ S, float* __restrict__ cmax,
    int* __restrict__ cnt, int max_ctx, int maxc) {
  __shared__ float wmax[kFThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int n = (pos_dev ? *pos_dev : pos_arg) + 1;
  if (blockIdx.x == 0)
    for (int h = threadIdx.x; h < n_heads; h += blockDim.x) cnt[h] = 0;   // fast_pv_kernel's counters
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = n_heads / n_kv;
  const int kv_dim = n_kv * hd;
  const int nchunk = (n + kFChunk - 1) / kFChunk;
  const int items = n_kv * nchunk;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    // kv head fastest: the CTAs that run together read every head of the
    // same positions, i.e. whole cache rows
    const int kvh = item % n_kv, c = item / n_kv;
    const int tw = c * kFChunk + warp * 16;   // this warp's first position
    for (int g = 0; g < group; ++g) {
      const int h = kvh * group + g;
      float v[16];
#pragma unroll
      for (int p = 0; p < 16; ++p) v[p] = 0.0f;
#pragma unroll 1
      for (int sl = 0; sl < kFSlabs; ++sl) {
        const int d = 128 * sl + 4 * lane;
        if (d < hd) {
          const float4 qv = *reinterpret_cast<const float4*>(q + (size_t)h * hd + d);
          typename RawT<ESZ>::type kr[16];
#pragma unroll
          for (int p = 0; p < 16; ++p)   // all 16 rows in flight at once
            kr[p] = tw + p < n ? ldraw<ESZ>(kc + ((size_t)(tw + p) * kv_dim + (size_t)kvh * hd + d) * ESZ)
                               : typename RawT<ESZ>::type{};
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            const float4 kv = unraw<ESZ>(kr[p]);
            v[p] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, v[p]))));
          }
        }
      }
      // reduce-scatter: after the steps over lane bits 4..1, lane l holds
      // position l >> 1 summed over 16 lanes; bit 0 finishes the sum
#pragma unroll
      for (int half = 8, o = 16; half >= 1; half >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float keep = up ? v[half + i] : v[i];
          const float send = up ? v[i] : v[half + i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      const float dot = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
      const int t = tw + (lane >> 1);
      const float sc = dot * scale;
      float m = -INFINITY;
      if (t < n) {
        m = sc;
        if ((lane & 1) == 0) S[(size_t)h * max_ctx + t] = sc;
      }
      m = warp_max(m);
      __syncthreads();
      if (lane == 0) wmax[warp] = m;
      __syncthreads();
      if (threadIdx.x == 0) {
        float cm = wmax[0];
        for (int w = 1; w < kFThreads / 32; ++w) cm = fmaxf(cm, wmax[w]);
        cmax[(size_t)h * maxc + c] = cm;
      }
    }
  }
}

template <int ESZ>
__global__ void __launch_bounds__(kFThreads, 8) fast_pv_kernel(
    const float* __restrict__ S, const float* __restrict__ cmax, const uint8_t* __restrict__ vc, int n_heads,
    int n_kv, int hd, const int* __restrict__ pos_dev, int pos_arg, float* __restrict__ lsum,
    float* __restrict__ opart, int* __restrict__ cnt, float* __restrict__ out, int max_ctx, int maxc) {
  __shared__ float es[kFChunk];
  __shared__ float red[kFThreads / 32];
  __shared__ __align__(16) float wpart[kFThreads / 32][kFMaxHd];
  __shared__ int s_last;
  pdl_wait();
  pdl_trigger();
  const int n = (pos_dev ? *pos_dev : pos_arg) + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = n_heads / n_kv;
  const int kv_dim = n_kv * hd;
  const int nchunk = (n + kFChunk - 1) / kFChunk;
  const int items = n_heads * nchunk;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int h = item % n_heads, c = item / n_heads;   // head fastest (whole cache rows together)
    const int kvh = h / group;
    const int t0 = c * kFChunk, cn = min(kFChunk, n - t0);
    // global max of the head's scores (llm.c:509-511) from the chunk maxima
    float m = -INFINITY;
    for (int i = threadIdx.x; i < nchunk; i += blockDim.x) m = fmaxf(m, cmax[(size_t)h * maxc + i]);
    m = warp_max(m);
    __syncthreads();
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float M = red[0];
    for (int w = 1; w < kFThreads / 32; ++w) M = fmaxf(M, red[w]);
    // e_t = llm_expf(s_t - max) (llm.c:514-517) and the chunk's e-sum
    float e = 0.0f;
    if (threadIdx.x < kFChunk) {
      if (threadIdx.x < cn) e = ref_expf(__fsub_rn(S[(size_t)h * max_ctx + t0 + threadIdx.x], M));
      es[threadIdx.x] = e;
    }
    float l = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    __syncthreads();
    if (lane == 0) red[warp] = l;
    // sum_t e_t v_t[d]: warp w takes 16 positions, lane l four consecutive d
    const int tw = warp * 16;
#pragma unroll 1
    for (int sl = 0; sl < kFSlabs; ++sl) {
      const int d = 128 * sl + 4 * lane;
      if (d < hd) {
        typename RawT<ESZ>::type vr[16];
#pragma unroll
        for (int p = 0; p < 16; ++p)   // all 16 rows in flight at once
          vr[p] = tw + p < cn ? ldraw<ESZ>(vc + ((size_t)(t0 + tw + p) * kv_dim + (size_t)kvh * hd + d) * ESZ)
                              : typename RawT<ESZ>::type{};
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float ep = es[tw + p];
          const float4 vv = unraw<ESZ>(vr[p]);
          acc.x = fmaf(ep, vv.x, acc.x);
          acc.y = fmaf(ep, vv.y, acc.y);
          acc.z = fmaf(ep, vv.z, acc.z);
          acc.w = fmaf(ep, vv.w, acc.w);
        }
        *reinterpret_cast<float4*>(&wpart[warp][d]) = acc;
      }
    }
    __syncthreads();
    float* op = opart + ((size_t)h * maxc + c) * kFMaxHd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      float o = wpart[0][d];
      for (int w = 1; w < kFThreads / 32; ++w) o += wpart[w][d];
      op[d] = o;
    }
    if (threadIdx.x == 0) {
      float lc = red[0];
      for (int w = 1; w < kFThreads / 32; ++w) lc += red[w];
      lsum[(size_t)h * maxc + c] = lc;
    }
    // the last chunk of the head to finish combines (chunk order, so the
    // result does not depend on which CTA that is)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&cnt[h], 1) == nchunk - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      // chunk order, eight chunks' loads in flight (L2: written by other CTAs)
      const float* ls = lsum + (size_t)h * maxc;
      const float* op = opart + (size_t)h * maxc * kFMaxHd;
      float L = 0.0f;
      for (int i0 = 0; i0 < nchunk; i0 += 8) {
        float lv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) lv[k] = i0 + k < nchunk ? __ldcg(ls + i0 + k) : 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (i0 + k < nchunk) L += lv[k];
      }
      const float inv = 1.0f / (L + 1e-10f);   // llm.c:519
      for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
        for (int i0 = 0; i0 < nchunk; i0 += 8) {
          float ov[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) ov[k] = i0 + k < nchunk ? __ldcg(op + (size_t)(i0 + k) * kFMaxHd + d) : 0.0f;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (i0 + k < nchunk) o += ov[k];
        }
        out[(size_t)h * hd + d] = o * inv;
      }
    }
  }
}

}  // namespace tos

using namespace tos;

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

extern "C" size_t tosk_attention_ws_bytes(int n_heads, int max_ctx) {
  const size_t maxc = (size_t)(max_ctx + kFChunk - 1) / kFChunk;
  return align256((size_t)n_heads * max_ctx * 4) + 2 * align256((size_t)n_heads * maxc * 4) +
         align256((size_t)n_heads * maxc * kFMaxHd * 4) + align256((size_t)n_heads * 4);
}

// Raises a kernel's dynamic shared-memory limit to the sm_100 maximum once
// (not inside stream capture: the first call of every launcher is eager).
static int allow_max_smem(const void* kern) {
  static const void* done[16];
  static int n_done = 0;
  for (int i = 0; i < n_done; ++i)
    if (done[i] == kern) return 0;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return (int)e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           227 * 1024 - (int)fa.sharedSizeBytes);
  if (e != cudaSuccess) return (int)e;
  if (n_done < 16) done[n_done++] = kern;
  return 0;
}

template <typename K>
static int launch_k(K kern, int grid, int threads, size_t smem, int pdl, cudaStream_t st, void** args) {
  int e0 = allow_max_smem((const void*)kern);
  if (e0) return e0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return (int)cudaLaunchKernelExC(&cfg, (const void*)kern, args);
}

// FAST mode (split-K flash decoding): scores + chunk maxima, then e_t, the
// chunk partials and the per-head combine by the last chunk to finish.
static int fast_attention(float* out, const float* q, const uint8_t* kc, const uint8_t* vc, int esz,
                          int n_heads, int n_kv, int hd, const int* pos_dev, int pos, int max_ctx, void* ws,
                          int pdl, cudaStream_t st) {
  // four consecutive elements per lane: hd a multiple of 4, rows 16-byte aligned
  if (hd > kFMaxHd || hd % 4 != 0 || (reinterpret_cast<uintptr_t>(kc) & 15) || (reinterpret_cast<uintptr_t>(vc) & 15) ||
      (reinterpret_cast<uintptr_t>(q) & 15))
    return (int)cudaErrorInvalidValue;
  const int maxc = (max_ctx + kFChunk - 1) / kFChunk;
  float* S = (float*)ws;
  float* cmax = (float*)((char*)S + align256((size_t)n_heads * max_ctx * 4));
  float* lsum = (float*)((char*)cmax + align256((size_t)n_heads * maxc * 4));
  float* opart = (float*)((char*)lsum + align256((size_t)n_heads * maxc * 4));
  int* cnt = (int*)((char*)opart + align256((size_t)n_heads * maxc * kFMaxHd * 4));
  const int cap = tosk_num_sms() * 8;
  {
    int grid = n_kv * maxc;
    if (grid > cap) grid = cap;
    void* args[] = {(void*)&q, (void*)&kc, &n_heads, &n_kv, &hd, (void*)&pos_dev, &pos, &S, &cmax, &cnt, &max_ctx, (void*)&maxc};
    int e = esz == 2 ? launch_k(fast_scores_kernel<2>, grid, kFThreads, 0, pdl, st, args)
                     : launch_k(fast_scores_kernel<4>, grid, kFThreads, 0, pdl, st, args);
    if (e) return e;
  }
  int grid = n_heads * maxc;
  if (grid > cap) grid = cap;
  void* args[] = {&S, &cmax, (void*)&vc, &n_heads, &n_kv, &hd, (void*)&pos_dev, &pos, &lsum, &opart, &cnt, &out, &max_ctx, (void*)&maxc};
  return esz == 2 ? launch_k(fast_pv_kernel<2>, grid, kFThreads, 0, pdl, st, args)
                  : launch_k(fast_pv_kernel<4>, grid, kFThreads, 0, pdl, st, args);
}

extern "C" int tosk_attention(float* out, const float* q, const void* k_cache, const void* v_cache,
                              int kv_type, int n_heads, int n_kv, int hd, const int* pos_dev, int pos,
                              int max_ctx, int mode, void* ws, size_t ws_bytes, int* err, int pdl,
                              cudaStream_t st) {
  (void)err;
  if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv != 0 || hd <= 0 || max_ctx <= 0) return (int)cudaErrorInvalidValue;
  if (kv_type != TOSK_F16 && kv_type != TOSK_F32) return (int)cudaErrorInvalidValue;
  const int esz = kv_type == TOSK_F16 ? 2 : 4;
  if ((hd * esz) % 16 != 0 || hd % 2 != 0) return (int)cudaErrorInvalidValue;
  if (ws_bytes < tosk_attention_ws_bytes(n_heads, max_ctx)) return (int)cudaErrorInvalidValue;
  if (!pos_dev && (pos < 0 || pos >= max_ctx)) return (int)cudaErrorInvalidValue;
  if (mode == TOSK_ATTN_FAST)
    return fast_attention(out, q, (const uint8_t*)k_cache, (const uint8_t*)v_cache, esz, n_heads, n_kv, hd,
                          pos_dev, pos, max_ctx, ws, pdl, st);
  if (mode != TOSK_ATTN_EXACT) return (int)cudaErrorInvalidValue;
  float* S = (float*)ws;
  const int group = n_heads / n_kv;
  // scores
  {
    const size_t smem = ((size_t)group * hd * 4 + 15) / 16 * 16 + (size_t)kScoreTile * (hd * esz + 16);
    if (smem > 227 * 1024) return (int)cudaErrorInvalidValue;
    const int tiles = (max_ctx + kScoreTile - 1) / kScoreTile;
    int grid = n_kv * tiles;
    const int cap = tosk_num_sms() * 4;
    if (grid > cap) grid = cap;
    const uint8_t* kc = (const uint8_t*)k_cache;
    void* args[] = {(void*)&q, (void*)&kc, &n_heads, &n_kv, &hd, (void*)&pos_dev, &pos, &S, &max_ctx};
    int e = esz == 2 ? launch_k(scores_kernel<2>, grid, kScoreTile, smem, pdl, st, args)
                     : launch_k(scores_kernel<4>, grid, kScoreTile, smem, pdl, st, args);
    if (e) return e;
  }
  const int ngr = (hd + 63) / 64;
  const uint8_t* vc = (const uint8_t*)v_cache;
  if (mode == TOSK_ATTN_EXACT) {
    const size_t ring = (size_t)kPvStages * kPvRows * 64 * esz;
    const size_t smem = (((size_t)max_ctx * 4 + 15) & ~(size_t)15) + ring;
    if (smem > 227 * 1024) return (int)cudaErrorInvalidValue;
    void* args[] = {&S, (void*)&vc, &n_heads, &n_kv, &hd, (void*)&pos_dev, &pos, &max_ctx, &out};
    return esz == 2 ? launch_k(softmax_pv_kernel<2>, n_heads * ngr, 32, smem, pdl, st, args)
                    : launch_k(softmax_pv_kernel<4>, n_heads * ngr, 32, smem, pdl, st, args);
  }
  return 0;
}



// ---------------------------------------------------------------------------
// Allocation-free entry point
//
// The decode path this library replaces keeps all of its scratch in static
// buffers and never allocates while it runs (runtime/nn/llm.c:48-65): it is
// meant for callers such as a kernel-mode or real-time inference loop, or a
// host whose device memory is owned by another allocator, that cannot call
// cudaMalloc in the middle of a step.  tos_attention_noalloc_dev serves them:
// it runs the same attention kernels as tos_attention_dev with the workspace
// taken from a file-scope device array instead of caller-provided memory.
//
//  * The array holds kNoAllocScratchBytes (4 MiB) on every GPU that loads
//    this library, for the life of the process.  A configuration whose
//    workspace (tos_attention_workspace_bytes(n_heads, max_ctx)) is larger
//    is rejected with TOS_ENOMEM before any work is queued.
//  * The first call on a device resolves the array's device address with
//    cudaGetSymbolAddress while that device is current (once per device,
//    std::call_once, so concurrent first calls are safe); make that first
//    call before any stream capture.  A cudaDeviceReset destroys every device
//    object this library holds on that device (its stream, registered
//    weights, models and this address alike): call tos_shutdown first and do
//    not use the library on that device afterwards.
//  * Every call shares the one array.  Nothing in it has to start at zero:
//    each call writes every workspace element before reading it.  Calls that
//    overlap on the GPU (different streams, or concurrent host threads) race
//    on the array and must be serialised by the caller.
//  * Nothing here allocates: no cudaMalloc/cudaFree and no library routine
//    that allocates; the library stream and error word are not touched.
// ---------------------------------------------------------------------------
namespace tos {
constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
}  // namespace tos

static constexpr int kNoAllocMaxDevices = 64;
static std::once_flag g_noalloc_once[kNoAllocMaxDevices];
static void* g_noalloc_ptr[kNoAllocMaxDevices];
static cudaError_t g_noalloc_status[kNoAllocMaxDevices];

extern "C" int tos_attention_noalloc_dev(float* out, const float* q, const void* k_cache, const void* v_cache,
                                         int kv_type, int n_heads, int n_kv, int head_dim, int pos, int max_ctx,
                                         int mode, void* stream) {
  // status values of include/tensoros_nn_gpu.h
  const int kOk = 0, kInval = -1, kNoMem = -2, kCuda = -3, kNoDev = -7;
  if (!out || !q || !k_cache || !v_cache) return kInval;
  if (n_heads <= 0 || n_kv <= 0 || head_dim <= 0 || max_ctx <= 0 || pos < 0 || pos >= max_ctx) return kInval;
  if (mode != TOSK_ATTN_EXACT && mode != TOSK_ATTN_FAST) return kInval;
  const size_t need = tosk_attention_ws_bytes(n_heads, max_ctx);
  if (need > tos::kNoAllocScratchBytes) return kNoMem;   // beyond the static scratch
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kNoDev;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return kInval;
  // the array's address on this device (the symbol's host-side name is not a
  // device address), resolved once with this device current
  std::call_once(g_noalloc_once[dev], [dev] {
    void* p = nullptr;
    g_noalloc_status[dev] = cudaGetSymbolAddress(&p, tos::g_noalloc_scratch);
    g_noalloc_ptr[dev] = g_noalloc_status[dev] == cudaSuccess ? p : nullptr;
  });
  if (g_noalloc_status[dev] != cudaSuccess || g_noalloc_ptr[dev] == nullptr) return kCuda;
  const int e = tosk_attention(out, q, k_cache, v_cache, kv_type, n_heads, n_kv, head_dim, nullptr, pos, max_ctx,
                               mode, g_noalloc_ptr[dev], tos::kNoAllocScratchBytes, nullptr, 0,
                               (cudaStream_t)stream);
  if (e == cudaSuccess) return kOk;
  return e == cudaErrorInvalidValue ? kInval : kCuda;
}
