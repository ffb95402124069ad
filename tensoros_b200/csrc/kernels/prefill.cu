// prefill.cu - per-token kernels of the batched prompt pass (prefill): the
// projections run as tensor-core GEMMs (gemm_tc.cu); these kernels do the
// row-wise work between them for n tokens at positions pos0 .. pos0+n-1
// (the RMSNorms run inside the GEMMs' activation prep, gemm_tc.cu).
// Reference: llm_forward_token per token (runtime/nn/llm.c:641-743).
//   pf_embed_kernel      llm_embed (llm.c:365-410), one CTA per token
//   pf_rope_store_kernel RoPE of q and k (llm.c:460-500, table of the decode
//                        path) and the K/V cache store (llm.c:673-681)
//   pf_attention_kernel  causal single-query attention of every token over
//                        the cache (llm.c:683-714) with llm_expf weights,
//                        tree sums (FAST numerics); for an fp16 cache and
//                        head dimension 128 the prompt pass uses
//                        pf_attention_tile_kernel (16 tokens of a head per
//                        CTA, each K / V row read once per tile)
// The residual adds (llm.c:718, 733) and SiLU(gate)*up (llm.c:726-729) run
// in the GEMMs' epilogues.
// The rope/store and attention kernels also serve batched decode: n tokens
// of n different sequences, each at its own position with its own cache.
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

__device__ __forceinline__ float embed_elem(const uint8_t* embd, int type, int dim, int tok, int i) {
  if (type == TOSK_Q4_0) {
    const uint8_t* blk = embd + ((size_t)tok * (dim / 32) + i / 32) * 18;
    const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    const int j = i & 31;
    const uint8_t byte = blk[2 + (j >> 1)];
    return __fmul_rn((float)(((j & 1) ? (byte >> 4) : (byte & 0x0F)) - 8), d);
  }
  if (type == TOSK_Q8_0) {
    const uint8_t* blk = embd + ((size_t)tok * (dim / 32) + i / 32) * 34;
    return __fmul_rn((float)(int8_t)blk[2 + (i & 31)], h2f((uint16_t)(blk[0] | (blk[1] << 8))));
  }
  if (type == TOSK_F16) return h2f(reinterpret_cast<const uint16_t*>(embd)[(size_t)tok * dim + i]);
  return reinterpret_cast<const float*>(embd)[(size_t)tok * dim + i];
}

__global__ void pf_embed_kernel(float* __restrict__ x, const uint8_t* __restrict__ embd, int type, int dim,
                                const int* __restrict__ toks) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int tok = toks[t];
  for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)t * dim + i] = embed_elem(embd, type, dim, tok, i);
}

constexpr int kRopeRows = 1024;   // rows of one token per CTA

// qkv rows [q_rows | kv_rows | kv_rows] per token; q (roped) -> q_out,
// k (roped) and v -> the caches at position pos0 + t.
// Batched decode (pos_arr non-null): row t is a token of sequence slot[t]
// at position pos_arr[t]; slot s's cache starts s*cstride elements in.
__global__ void pf_rope_store_kernel(const float* __restrict__ qkv, int q_rows, int kv_rows, int hd,
                                     const float2* __restrict__ cs, int pos0, float* __restrict__ q_out,
                                     void* __restrict__ kc, void* __restrict__ vc, int kv_type,
                                     const int* __restrict__ pos_arr, const int* __restrict__ slot,
                                     size_t cstride) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int pos = pos_arr ? pos_arr[t] : pos0 + t;
  const size_t esz = kv_type == TOSK_F16 ? 2 : 4;
  if (pos_arr) {
    kc = reinterpret_cast<char*>(kc) + (size_t)slot[t] * cstride * esz;
    vc = reinterpret_cast<char*>(vc) + (size_t)slot[t] * cstride * esz;
  }
  const int nrow = q_rows + 2 * kv_rows;
  const float* row = qkv + (size_t)t * nrow;
  const int rend = min(nrow, (int)(blockIdx.y + 1) * kRopeRows);   // grid.y splits a token's rows
  for (int r = blockIdx.y * kRopeRows + threadIdx.x; r < rend; r += blockDim.x) {
    const float y = row[r];
    float v = y;
    if (r < q_rows + kv_rows) {
      const float partner = row[r ^ 1];
      const int i = (r < q_rows ? r : r - q_rows) % hd;
      const float2 c = cs[(size_t)pos * (hd >> 1) + (i >> 1)];
      v = (i & 1) == 0 ? __fsub_rn(__fmul_rn(y, c.x), __fmul_rn(partner, c.y))
                       : __fadd_rn(__fmul_rn(partner, c.y), __fmul_rn(y, c.x));
    }
    if (r < q_rows) {
      q_out[(size_t)t * q_rows + r] = v;
    } else {
      const bool is_k = r < q_rows + kv_rows;
      const int e = is_k ? r - q_rows : r - q_rows - kv_rows;
      void* cache = is_k ? kc : vc;
      const size_t idx = (size_t)pos * kv_rows + e;
      if (kv_type == TOSK_F16)
        reinterpret_cast<uint16_t*>(cache)[idx] = f2h(v);
      else
        reinterpret_cast<float*>(cache)[idx] = v;
    }
  }
}

__device__ __forceinline__ float kv_load(const void* c, int kv_type, size_t idx) {
  return kv_type == TOSK_F16 ? h2f(reinterpret_cast<const uint16_t*>(c)[idx])
                             : reinterpret_cast<const float*>(c)[idx];
}

// One CTA of kPfWarps warps per (head, token): scores over positions
// 0..pos0+t, llm_expf weights of (s - max), tree sums, sum_j e_j v_j /
// (sum_j e_j + 1e-10).
constexpr int kPfWarps = 8;
__global__ void __launch_bounds__(32 * kPfWarps) pf_attention_kernel(const float* __restrict__ q, const void* __restrict__ kc,
                                                           const void* __restrict__ vc, int kv_type, int n_heads,
                                                           int n_kv, int hd, int pos0, float* __restrict__ out,
                                                           const int* __restrict__ pos_arr,
                                                           const int* __restrict__ slot, size_t cstride) {
  extern __shared__ float sc[];   // [pos0 + n] scores, then weights
  __shared__ float red[kPfWarps];
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, t = blockIdx.y;
  const int n = (pos_arr ? pos_arr[t] : pos0 + t) + 1;
  if (pos_arr) {
    const size_t esz = kv_type == TOSK_F16 ? 2 : 4;
    kc = reinterpret_cast<const char*>(kc) + (size_t)slot[t] * cstride * esz;
    vc = reinterpret_cast<const char*>(vc) + (size_t)slot[t] * cstride * esz;
  }
  const int kvh = h / (n_heads / n_kv);
  const int kv_dim = n_kv * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qh = q + ((size_t)t * n_heads + h) * hd;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  if (kv_type == TOSK_F16 && hd % 32 == 0 && hd <= 256) {
    // 8 positions per warp step, 4 lanes a position, each lane a contiguous
    // quarter of the head in 16-byte loads; q from shared memory
    __shared__ float qsh[256];
    for (int d = threadIdx.x; d < hd; d += blockDim.x) qsh[d] = qh[d];
    __syncthreads();
    const int sub = lane & 3, dpl = hd >> 2;
    const float* qs = qsh + sub * dpl;
    for (int j0 = warp * 8; j0 < n; j0 += 8 * kPfWarps) {
      const int j = j0 + (lane >> 2);
      float acc = 0.0f;
      if (j < n) {
        const uint4* kr = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(kc) +
                                                         (size_t)j * kv_dim + (size_t)kvh * hd + sub * dpl);
        for (int v = 0; v < dpl / 8; ++v) {
          const uint4 w = kr[v];
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[e]));
            acc = fmaf(qs[8 * v + 2 * e], f.x, acc);
            acc = fmaf(qs[8 * v + 2 * e + 1], f.y, acc);
          }
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (sub == 0 && j < n) sc[j] = acc * scale;
    }
  } else {
    for (int j = warp; j < n; j += kPfWarps) {
      float acc = 0.0f;
      for (int d = lane; d < hd; d += 32) acc = fmaf(qh[d], kv_load(kc, kv_type, (size_t)j * kv_dim + (size_t)kvh * hd + d), acc);
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) sc[j] = acc * scale;
    }
  }
  __syncthreads();
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += blockDim.x) m = fmaxf(m, sc[j]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float M = red[0];
  for (int w = 1; w < kPfWarps; ++w) M = fmaxf(M, red[w]);
  __syncthreads();
  float l = 0.0f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float e = ref_expf(__fsub_rn(sc[j], M));   // llm.c:514-517
    sc[j] = e;
    l += e;
  }
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  float L = red[0];
  for (int w = 1; w < kPfWarps; ++w) L += red[w];
  const float inv = 1.0f / (L + 1e-10f);
  if (hd % 32 == 0 && hd <= 256) {
    // warp w takes positions 8 w .. 8 w + 7, then 8 kPfWarps further on
    // (eight V rows in flight); lane l covers d = 4 l .. 4 l + 3 (+ 128); the
    // warps' partial sums are added in warp order
    __shared__ float part[kPfWarps][256];
    const bool f16 = kv_type == TOSK_F16;
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int j0 = warp * 8; j0 < n; j0 += 8 * kPfWarps) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int d = 128 * s + 4 * lane;
        if (d < hd) {
          float4 v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const size_t idx = (size_t)(j0 + k) * kv_dim + (size_t)kvh * hd + d;
            if (j0 + k >= n) {
              v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            } else if (f16) {
              const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(vc) + idx);
              const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
              const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
              v[k] = make_float4(a.x, a.y, b.x, b.y);
            } else {
              v[k] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(vc) + idx);
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float e = j0 + k < n ? sc[j0 + k] : 0.0f;
            acc[s].x = fmaf(e, v[k].x, acc[s].x);
            acc[s].y = fmaf(e, v[k].y, acc[s].y);
            acc[s].z = fmaf(e, v[k].z, acc[s].z);
            acc[s].w = fmaf(e, v[k].w, acc[s].w);
          }
        }
      }
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int d = 128 * s + 4 * lane;
      if (d < hd) *reinterpret_cast<float4*>(&part[warp][d]) = acc[s];
    }
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      float o = part[0][d];
      for (int w = 1; w < kPfWarps; ++w) o += part[w][d];
      out[((size_t)t * n_heads + h) * hd + d] = o * inv;
    }
    return;
  }
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    // eight independent chains (eight V rows in flight), added in a fixed order
    float a[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const size_t col = (size_t)kvh * hd + d;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = kv_load(vc, kv_type, (size_t)(j + k) * kv_dim + col);
#pragma unroll
      for (int k = 0; k < 8; ++k) a[k] = fmaf(sc[j + k], v[k], a[k]);
    }
    for (; j < n; ++j) a[j & 7] = fmaf(sc[j], kv_load(vc, kv_type, (size_t)j * kv_dim + col), a[j & 7]);
    const float s = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    out[((size_t)t * n_heads + h) * hd + d] = s * inv;
  }
}


// Prefill attention, a tile of kTT consecutive tokens of one head per CTA
// (fp16 cache, head dimension 128): each K and V row of the head is read
// once per tile instead of once per token.  Same arithmetic as
// pf_attention_kernel: score = (q . k) * (1 / sqrt(hd)) over the token's
// positions 0..pos0+t, llm_expf(s - max) weights (llm.c:506-532, 683-714),
// sum_j e_j v_j / (sum_j e_j + 1e-10); only the fp32 summation orders differ
// (tree sums, FAST numerics).
//   scores: lane l of warp w takes position j = 32 (w + 8 i) + l and all kTT
//           tokens (q of the tile in shared memory, read as broadcasts);
//   softmax: warp w takes tokens 2w, 2w + 1;
//   softmax * V: warp w takes tokens 2w, 2w + 1, lane l dimensions 4l..4l+3.
constexpr int kTT = 16;
constexpr int kTHd = 128;
__global__ void __launch_bounds__(256) pf_attention_tile_kernel(const float* __restrict__ q,
                                                                const uint16_t* __restrict__ kc,
                                                                const uint16_t* __restrict__ vc, int n_heads,
                                                                int n_kv, int pos0, int n, float* __restrict__ out) {
  extern __shared__ float tsm[];
  float* qs = tsm;                  // [kTT][kTHd]
  float* sc = tsm + kTT * kTHd;     // [kTT][P]: scores, then weights
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, t0 = blockIdx.y * kTT;
  const int nt = min(kTT, n - t0);
  const int P = pos0 + t0 + nt;     // positions the tile's last token sees
  const int kvh = h / (n_heads / n_kv);
  const int kv_dim = n_kv * kTHd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)kTHd));
  for (int i = threadIdx.x; i < kTT * kTHd; i += blockDim.x) {
    const int tt = i / kTHd, d = i % kTHd;
    qs[i] = tt < nt ? q[((size_t)(t0 + tt) * n_heads + h) * kTHd + d] : 0.0f;
  }
  __syncthreads();
  for (int jb = 32 * warp; jb < P; jb += 32 * 8) {
    const int j = jb + lane;
    float acc[kTT];
#pragma unroll
    for (int tt = 0; tt < kTT; ++tt) acc[tt] = 0.0f;
    if (j < P) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (size_t)j * kv_dim + (size_t)kvh * kTHd);
#pragma unroll 2
      for (int v = 0; v < kTHd / 8; ++v) {
        const uint4 w = kr[v];
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[e]));
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int tt = 0; tt < kTT; ++tt) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + tt * kTHd + 8 * v);
          const float4 qb = *reinterpret_cast<const float4*>(qs + tt * kTHd + 8 * v + 4);
          float a = acc[tt];
          a = fmaf(qa.x, kf[0], a);
          a = fmaf(qa.y, kf[1], a);
          a = fmaf(qa.z, kf[2], a);
          a = fmaf(qa.w, kf[3], a);
          a = fmaf(qb.x, kf[4], a);
          a = fmaf(qb.y, kf[5], a);
          a = fmaf(qb.z, kf[6], a);
          a = fmaf(qb.w, kf[7], a);
          acc[tt] = a;
        }
      }
#pragma unroll
      for (int tt = 0; tt < kTT; ++tt) sc[tt * P + j] = acc[tt] * scale;
    }
  }
  __syncthreads();
  float inv[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int tt = 2 * warp + u;
    inv[u] = 0.0f;
    if (tt >= nt) continue;
    const int len = pos0 + t0 + tt + 1;
    float* s = sc + tt * P;
    float m = -INFINITY;
    for (int j = lane; j < len; j += 32) m = fmaxf(m, s[j]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.0f;
    for (int j = lane; j < len; j += 32) {
      const float e = ref_expf(__fsub_rn(s[j], m));   // llm.c:514-517
      s[j] = e;
      l += e;
    }
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    inv[u] = 1.0f / (l + 1e-10f);
  }
  __syncwarp();
  // softmax * V for this warp's two tokens (its own weights: no CTA barrier)
  const int ta = 2 * warp, tb = 2 * warp + 1;
  if (ta >= nt) return;
  const int la = pos0 + t0 + ta + 1, lb = tb < nt ? la + 1 : 0;
  const float* sa = sc + ta * P;
  const float* sb = sc + tb * P;
  float4 oa = make_float4(0.f, 0.f, 0.f, 0.f), ob = make_float4(0.f, 0.f, 0.f, 0.f);
  const uint16_t* vcol = vc + (size_t)kvh * kTHd + 4 * lane;
  int j = 0;
  for (; j + 8 <= la; j += 8) {
    float4 vv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint2 u = *reinterpret_cast<const uint2*>(vcol + (size_t)(j + k) * kv_dim);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      vv[k] = make_float4(a.x, a.y, b.x, b.y);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float ea = sa[j + k];
      const float eb = j + k < lb ? sb[j + k] : 0.0f;
      oa.x = fmaf(ea, vv[k].x, oa.x); oa.y = fmaf(ea, vv[k].y, oa.y);
      oa.z = fmaf(ea, vv[k].z, oa.z); oa.w = fmaf(ea, vv[k].w, oa.w);
      ob.x = fmaf(eb, vv[k].x, ob.x); ob.y = fmaf(eb, vv[k].y, ob.y);
      ob.z = fmaf(eb, vv[k].z, ob.z); ob.w = fmaf(eb, vv[k].w, ob.w);
    }
  }
  for (; j < max(la, lb); ++j) {
    const uint2 u = *reinterpret_cast<const uint2*>(vcol + (size_t)j * kv_dim);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    const float ea = j < la ? sa[j] : 0.0f;
    const float eb = j < lb ? sb[j] : 0.0f;
    oa.x = fmaf(ea, a.x, oa.x); oa.y = fmaf(ea, a.y, oa.y); oa.z = fmaf(ea, b.x, oa.z); oa.w = fmaf(ea, b.y, oa.w);
    ob.x = fmaf(eb, a.x, ob.x); ob.y = fmaf(eb, a.y, ob.y); ob.z = fmaf(eb, b.x, ob.z); ob.w = fmaf(eb, b.y, ob.w);
  }
  float* oo = out + ((size_t)(t0 + ta) * n_heads + h) * kTHd + 4 * lane;
  *reinterpret_cast<float4*>(oo) = make_float4(oa.x * inv[0], oa.y * inv[0], oa.z * inv[0], oa.w * inv[0]);
  if (tb < nt) {
    float* ob_ = out + ((size_t)(t0 + tb) * n_heads + h) * kTHd + 4 * lane;
    *reinterpret_cast<float4*>(ob_) = make_float4(ob.x * inv[1], ob.y * inv[1], ob.z * inv[1], ob.w * inv[1]);
  }
}

}  // namespace tos

using namespace tos;

namespace {
int launch_pf(const void* func, dim3 grid, dim3 block, size_t smem, void** args, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelExC(&cfg, func, args);
}
}  // namespace

extern "C" int tosk_pf_embed(float* x, const void* embd, int type, int dim, const int* toks, int n, cudaStream_t st) {
  void* args[] = {&x, (void*)&embd, &type, &dim, (void*)&toks};
  return launch_pf((const void*)pf_embed_kernel, dim3(n), dim3(256), 0, args, st);
}

extern "C" int tosk_pf_rope_store(const float* qkv, int q_rows, int kv_rows, int hd, const float2* cs, int pos0,
                                  float* q_out, void* kc, void* vc, int kv_type, int n, cudaStream_t st) {
  const int* pos_arr = nullptr;
  const int* slot = nullptr;
  size_t cstride = 0;
  void* args[] = {(void*)&qkv, &q_rows, &kv_rows, &hd, (void*)&cs, &pos0, &q_out, &kc, &vc, &kv_type,
                  (void*)&pos_arr, (void*)&slot, &cstride};
  return launch_pf((const void*)pf_rope_store_kernel, dim3(n, (q_rows + 2 * kv_rows + kRopeRows - 1) / kRopeRows),
                   dim3(256), 0, args, st);
}

extern "C" int tosk_bd_rope_store(const float* qkv, int q_rows, int kv_rows, int hd, const float2* cs,
                                  const int* pos, const int* slot, float* q_out, void* kc, void* vc, size_t cstride,
                                  int kv_type, int n, cudaStream_t st) {
  if (!pos || !slot) return (int)cudaErrorInvalidValue;
  int pos0 = 0;
  void* args[] = {(void*)&qkv, &q_rows, &kv_rows, &hd, (void*)&cs, &pos0, &q_out, &kc, &vc, &kv_type,
                  (void*)&pos, (void*)&slot, &cstride};
  return launch_pf((const void*)pf_rope_store_kernel, dim3(n, (q_rows + 2 * kv_rows + kRopeRows - 1) / kRopeRows),
                   dim3(256), 0, args, st);
}

extern "C" int tosk_pf_attention(const float* q, const void* kc, const void* vc, int kv_type, int n_heads, int n_kv,
                                 int hd, int pos0, int n, float* out, cudaStream_t st) {
  // fp16 cache, head dimension 128: token tiles (pf_attention_tile_kernel)
  const size_t tsmem = ((size_t)kTT * kTHd + (size_t)kTT * (pos0 + n)) * 4;
  if (kv_type == TOSK_F16 && hd == kTHd && tsmem <= 200 * 1024 && n > 0) {
    static bool tattr = false;
    if (!tattr) {
      const cudaError_t e = cudaFuncSetAttribute(pf_attention_tile_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) return (int)e;
      tattr = true;
    }
    const uint16_t* k16 = (const uint16_t*)kc;
    const uint16_t* v16 = (const uint16_t*)vc;
    void* args[] = {(void*)&q, (void*)&k16, (void*)&v16, &n_heads, &n_kv, &pos0, &n, &out};
    return launch_pf((const void*)pf_attention_tile_kernel, dim3(n_heads, (n + kTT - 1) / kTT), dim3(256), tsmem,
                     args, st);
  }
  const size_t smem = (size_t)(pos0 + n) * 4;
  if (smem > 200 * 1024) return (int)cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr && smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(pf_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024);
    if (e != cudaSuccess) return (int)e;
    attr = true;
  }
  const int* pos_arr = nullptr;
  const int* slot = nullptr;
  size_t cstride = 0;
  void* args[] = {(void*)&q, (void*)&kc, (void*)&vc, &kv_type, &n_heads, &n_kv, &hd, &pos0, &out,
                  (void*)&pos_arr, (void*)&slot, &cstride};
  return launch_pf((const void*)pf_attention_kernel, dim3(n_heads, n), dim3(32 * kPfWarps), smem, args, st);
}

extern "C" int tosk_bd_attention(const float* q, const void* kc, const void* vc, size_t cstride, int kv_type,
                                 int n_heads, int n_kv, int hd, const int* pos, const int* slot, int max_ctx, int n,
                                 float* out, cudaStream_t st) {
  const size_t smem = (size_t)max_ctx * 4;
  if (!pos || !slot || smem > 200 * 1024) return (int)cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr && smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(pf_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024);
    if (e != cudaSuccess) return (int)e;
    attr = true;
  }
  int pos0 = 0;
  void* args[] = {(void*)&q, (void*)&kc, (void*)&vc, &kv_type, &n_heads, &n_kv, &hd, &pos0, &out,
                  (void*)&pos, (void*)&slot, &cstride};
  return launch_pf((const void*)pf_attention_kernel, dim3(n_heads, n), dim3(32 * kPfWarps), smem, args, st);
}
