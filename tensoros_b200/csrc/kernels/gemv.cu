// gemv.cu - Q4_0 / Q8_0 GEMV for sm_100a (TensorOS runtime/nn llm_gemv), EXACT and FAST.
//
// Reference semantics (runtime/nn/llm.c):
//   q4_0_dot32 / q8_0_dot32 (llm.c:148-209): per 32-weight block, eight lane
//     chains c = 0..7 each summing the products (float)q[8k+c] * x[8k+c] over
//     k = 0..3 from +0.0f; t_l = chain_l + chain_{l+4}; r = ((t0+t1)+t2)+t3;
//     the block value is r * fp16_to_fp32(scale).
//   llm_vec_dot (llm.c:221-237): row sum = 0.0f, then += block value in block
//     order (a serial fp32 chain).
//   llm_gemv (llm.c:329-349): one row sum per output element.
//
// Design (B200):
//   * Weights are repacked once into two planes: quants [rows][nb][16|32 B]
//     and fp16 scales [rows][nbp] (nbp = nb rounded up to 8).  Every run of
//     rows of either plane is one contiguous, 16-byte aligned range, so a
//     stage of up to 16 rows is fetched with two cp.async.bulk copies.
//     Algorithmic bytes are the GGUF bytes (18 or 34 per block).
//   * One persistent CTA per SM owns a contiguous row range.  Warp 0 fills an
//     S-deep shared-memory ring of stages (mbarrier complete_tx); weights do
//     not depend on the previous kernel, so the ring fills before
//     griddepcontrol.wait returns (programmatic dependent launch).  The
//     compute warp that releases a slot last refills it.
//   * x arrives by one bulk copy (after the first stage, ahead of the rest of
//     the ring), is RMS-normalised in place when the norm is fused
//     (llm.c:416-442), and is swizzled so that every lane reads its block
//     from distinct banks.
//   * Compute warps: thread (block b, row group g) keeps its block of x in
//     registers for the whole kernel and writes one value per (row, block)
//     of every stage to a shared "partials" tile P[tr][nb].
//       EXACT: the reference block value with packed f32x2 IEEE ops
//         (nibble/byte -> float via the 2^23 magic, lane chains in order).
//       FAST: integer dot products on 24-bit fixed-point x
//         (gemv_fastmath.cuh); the swizzle pass turns each block of x into
//         its fixed-point record cooperatively.
//   * Four chain warps take stages in turn.  EXACT: lane r adds the nb
//     partials of row r serially (the reference's row chain).  FAST: lanes
//     split a stage's rows and blocks, four running sums each, then a
//     butterfly (fixed order: results are deterministic).  Then the fused
//     epilogue: plain store, residual add, RoPE + KV-cache store, or
//     SiLU(gate)*up.
//   Every mbarrier wait is bounded (tos::mbar_wait) and reports through *err.
#include "gemv_common.cuh"
#include "gemv_fastmath.cuh"

namespace tos {

constexpr int kTR = 16;   // most rows per stage
constexpr int kNCH = 4;   // chain warps: an EXACT row chain is serial (~1 us per stage of 128
                          // blocks), so four partial buffers keep the compute warps fed

// Exact block dot, Q4_0.  q holds qs[0..15]; word k = bytes 4k..4k+3 covers
// elements 8k..8k+7; byte j of the word gives element 8k+2j (low nibble) and
// 8k+2j+1 (high nibble), i.e. lane chains 2j and 2j+1.  Pair p of the f32x2
// accumulators is (chain 2p, chain 2p+1).
// kZeroInit adds the reference's leading +0.0f; it only changes the sign of
// an all-zero chain, which a row sum starting from +0.0f cannot observe, so
// the GEMV skips it and the per-block entry point keeps it.
template <bool kZeroInit>
__device__ __forceinline__ float dot_q4_0(const uint4 q, const float d, const float (&x)[32]) {
  const float kM = 8388616.0f;  // 2^23 + 8
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  float2 acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = w[k] & 0x0F0F0F0Fu;
    const uint32_t hi = (w[k] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t sel = 0x7540u | (uint32_t)p;
      const float a = __uint_as_float(prmt(lo, 0x4B000000u, sel));
      const float b = __uint_as_float(prmt(hi, 0x4B000000u, sel));
      const float2 qv = __fadd2_rn(make_float2(a, b), make_float2(-kM, -kM));
      const float2 pr = mul2_rn(qv, make_float2(x[8 * k + 2 * p], x[8 * k + 2 * p + 1]));
      if (k == 0)
        acc[p] = kZeroInit ? __fadd2_rn(make_float2(0.0f, 0.0f), pr) : pr;
      else
        acc[p] = __fadd2_rn(acc[p], pr);
    }
  }
  const float2 t01 = __fadd2_rn(acc[0], acc[2]);
  const float2 t23 = __fadd2_rn(acc[1], acc[3]);
  const float r = __fadd_rn(__fadd_rn(__fadd_rn(t01.x, t01.y), t23.x), t23.y);
  return __fmul_rn(r, d);
}

// Exact block dot, Q8_0.  Elements 8k..8k+3 are word 2k, 8k+4..8k+7 word 2k+1.
template <bool kZeroInit>
__device__ __forceinline__ float dot_q8_0(const uint4 qa, const uint4 qb, const float d,
                                          const float (&x)[32]) {
  const float kM = 8388736.0f;  // 2^23 + 128
  const uint32_t w[8] = {qa.x ^ 0x80808080u, qa.y ^ 0x80808080u, qa.z ^ 0x80808080u,
                         qa.w ^ 0x80808080u, qb.x ^ 0x80808080u, qb.y ^ 0x80808080u,
                         qb.z ^ 0x80808080u, qb.w ^ 0x80808080u};
  float2 acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t word = w[2 * k + (p >> 1)];
      const uint32_t s0 = 0x7540u | (uint32_t)((2 * p) & 3);
      const uint32_t s1 = 0x7540u | (uint32_t)((2 * p + 1) & 3);
      const float a = __uint_as_float(prmt(word, 0x4B000000u, s0));
      const float b = __uint_as_float(prmt(word, 0x4B000000u, s1));
      const float2 qv = __fadd2_rn(make_float2(a, b), make_float2(-kM, -kM));
      const float2 pr = mul2_rn(qv, make_float2(x[8 * k + 2 * p], x[8 * k + 2 * p + 1]));
      if (k == 0)
        acc[p] = kZeroInit ? __fadd2_rn(make_float2(0.0f, 0.0f), pr) : pr;
      else
        acc[p] = __fadd2_rn(acc[p], pr);
    }
  }
  const float2 t01 = __fadd2_rn(acc[0], acc[2]);
  const float2 t23 = __fadd2_rn(acc[1], acc[3]);
  const float r = __fadd_rn(__fadd_rn(__fadd_rn(t01.x, t01.y), t23.x), t23.y);
  return __fmul_rn(r, d);
}

template <int QB>
__device__ __forceinline__ float block_value(const uint8_t* stq, const uint16_t* sts, int r, int b,
                                             int nb, int nbp, const float (&x)[32]) {
  const float d = h2f(sts[r * nbp + b]);
  if constexpr (QB == 16) {
    const uint4 q = *reinterpret_cast<const uint4*>(stq + ((size_t)r * nb + b) * 16);
    return dot_q4_0<false>(q, d, x);
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(stq + ((size_t)r * nb + b) * 32);
    return dot_q8_0<false>(p[0], p[1], d, x);
  }
}

// (Capping registers at 72 so that two CTAs share an SM made every stage ~25%
// slower than the overlap it buys; one CTA per SM keeps ~85 registers.)

template <int QB, bool kNorm, int kEpi, bool kFast>
__global__ void __launch_bounds__(704, 1) tos_gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = a.S;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  int* slot_cnt = reinterpret_cast<int*>(full + S);   // S ints (room for S mbarriers)
  uint64_t* pfull = full + 2 * S;
  uint64_t* pempty = pfull + kNCH;
  uint64_t* xbar = pempty + kNCH;
  float* misc = reinterpret_cast<float*>(xbar + 1);
  float* xs = reinterpret_cast<float*>(smem + a.off_x);
  float* P = reinterpret_cast<float*>(smem + a.off_p);
  float* ws = P;   // RMSNorm weights (kNorm): the partials area is idle until the x pass
  uint8_t* stages = smem + a.off_st;

  const int NU = (a.R + a.unit - 1) / a.unit;
  const int u0 = (int)(((long long)blockIdx.x * NU) / gridDim.x);
  const int u1 = (int)(((long long)(blockIdx.x + 1) * NU) / gridDim.x);
  const int rb = u0 * a.unit;
  const int re = min(u1 * a.unit, a.R);
  const int tr = a.tr;
  const int nst = re > rb ? (re - rb + tr - 1) / tr : 0;
  const int ncw = a.nwb * a.rg;
  const int nb = a.nb, nbp = a.nbp;

  int* s_failed = reinterpret_cast<int*>(misc + 6);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      slot_cnt[s] = 0;
    }
    for (int c = 0; c < kNCH; ++c) {
      mbar_init(&pfull[c], ncw);
      mbar_init(&pempty[c], 1);
    }
    mbar_init(xbar, 1);   // one arrival (with the byte count of x and the norm weights)
    *reinterpret_cast<volatile int*>(misc + 7) = 0;
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  volatile int* xflag = reinterpret_cast<volatile int*>(misc + 7);
  if (warp == 0) {
    // ---------------- initial ring fill ----------------
    if (lane == 0) {
      // Weights do not depend on earlier kernels, so the ring fills at once.
      // After the first stage the x copy (issued by the first chain warp once
      // the previous kernel is complete) gets up to ~1.5 us to enter the copy
      // queue first: x gates all compute, and copies complete roughly in
      // issue order.  Later refills are issued by the compute warp that
      // releases a slot last, so no thread has to win issue slots from the
      // compute warps to keep the ring moving.
      const int first = min(S, nst);
      for (int it = 0; it < first; ++it) {
        if (it == 1) {
          const long long t0 = clock64();
          while (*xflag == 0 && clock64() - t0 < 3000) {
          }
          if constexpr (kNorm) bulk_g2s(ws, a.norm_w, (uint32_t)(a.cols * 4), xbar);
        }
        issue_stage<QB>(a, stages, full, it, it, rb, re);
      }
      if (kNorm && first <= 1) bulk_g2s(ws, a.norm_w, (uint32_t)(a.cols * 4), xbar);
      mbar_wait(xbar, 0, a.err, 6);
    }
    return;
  }

  // ---------------- all non-producer warps ----------------
  const int nthr = (int)blockDim.x - 32;
  pdl_wait();  // x, the residual and the position come from earlier kernels
  if (threadIdx.x == 32) {
    // x (and the norm weights, issued by the producer) land on xbar
    mbar_arrive_expect_tx(xbar, (uint32_t)(a.cols * 4) * (kNorm ? 2u : 1u));
    bulk_g2s(xs, a.x, (uint32_t)(a.cols * 4), xbar);
    *xflag = 1;
    // An earlier kernel whose bounded wait ran out leaves *err set: this
    // one then skips its work, so one failure cannot turn into a chain of
    // timeouts.  Read once the earlier kernels are complete, while x is in
    // flight (checked after the next CTA barrier).
    *s_failed = a.err ? *reinterpret_cast<volatile int*>(a.err) : 0;
  }
  if (!mbar_wait(xbar, 0, a.err, 7)) return;   // x has landed in shared memory
  float ss = 1.0f;
  if constexpr (kFast && kNorm) {
    // RMSNorm (llm.c:416-442) scale from a tree sum of squares: per-thread
    // strided sums, warp sums, then the warp partials in warp order
    float* wpart = misc + 8;
    float q = 0.0f;
    for (int i = threadIdx.x - 32; i < a.cols; i += nthr) q = fmaf(xs[i], xs[i], q);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if (lane == 0) wpart[warp - 1] = q;
    named_sync(1, nthr);
    float s2 = 0.0f;
    for (int i = 0; i < nthr / 32; ++i) s2 += wpart[i];
    ss = 1.0f / sqrtf(s2 / (float)a.cols + a.eps);
  }
  if constexpr (kNorm && !kFast) {
    // llm.c:421-427: lane l sums x[4i+l]^2 serially.  Each of four lanes
    // reads x four elements at a time (a broadcast load), squares its own
    // element and adds it; loads are batched ahead of the dependent adds.
    if (warp == 1 && lane < 4) {
      const int q4 = a.cols >> 2;
      float acc = 0.0f;
      int k = 0;
      for (; k + 8 <= q4; k += 8) {
        float e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = xs[4 * (k + j) + lane];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(e[j], e[j]));
      }
      for (; k < q4; ++k) {
        const float v = xs[4 * k + lane];
        acc = __fadd_rn(acc, __fmul_rn(v, v));
      }
      misc[lane] = acc;
    }
    named_sync(1, nthr);
    if (threadIdx.x == 32) {
      float s2 = __fadd_rn(__fadd_rn(__fadd_rn(misc[0], misc[1]), misc[2]), misc[3]);
      for (int i = a.cols & ~3; i < a.cols; ++i) s2 = __fadd_rn(s2, __fmul_rn(xs[i], xs[i]));
      // llm.c:431: ss = 1 / sqrt(ss/dim + eps)
      misc[4] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s2, (float)a.cols), a.eps)));
    }
    named_sync(1, nthr);
    ss = misc[4];
  }
  // One in-place pass over x (normalised here when the norm is fused:
  // (x*ss)*w, llm.c:437-440): the 16-byte chunk c of block b moves to slot
  // c ^ (b & 7), so that below every lane reads its own block's chunks from
  // distinct banks.  Eight consecutive threads own one block's eight chunks.
  {
    float4* x4 = reinterpret_cast<float4*>(xs);
    const float4* w4 = reinterpret_cast<const float4*>(ws);
    const int nchunk = a.cols >> 2;
    for (int base = threadIdx.x - 32; base - (threadIdx.x - 32) < nchunk; base += nthr) {
      const int t = base;   // chunk index owned by this thread in this pass
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < nchunk) {
        v = x4[t];
        if constexpr (kNorm) {
          const float4 wv = w4[t];
          v.x = __fmul_rn(__fmul_rn(v.x, ss), wv.x);
          v.y = __fmul_rn(__fmul_rn(v.y, ss), wv.y);
          v.z = __fmul_rn(__fmul_rn(v.z, ss), wv.z);
          v.w = __fmul_rn(__fmul_rn(v.w, ss), wv.w);
        }
      }
      if constexpr (kFast) {
        // FAST: the block becomes its fixed-point record in place (128 B:
        // limb words 0..23, c, s), 16-byte chunk j at slot j ^ (b & 7)
        uint32_t w0, w1, w2;
        int wi, csum;
        float sc;
        xfix_group<QB>(v, t & 7, w0, w1, w2, wi, csum, sc);
        __syncwarp();
        if (t < nchunk) {
          const int blk = t >> 3;
          uint32_t* rec = reinterpret_cast<uint32_t*>(xs) + 32 * blk;
          const int sw = blk & 7;
          auto put = [&](int word, uint32_t val) { rec[(((word >> 2) ^ sw) << 2) | (word & 3)] = val; };
          put(wi, w0);
          put(8 + wi, w1);
          put(16 + wi, w2);
          if ((t & 7) == 0) {
            put(24, (uint32_t)csum);
            put(25, __float_as_uint(sc));
          }
        }
      } else {
        __syncwarp();
        if (t < nchunk) {
          const int blk = t >> 3, c = t & 7;
          x4[(blk << 3) | (c ^ (blk & 7))] = v;
        }
      }
    }
    named_sync(1, nthr);
  }
  if (*s_failed) {
    // skip the work, but let the stages already in flight land first
    const int first = min(S, nst);
    for (int s = 0; s < first; ++s) mbar_wait(&full[s], 0, nullptr, 0);
    return;
  }

  if (warp >= 1 + kNCH) {
    // ---------------- compute warps ----------------
    const int ct = (warp - 1 - kNCH) * 32 + lane;
    const int bw = a.nwb * 32;
    const int b = ct % bw;
    const int g = ct / bw;
    const bool valid = b < nb;
    float xr[32];
    XFix xf;
#pragma unroll
    for (int i = 0; i < 32; ++i) xr[i] = 0.0f;
    if (valid) {
      const uint4* xv = reinterpret_cast<const uint4*>(xs) + 8 * b;
      if constexpr (kFast) {
        // the block's fixed-point record (chunks 0..6 of 8)
        uint32_t wds[28];
#pragma unroll
        for (int j = 0; j < 7; ++j) {
          const uint4 u = xv[j ^ (b & 7)];
          wds[4 * j] = u.x; wds[4 * j + 1] = u.y; wds[4 * j + 2] = u.z; wds[4 * j + 3] = u.w;
        }
#pragma unroll
        for (int l = 0; l < 3; ++l)
#pragma unroll
          for (int w = 0; w < 8; ++w) xf.l[l][w] = wds[8 * l + w];
        xf.c = (int)wds[24];
        xf.s = __uint_as_float(wds[25]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 v = *reinterpret_cast<const float4*>(&xv[i ^ (b & 7)]);
          xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
        }
      }
    }
    for (int it = 0; it < nst; ++it) {
      const int s = it % S;
      if (!mbar_wait(&full[s], (it / S) & 1, a.err, 2)) break;
      const int c = it % kNCH;
      if (it >= kNCH && !mbar_wait(&pempty[c], ((it / kNCH) & 1) ^ 1, a.err, 3)) break;
      const int n = min(tr, re - (rb + it * tr));
      const uint8_t* stq = stages + (size_t)s * a.stage_bytes;
      const uint16_t* sts = reinterpret_cast<const uint16_t*>(stq + a.stage_sc_off);
      float* Pc = P + c * tr * a.pstride;
      if (valid) {
        // two rows per iteration: independent dot chains interleave
        const int rg = a.rg;
        int r = g;
        if constexpr (kFast) {
          for (; r + rg < n; r += 2 * rg) {
            const float y0 = block_value_fast<QB>(stq, sts, r, b, nb, nbp, xf);
            const float y1 = block_value_fast<QB>(stq, sts, r + rg, b, nb, nbp, xf);
            Pc[r * a.pstride + b] = y0;
            Pc[(r + rg) * a.pstride + b] = y1;
          }
          if (r < n) Pc[r * a.pstride + b] = block_value_fast<QB>(stq, sts, r, b, nb, nbp, xf);
        } else {
          for (; r + rg < n; r += 2 * rg) {
            const float y0 = block_value<QB>(stq, sts, r, b, nb, nbp, xr);
            const float y1 = block_value<QB>(stq, sts, r + rg, b, nb, nbp, xr);
            Pc[r * a.pstride + b] = y0;
            Pc[(r + rg) * a.pstride + b] = y1;
          }
          if (r < n) Pc[r * a.pstride + b] = block_value<QB>(stq, sts, r, b, nb, nbp, xr);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&pfull[c]);
        // release slot s; the last of the compute warps refills it
        if (atomicAdd(&slot_cnt[s], 1) == ncw - 1) {
          slot_cnt[s] = 0;
          if (it + S < nst) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_stage<QB>(a, stages, full, it + S, s, rb, re);
          }
        }
      }
    }
    return;
  }

  // ---------------- chain warps (warp 1 .. kNCH) ----------------
  const int cw = warp - 1;
  int pos = 0;
  if constexpr (kEpi == TOSK_EPI_QKV) pos = *a.epi.pos;
  for (int it = cw; it < nst; it += kNCH) {
    if (!mbar_wait(&pfull[cw], (it / kNCH) & 1, a.err, 4)) break;
    const int r0 = rb + it * tr;
    const int n = min(tr, re - r0);
    const float* Pr = P + (cw * tr + min(lane, tr - 1)) * a.pstride;
    float y = 0.0f;  // llm.c:223: sum = 0.0f, then += block value, in block order
    if constexpr (kFast) {
      // tree sum: lane = (row lane % tr, segment lane / tr); four running sums
      // per lane over its segment, then a butterfly across the segments
      const int nseg = 32 / tr;
      const int seg = lane / tr;
      const int L = (((nb + nseg - 1) / nseg) + 3) & ~3;
      const int j0 = min(nb, seg * L), j1 = min(nb, seg * L + L);
      const float* Prow = P + (cw * tr + lane % tr) * a.pstride;
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
      int j = j0;
      for (; j + 4 <= j1; j += 4) {
        const float4 v = *reinterpret_cast<const float4*>(Prow + j);
        s0 += v.x; s1 += v.y; s2 += v.z; s3 += v.w;
      }
      for (; j < j1; ++j) s0 += Prow[j];
      float t = (s0 + s1) + (s2 + s3);
      for (int o = tr; o < 32; o <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      y = t;
    } else if (lane < n) {
      // loads batched ahead of the dependent adds (the chain itself is serial)
      int bb = 0;
      for (; bb + 32 <= nb; bb += 32) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const float4*>(Pr + bb + 4 * j);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          y = __fadd_rn(y, v[j].x);
          y = __fadd_rn(y, v[j].y);
          y = __fadd_rn(y, v[j].z);
          y = __fadd_rn(y, v[j].w);
        }
      }
      for (; bb + 4 <= nb; bb += 4) {
        const float4 v = *reinterpret_cast<const float4*>(Pr + bb);
        y = __fadd_rn(y, v.x);
        y = __fadd_rn(y, v.y);
        y = __fadd_rn(y, v.z);
        y = __fadd_rn(y, v.w);
      }
      for (; bb < nb; ++bb) y = __fadd_rn(y, Pr[bb]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&pempty[cw]);
    gemv_epilogue<kEpi>(a, y, r0, n, lane, pos);
  }
}

// ---------------------------------------------------------------------------
// Weight repack: GGUF blocks -> planes
// ---------------------------------------------------------------------------
__global__ void repack_kernel(const uint8_t* __restrict__ src, int src_rows, int nb, int qb,
                              uint8_t* __restrict__ qs, uint16_t* __restrict__ sc, int nbp,
                              int dst_row0, int dst_row_step) {
  const size_t total = (size_t)src_rows * nb;
  const int bsz = qb + 2;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / nb);
    const int b = (int)(i % nb);
    const uint8_t* s = src + i * bsz;
    const size_t drow = (size_t)dst_row0 + (size_t)row * dst_row_step;
    sc[drow * nbp + b] = (uint16_t)(s[0] | (s[1] << 8));
    uint8_t* d = qs + (drow * nb + b) * qb;
    for (int j = 0; j < qb; ++j) d[j] = s[2 + j];
  }
}

// Per-block exact values (with the reference's leading +0.0f), GGUF layout.
__global__ void block_dots_kernel(const uint8_t* __restrict__ blocks, int type,
                                  const float* __restrict__ x, int n_blocks,
                                  float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_blocks) return;
  float xr[32];
  const float4* xv = reinterpret_cast<const float4*>(x + 32 * (size_t)i);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 v = xv[k];
    xr[4 * k] = v.x; xr[4 * k + 1] = v.y; xr[4 * k + 2] = v.z; xr[4 * k + 3] = v.w;
  }
  if (type == TOSK_Q4_0) {
    const uint8_t* p = blocks + (size_t)i * 18;
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = p[2 + 4 * k] | (p[3 + 4 * k] << 8) | (p[4 + 4 * k] << 16) | ((uint32_t)p[5 + 4 * k] << 24);
    out[i] = dot_q4_0<true>(make_uint4(w[0], w[1], w[2], w[3]), h2f((uint16_t)(p[0] | (p[1] << 8))), xr);
  } else {
    const uint8_t* p = blocks + (size_t)i * 34;
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      w[k] = p[2 + 4 * k] | (p[3 + 4 * k] << 8) | (p[4 + 4 * k] << 16) | ((uint32_t)p[5 + 4 * k] << 24);
    out[i] = dot_q8_0<true>(make_uint4(w[0], w[1], w[2], w[3]), make_uint4(w[4], w[5], w[6], w[7]),
                            h2f((uint16_t)(p[0] | (p[1] << 8))), xr);
  }
}

}  // namespace tos

using namespace tos;

static int g_num_sms = 0;

extern "C" int tosk_num_sms(void) {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

extern "C" int tosk_qmat_alloc(tosk_qmat_t* m, int type, int rows, int cols, cudaStream_t st) {
  if (!m || rows <= 0 || cols <= 0 || (cols % 32) != 0) return (int)cudaErrorInvalidValue;
  if (type != TOSK_Q4_0 && type != TOSK_Q8_0) return (int)cudaErrorInvalidValue;
  m->type = type;
  m->rows = rows;
  m->cols = cols;
  m->nb = cols / 32;
  m->nbp = (m->nb + 7) & ~7;
  m->qb = type == TOSK_Q4_0 ? 16 : 32;
  const size_t qbytes = (size_t)rows * m->nb * m->qb;
  const size_t sbytes = (size_t)rows * m->nbp * 2;
  m->qs = nullptr;
  m->sc = nullptr;
  m->rws = nullptr;
  cudaError_t e = cudaMalloc((void**)&m->qs, qbytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaMalloc((void**)&m->sc, sbytes);
  if (e == cudaSuccess) e = cudaMalloc((void**)&m->rws, (size_t)rows * 4);
  if (e != cudaSuccess) {
    cudaFree(m->qs);
    if (m->sc) cudaFree(m->sc);
    m->qs = nullptr;
    m->sc = nullptr;
    return (int)e;
  }
  m->bytes = qbytes + sbytes + (size_t)rows * 4;
  // the padding of the scale rows is cleared on the stream that repacks into
  // the planes next, so the clear cannot land after the repack
  return (int)cudaMemsetAsync(m->sc, 0, sbytes, st);
}

extern "C" void tosk_qmat_free(tosk_qmat_t* m) {
  if (!m) return;
  if (m->qs) cudaFree(m->qs);
  if (m->sc) cudaFree(m->sc);
  if (m->rws) cudaFree(m->rws);
  m->qs = nullptr;
  m->sc = nullptr;
  m->rws = nullptr;
  m->bytes = 0;
}

extern "C" int tosk_qmat_repack(tosk_qmat_t* m, const void* const* src, const int* src_rows,
                                int n_src, int interleave, cudaStream_t st) {
  int row0 = 0;
  for (int s = 0; s < n_src; ++s) {
    const int dst_row0 = interleave ? s : row0;
    const int step = interleave ? n_src : 1;
    const size_t total = (size_t)src_rows[s] * m->nb;
    const int threads = 256;
    const int grid = (int)((total + threads - 1) / threads < 65535 ? (total + threads - 1) / threads : 65535);
    repack_kernel<<<grid, threads, 0, st>>>((const uint8_t*)src[s], src_rows[s], m->nb, m->qb, m->qs,
                                            m->sc, m->nbp, dst_row0, step);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    row0 += src_rows[s];
  }
  return tosk_qmat_row_scales(m, st);
}

template <int QB, bool kNorm, int kEpi, bool kFast>
static int launch_gemv(const GemvArgs& a, int grid, int threads, size_t smem, int pdl,
                       cudaStream_t st) {
  static bool done = false;
  auto kern = tos_gemv_kernel<QB, kNorm, kEpi, kFast>;
  if (!done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return (int)e;
    done = true;
  }
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
  return (int)cudaLaunchKernelEx(&cfg, kern, a);
}

template <int QB, bool kFast>
static int dispatch_gemv(const GemvArgs& a, bool norm, int epi, int grid, int threads, size_t smem,
                         int pdl, cudaStream_t st) {
  if (norm) {
    switch (epi) {
      case TOSK_EPI_STORE: return launch_gemv<QB, true, TOSK_EPI_STORE, kFast>(a, grid, threads, smem, pdl, st);
      case TOSK_EPI_QKV: return launch_gemv<QB, true, TOSK_EPI_QKV, kFast>(a, grid, threads, smem, pdl, st);
      case TOSK_EPI_SWIGLU: return launch_gemv<QB, true, TOSK_EPI_SWIGLU, kFast>(a, grid, threads, smem, pdl, st);
      default: return (int)cudaErrorInvalidValue;
    }
  }
  switch (epi) {
    case TOSK_EPI_STORE: return launch_gemv<QB, false, TOSK_EPI_STORE, kFast>(a, grid, threads, smem, pdl, st);
    case TOSK_EPI_RESID: return launch_gemv<QB, false, TOSK_EPI_RESID, kFast>(a, grid, threads, smem, pdl, st);
    case TOSK_EPI_QKV: return launch_gemv<QB, false, TOSK_EPI_QKV, kFast>(a, grid, threads, smem, pdl, st);
    case TOSK_EPI_SWIGLU: return launch_gemv<QB, false, TOSK_EPI_SWIGLU, kFast>(a, grid, threads, smem, pdl, st);
    default: return (int)cudaErrorInvalidValue;
  }
}

static inline uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

extern "C" int tosk_gemv(const tosk_qmat_t* w, const float* x, const tosk_norm_t* norm, float* out,
                         const tosk_epi_t* epi, int mode, int* err, int pdl, cudaStream_t st) {
  if (!w || !x || !out) return (int)cudaErrorInvalidValue;
  if (mode != TOSK_GEMV_EXACT && mode != TOSK_GEMV_FAST) return (int)cudaErrorInvalidValue;
  // x and the norm weights are fetched with bulk copies: 16-byte alignment
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (norm && (reinterpret_cast<uintptr_t>(norm->norm_w) & 15)))
    return (int)cudaErrorInvalidValue;
  GemvArgs a = {};
  a.qs = w->qs;
  a.sc = w->sc;
  a.x = x;
  const bool fuse_norm = norm && norm->norm_w;
  a.norm_w = fuse_norm ? norm->norm_w : nullptr;
  a.eps = norm ? norm->eps : 1e-6f;
  a.out = out;
  a.err = err;
  a.R = w->rows;
  a.nb = w->nb;
  a.nbp = w->nbp;
  a.cols = w->cols;
  const int kind = epi ? epi->kind : TOSK_EPI_STORE;
  a.unit = (kind == TOSK_EPI_QKV || kind == TOSK_EPI_SWIGLU) ? 2 : 1;
  if (epi) a.epi = *epi;
  a.epi.kind = kind;
  a.nwb = (w->nb + 31) / 32;
  // cols > 16*1024 would need several blocks per thread: not supported
  if (a.nwb > 16) return (int)cudaErrorInvalidValue;
  // Row groups split a stage's rows between warps holding the same blocks,
  // each thread taking tr/rg rows of every stage.  EXACT: ~8 compute warps
  // per CTA (one CTA per SM); FAST (cheaper block values): ~16.
  const int want = mode == TOSK_GEMV_FAST ? 16 : 8;
  a.rg = a.nwb >= want ? 1 : (want / a.nwb);
  if (a.rg > kTR) a.rg = kTR;
  const int threads = 32 * (1 + kNCH + a.nwb * a.rg);
  a.pstride = (int)round_up((uint32_t)w->nb, 8) + 4;
  const uint32_t hdr = 384;   // up to 2*8 + 2*kNCH + 1 mbarriers, 8 floats, 24 warp partials
  a.off_x = hdr;
  const uint32_t xbytes = round_up((uint32_t)w->cols * 4, 128);
  a.off_w = 0;
  a.off_p = a.off_x + xbytes;
  // ~200 KB of shared memory (one CTA per SM).  Rows per stage: 16 unless two
  // stages of long rows and their partials would not fit; paired epilogues
  // (RoPE, SiLU*up) need an even count.
  const uint32_t budget_hi = 227 * 1024;
  const uint32_t budget_lo = 200 * 1024;
  uint32_t pbytes = 0;
  a.tr = kTR;
  for (;;) {
    pbytes = (uint32_t)(kNCH * a.tr * a.pstride * 4);
    // the partials area also holds the RMSNorm weights until the x pass
    if (fuse_norm && pbytes < (uint32_t)w->cols * 4) pbytes = (uint32_t)w->cols * 4;
    pbytes = round_up(pbytes, 128);
    a.off_st = a.off_p + pbytes;
    const uint32_t qbytes = (uint32_t)(a.tr * w->nb * w->qb);
    a.stage_sc_off = round_up(qbytes, 16);
    a.stage_bytes = round_up(a.stage_sc_off + (uint32_t)(a.tr * w->nbp * 2), 128);
    if (a.off_st + 2 * a.stage_bytes <= budget_hi || a.tr <= a.unit) break;
    a.tr >>= 1;
  }
  int S = (int)((budget_lo > a.off_st ? budget_lo - a.off_st : 0) / a.stage_bytes);
  if (S < 2) S = 2;
  if (S > 8) S = 8;
  if (a.off_st + (uint32_t)S * a.stage_bytes > budget_hi) return (int)cudaErrorInvalidValue;
  // header holds 2*S + 2*kNCH barriers, 8 floats and 24 warp partials
  if ((uint32_t)(8 * (2 * S + 2 * kNCH + 1) + 32 + 96) > hdr || threads / 32 - 1 > 24)
    return (int)cudaErrorInvalidValue;
  a.S = S;
  const size_t smem = a.off_st + (size_t)S * a.stage_bytes;
  // layout checks: every region inside its own range
  if (a.off_x + (uint32_t)w->cols * 4 > a.off_p || a.off_p + pbytes > a.off_st ||
      a.off_p + (uint32_t)(kNCH * a.tr * a.pstride * 4) > a.off_st || smem > budget_hi)
    return (int)cudaErrorInvalidValue;
  const int NU = (a.R + a.unit - 1) / a.unit;
  int grid = tosk_num_sms();
  if (grid > NU) grid = NU;
  const bool fast = mode == TOSK_GEMV_FAST;
  if (w->qb == 16)
    return fast ? dispatch_gemv<16, true>(a, fuse_norm, kind, grid, threads, smem, pdl, st)
                : dispatch_gemv<16, false>(a, fuse_norm, kind, grid, threads, smem, pdl, st);
  return fast ? dispatch_gemv<32, true>(a, fuse_norm, kind, grid, threads, smem, pdl, st)
              : dispatch_gemv<32, false>(a, fuse_norm, kind, grid, threads, smem, pdl, st);
}

extern "C" int tosk_block_dots(const void* blocks, int type, const float* x, int n_blocks, float* out,
                               cudaStream_t st) {
  if (type != TOSK_Q4_0 && type != TOSK_Q8_0) return (int)cudaErrorInvalidValue;
  if (n_blocks <= 0) return 0;
  block_dots_kernel<<<(n_blocks + 127) / 128, 128, 0, st>>>((const uint8_t*)blocks, type, x, n_blocks, out);
  return (int)cudaGetLastError();
}
