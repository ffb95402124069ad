// gemm_tc.cu - batched Q4_0 / Q8_0 GEMM on the 5th-generation tensor cores
// (tcgen05, TMEM accumulators) for prefill and batched decode.
//
// Y[M][N] = X[M][K] . W[N][K]^T, W in the repacked GGUF planes of the GEMV.
// The reference has no batched path: it runs llm_forward_token per token
// (runtime/nn/llm.c:641-743), i.e. M independent GEMVs (llm.c:329-349).
//
// Precision.  Each weight (n - 8)*d (Q4_0, at most 15 significant bits) or
// q*d (Q8_0, at most 19) is, after a per-row power-of-two scale, exactly
// W_hi + W_lo with W_hi, W_lo fp16.  Each activation row is scaled by a power
// of two and split into X_hi + X_lo (fp16, 22 significant bits).  The kernel
// accumulates X_hi W_hi + X_lo W_hi + X_hi W_lo in fp32 TMEM (the dropped
// X_lo W_lo is below 2^-22 relative) and undoes both scales exactly in the
// epilogue: results agree with the fp32 GEMV to ~1e-6 (normwise).
//
// Design (sm_100a, one CTA per 128x128 output tile and K slice):
//   * prep kernel: X (fp32, row-major) -> per-row scale and X_hi / X_lo in
//     the UMMA K-major SWIZZLE_128B layout, one 16 KB block per 64-wide K
//     chunk, so the GEMM fetches each with a single cp.async.bulk.
//   * warp 0: TMEM allocation and the A (activation) bulk copies;
//     warp 1: one elected thread issues the tcgen05.mma (3 per 16-wide K step)
//     and commits each stage back to the producers;
//     warps 2..9: dequantise 128 weight rows x 64 columns per stage straight
//     into the swizzled B tiles (2 threads per row), then run the epilogue
//     (tcgen05.ld of the fp32 accumulator, exact unscaling, store).
//   * S-stage shared-memory ring; every wait is bounded and reports through
//     *err; TMEM is always released.
//   * K is split over CTAs when the tile grid alone does not fill the GPU;
//     partial tiles are added in split order by a reduce kernel.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

constexpr int kBM = 128;                  // tokens per tile (TMEM lanes)
constexpr int kBN = 128;                  // weight rows per tile (TMEM columns)
constexpr int kBK = 64;                   // K per stage: one 128-byte fp16 row
constexpr int kPart = kBM * kBK * 2;      // 16 KB: one operand part of a stage
constexpr int kStageBytes = 4 * kPart;    // A_hi, A_lo, B_hi, B_lo
constexpr int kGStages = 3;
constexpr int kDqWarps = 8;               // dequantising / epilogue warps
constexpr int kGThreads = 32 * (2 + kDqWarps);

// ---------------------------------------------------------------------------
// tcgen05 / descriptor helpers (PTX ISA 8.7, sm_100a)
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, K-major, SWIZZLE_128B: 8-row atoms of
// 1024 bytes (stride byte offset 1024), version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);          // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused, 16 B)
  d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset
  d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp32 accumulate, fp16 A and B, both K-major,
// N = kBN, M = kBM.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread has
// finished (its shared-memory operands may then be overwritten).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of 16-byte chunk c (0..7) of row r in a K-major SWIZZLE_128B
// tile of 128-byte rows.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Power of two 2^k with m * 2^k in [2^13, 2^14) (m > 0 finite), else 1.
__device__ __forceinline__ float pow2_to_2p13(float m) {
  const int eb = (int)((__float_as_uint(m) >> 23) & 0xFF);
  if (m <= 0.0f || eb == 255) return 1.0f;
  int k = 13 - (eb - 127);
  k = max(-126, min(127, k));
  return __uint_as_float((uint32_t)(k + 127) << 23);
}

// Splits two floats with at most 22 significant bits into fp16 pairs
// hi + lo: Veltkamp split at 11 bits (t = v (2^13 + 1), hi = t - (t - v),
// lo = v - hi, all exact in round-to-nearest fp32), then one packed
// conversion per pair.  hi has 11 significant bits (exact in fp16); lo is
// exact for weights (at most 15 bits in all) and keeps 11 more bits of an
// activation.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi2, uint32_t& lo2) {
  const float ta = __fmul_rn(a, 8193.0f), tb = __fmul_rn(b, 8193.0f);
  const float ha = __fsub_rn(ta, __fsub_rn(ta, a)), hb = __fsub_rn(tb, __fsub_rn(tb, b));
  const __half2 H = __floats2half2_rn(ha, hb);
  const __half2 L = __floats2half2_rn(__fsub_rn(a, ha), __fsub_rn(b, hb));
  hi2 = *reinterpret_cast<const uint32_t*>(&H);
  lo2 = *reinterpret_cast<const uint32_t*>(&L);
}

struct GemmArgs {
  const uint8_t* qs;    // weight quants [N][nb][qb]
  const uint16_t* sc;   // weight scales [N][nbp] (fp16)
  const float* rws;     // per-row power-of-two weight scales [N]
  int qb, nb, nbp;      // 16 (Q4_0) or 32 (Q8_0) bytes per block
  int N, K;
  const uint8_t* xa;    // prepared activations [mtiles][nkc][hi, lo][16 KB]
  const float* xs;      // per-row activation scales [Mpad]
  float* out;           // splits == 1: Y [M][N]; else partials [split][Mpad][N]
  int M, Mpad, mtiles, ntiles;
  int splits, kc_per_split, nkc;
  int* err;
};

// ---------------------------------------------------------------------------
// prep: X[M][K] fp32 -> per-row power-of-two scale and fp16 hi/lo parts in
// the swizzled K-major layout (rows beyond M are zero)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) gemm_prep_kernel(const float* __restrict__ x, int M, int K,
                                                        uint8_t* __restrict__ xa, float* __restrict__ xs) {
  __shared__ float red[4];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;           // padded row
  const int mt = m / kBM, r = m % kBM;
  const int nkc = K / kBK;
  const bool valid = m < M;
  const float* xr = x + (size_t)m * K;
  float mx = 0.0f;
  if (valid)
    for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(xr[i]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float s = pow2_to_2p13(mx);
  if (threadIdx.x == 0) xs[m] = s;
  // one 16-byte chunk (8 elements) per thread and step
  for (int q = threadIdx.x; q < K / 8; q += blockDim.x) {
    const int kc = q / 8, c = q % 8;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v0 = valid ? __fmul_rn(xr[8 * q + 2 * e], s) : 0.0f;
      const float v1 = valid ? __fmul_rn(xr[8 * q + 2 * e + 1], s) : 0.0f;
      split2(v0, v1, hi[e], lo[e]);
    }
    uint8_t* blk = xa + ((size_t)mt * nkc + kc) * 2 * kPart;
    *reinterpret_cast<uint4*>(blk + sw128_off(r, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(blk + kPart + sw128_off(r, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// split-K partials added in split order
__global__ void gemm_reduce_kernel(const float* __restrict__ part, int splits, int M, int Mpad, int N,
                                   float* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const size_t total = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int s = 1; s < splits; ++s) acc += part[(size_t)s * Mpad * N + i];
    y[i] = acc;
  }
}

// Dequantises one 32-element block (quants in q0[, q1], scale d) into fp16
// hi / lo pairs scaled by ws, exactly (Q4_0: 15 significant bits at most,
// Q8_0: 19, split 11 + 8 by split2).
template <int QB>
__device__ __forceinline__ void dequant_block(const uint4 q0, const uint4 q1, float d, float ws,
                                              uint32_t (&hi)[16], uint32_t (&lo)[16]) {
  const float ds = __fmul_rn(d, ws);   // exact (power-of-two ws)
  if constexpr (QB == 16) {
    // Q4_0: (n - 8) is exact in fp16, and so are its products with the two
    // parts of D = d*ws (11 significant bits) split 7 + 4: the weight is
    // W_hi + W_lo = (n-8) D_hi + (n-8) D_lo without rounding, in packed
    // half2 arithmetic.  Nibbles become 1024 + n through the 0x6400 magic.
    const float D = ds;
    const float Dh = __uint_as_float(__float_as_uint(D) & ~((1u << 17) - 1u));   // top 7 bits
    const __half2 dh2 = __float2half2_rn(Dh);
    const __half2 dl2 = __float2half2_rn(__fsub_rn(D, Dh));
    const __half2 k1032 = __float2half2_rn(1032.0f);
    const uint32_t w[4] = {q0.x, q0.y, q0.z, q0.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lw = w[k] & 0x0F0F0F0Fu, hw = (w[k] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        // byte j = 4k + p: element 2j = low nibble, 2j+1 = high (llm.c:162-165)
        const uint32_t sel = (uint32_t)(p | (p << 4) | ((4 + p) << 8) | ((4 + p) << 12));
        const uint32_t t = (__byte_perm(lw, hw, sel) & 0x00FF00FFu) | 0x64006400u;
        const __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&t), k1032);
        const __half2 H = __hmul2(v, dh2), L = __hmul2(v, dl2);
        hi[4 * k + p] = *reinterpret_cast<const uint32_t*>(&H);
        lo[4 * k + p] = *reinterpret_cast<const uint32_t*>(&L);
      }
    }
  } else {
    const float kM = 8388736.0f;       // 2^23 + 128
    const uint32_t w[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u, q0.w ^ 0x80808080u,
                           q1.x ^ 0x80808080u, q1.y ^ 0x80808080u, q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t word = w[j >> 1];
      const uint32_t b0 = (uint32_t)((2 * j) & 3), b1 = (uint32_t)((2 * j + 1) & 3);
      const float e0 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | b0)), kM);
      const float e1 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | b1)), kM);
      split2(__fmul_rn(e0, ds), __fmul_rn(e1, ds), hi[j], lo[j]);   // llm.c:199-200
    }
  }
}

template <int QB>
__global__ void __launch_bounds__(kGThreads, 1) gemm_tc_kernel(const GemmArgs a) {
  extern __shared__ uint8_t gsm[];
  // header (barriers, TMEM address, row scales), then 1024-aligned stages
  uint64_t* a_full = reinterpret_cast<uint64_t*>(gsm);
  uint64_t* b_full = a_full + kGStages;
  uint64_t* empty = b_full + kGStages;
  uint64_t* done = empty + kGStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* s_inv_ws = reinterpret_cast<float*>(gsm + 128);            // [kBN]
  const uint32_t sbase = (smem_u32(gsm) + 640 + 1023) & ~1023u;
  uint8_t* stages = gsm + (sbase - smem_u32(gsm));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int t = blockIdx.x;
  const int nt = t % a.ntiles;
  t /= a.ntiles;
  const int mt = t % a.mtiles;
  const int split = t / a.mtiles;
  const int n0 = nt * kBN;
  const int kc0 = split * a.kc_per_split;
  const int nk = min(a.nkc, kc0 + a.kc_per_split) - kc0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&b_full[s], kDqWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kBN);   // fp32 accumulator: 128 lanes x 128 columns
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ---------------- activation tiles: one bulk copy per part ----------------
    if (lane == 0) {
      pdl_wait();   // the prepared activations come from the previous kernel
      for (int i = 0; i < nk; ++i) {
        const int s = i % kGStages;
        if (i >= kGStages && !mbar_wait(&empty[s], ((i / kGStages) - 1) & 1, a.err, 21)) break;
        uint8_t* st = stages + (size_t)s * kStageBytes;
        const uint8_t* src = a.xa + ((size_t)mt * a.nkc + kc0 + i) * 2 * kPart;
        mbar_arrive_expect_tx(&a_full[s], 2 * kPart);
        bulk_g2s(st, src, kPart, &a_full[s]);
        bulk_g2s(st + kPart, src + kPart, kPart, &a_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issue (one thread) ----------------
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % kGStages;
        ok = mbar_wait(&a_full[s], (i / kGStages) & 1, a.err, 22) &&
             mbar_wait(&b_full[s], (i / kGStages) & 1, a.err, 23);
        if (!ok) break;
        tc_fence_after();
        const uint32_t base = smem_u32(stages + (size_t)s * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ah = sw128_desc(base + 32 * kk);
          const uint64_t al = sw128_desc(base + kPart + 32 * kk);
          const uint64_t bh = sw128_desc(base + 2 * kPart + 32 * kk);
          const uint64_t bl = sw128_desc(base + 3 * kPart + 32 * kk);
          umma_f16(taddr, ah, bh, (i > 0 || kk > 0) ? 1u : 0u);
          umma_f16(taddr, al, bh, 1u);
          umma_f16(taddr, ah, bl, 1u);
        }
        umma_commit(&empty[s]);   // operands of stage s may be refilled once read
      }
      umma_commit(done);          // the accumulator is final
    }
  } else {
    // ---------------- weight dequantisation, then the epilogue ----------------
    const int tid = threadIdx.x - 64;       // 0..255
    const int r = tid >> 1, h = tid & 1;    // weight row in the tile, half of the 64 columns
    const int n = n0 + r;
    const bool valid = n < a.N;
    const float ws = valid ? a.rws[n] : 1.0f;
    if (h == 0) s_inv_ws[r] = 1.0f / ws;   // exact: power of two
    // raw blocks are loaded kPf stages ahead (registers), so the global
    // latency overlaps the dequantisation of the stages before
    constexpr int kPf = 3;
    uint4 qv[kPf], qv2[kPf];
    float dv[kPf];
    auto fetch = [&](int i, uint4& q0, uint4& q1, float& d) {
      if (valid && i < nk) {
        const int b = 2 * (kc0 + i) + h;
        const uint8_t* src = a.qs + ((size_t)n * a.nb + b) * QB;
        q0 = *reinterpret_cast<const uint4*>(src);
        if constexpr (QB == 32) q1 = *reinterpret_cast<const uint4*>(src + 16);
        d = h2f(a.sc[(size_t)n * a.nbp + b]);
      }
    };
#pragma unroll
    for (int u = 0; u < kPf; ++u) {
      qv[u] = qv2[u] = make_uint4(0, 0, 0, 0);
      dv[u] = 0.0f;
      fetch(u, qv[u], qv2[u], dv[u]);
    }
    bool ok = true;
    for (int i0 = 0; i0 < nk && ok; i0 += kPf) {
#pragma unroll
      for (int u = 0; u < kPf; ++u) {
        const int i = i0 + u;
        if (i >= nk) break;
        const int s = i % kGStages;
        if (i >= kGStages && !mbar_wait(&empty[s], ((i / kGStages) - 1) & 1, a.err, 24)) { ok = false; break; }
        uint32_t hi[16], lo[16];
        if (valid) {
          dequant_block<QB>(qv[u], qv2[u], dv[u], ws, hi, lo);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) hi[e] = lo[e] = 0u;
        }
        fetch(i + kPf, qv[u], qv2[u], dv[u]);
        uint8_t* st = stages + (size_t)s * kStageBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          *reinterpret_cast<uint4*>(st + 2 * kPart + sw128_off(r, 4 * h + c)) =
              make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
          *reinterpret_cast<uint4*>(st + 3 * kPart + sw128_off(r, 4 * h + c)) =
              make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&b_full[s]);
      }
    }
    // epilogue: warp w reads TMEM lanes 32*(w%4).. and columns 64*((w-2)/4)..
    asm volatile("barrier.sync 1, %0;" ::"r"(32 * kDqWarps) : "memory");   // s_inv_ws complete
    if (ok && mbar_wait(done, 0, a.err, 25)) {
      tc_fence_after();
      pdl_wait();   // the activation scales come from the previous kernel (already complete here)
      const int q = warp & 3;
      const int cb = 64 * ((warp - 2) >> 2);
      const int m = mt * kBM + 32 * q + lane;
      const float inv_s = 1.0f / a.xs[m];   // exact: power of two
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v[32];
        tmem_ld32(taddr + ((uint32_t)(32 * q) << 16) + (uint32_t)(cb + 32 * half), v);
        const int c0 = cb + 32 * half;
        if (a.splits == 1) {
          if (m < a.M)
            for (int j = 0; j < 32; ++j)
              if (n0 + c0 + j < a.N) a.out[(size_t)m * a.N + n0 + c0 + j] = (v[j] * inv_s) * s_inv_ws[c0 + j];
        } else {
          float* p = a.out + ((size_t)split * a.Mpad + m) * a.N;
          for (int j = 0; j < 32; ++j)
            if (n0 + c0 + j < a.N) p[n0 + c0 + j] = (v[j] * inv_s) * s_inv_ws[c0 + j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(taddr, kBN);
  }
}

// Per-row power-of-two scale keeping every |dequantised weight| * ws below
// 2^14 (one warp per row).
__global__ void row_scale_kernel(const uint16_t* __restrict__ sc, int rows, int nb, int nbp, float qmax,
                                 float* __restrict__ rws) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float md = 0.0f;
  for (int b = lane; b < nb; b += 32) md = fmaxf(md, fabsf(h2f(sc[(size_t)warp * nbp + b])));
  for (int o = 16; o > 0; o >>= 1) md = fmaxf(md, __shfl_xor_sync(0xffffffffu, md, o));
  if (lane == 0) rws[warp] = pow2_to_2p13(md * qmax);
}

}  // namespace tos

using namespace tos;

extern "C" int tosk_qmat_row_scales(tosk_qmat_t* m, cudaStream_t st) {
  if (!m || !m->rws) return (int)cudaErrorInvalidValue;
  const int threads = 256;
  const int grid = (int)(((size_t)m->rows * 32 + threads - 1) / threads);
  row_scale_kernel<<<grid, threads, 0, st>>>(m->sc, m->rows, m->nb, m->nbp, m->qb == 16 ? 8.0f : 128.0f,
                                             m->rws);
  return (int)cudaGetLastError();
}

namespace {
struct GemmPlan {
  int mtiles, ntiles, nkc, splits, kcps, Mpad;
  size_t off_xs, off_part, bytes;
};

GemmPlan gemm_plan(int M, int N, int K) {
  GemmPlan p;
  p.mtiles = (M + kBM - 1) / kBM;
  p.Mpad = p.mtiles * kBM;
  p.ntiles = (N + kBN - 1) / kBN;
  p.nkc = K / kBK;
  const int tiles = p.mtiles * p.ntiles;
  const int sms = tosk_num_sms();
  int splits = sms / tiles;                        // fill the GPU in one wave
  if (splits > p.nkc) splits = p.nkc;
  if (splits < 1) splits = 1;
  p.kcps = (p.nkc + splits - 1) / splits;
  p.splits = (p.nkc + p.kcps - 1) / p.kcps;        // every split gets >= 1 chunk
  const size_t xa = (size_t)p.mtiles * p.nkc * 2 * kPart;
  p.off_xs = xa;
  p.off_part = (p.off_xs + (size_t)p.Mpad * 4 + 255) & ~(size_t)255;
  p.bytes = p.off_part + (p.splits > 1 ? (size_t)p.splits * p.Mpad * N * 4 : 0);
  return p;
}

template <typename Kern>
int launch_ex(Kern kern, int grid, int threads, size_t smem, int pdl, cudaStream_t st, void** args) {
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
}  // namespace

extern "C" size_t tosk_gemm_ws_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % kBK) return 0;
  return gemm_plan(M, N, K).bytes;
}

extern "C" int tosk_gemm_q(const tosk_qmat_t* w, const float* x, int M, float* y, void* ws, size_t ws_bytes,
                           int* err, int pdl, cudaStream_t st) {
  if (!w || !x || !y || !ws || M <= 0) return (int)cudaErrorInvalidValue;
  const int N = w->rows, K = w->cols;
  if (K % kBK || (reinterpret_cast<uintptr_t>(ws) & 255)) return (int)cudaErrorInvalidValue;
  const GemmPlan p = gemm_plan(M, N, K);
  if (ws_bytes < p.bytes) return (int)cudaErrorInvalidValue;
  uint8_t* xa = (uint8_t*)ws;
  float* xs = (float*)((uint8_t*)ws + p.off_xs);
  float* part = (float*)((uint8_t*)ws + p.off_part);
  {
    int Mi = M, Ki = K;
    void* args[] = {(void*)&x, &Mi, &Ki, &xa, &xs};
    const int e = launch_ex(gemm_prep_kernel, p.Mpad, 128, 0, pdl, st, args);
    if (e) return e;
  }
  GemmArgs a = {};
  a.qs = w->qs;
  a.sc = w->sc;
  a.rws = w->rws;
  a.qb = w->qb;
  a.nb = w->nb;
  a.nbp = w->nbp;
  a.N = N;
  a.K = K;
  a.xa = xa;
  a.xs = xs;
  a.out = p.splits > 1 ? part : y;
  a.M = M;
  a.Mpad = p.Mpad;
  a.mtiles = p.mtiles;
  a.ntiles = p.ntiles;
  a.splits = p.splits;
  a.kc_per_split = p.kcps;
  a.nkc = p.nkc;
  a.err = err;
  const size_t smem = 640 + 1024 + (size_t)kGStages * kStageBytes;
  static bool attr_done[2] = {false, false};
  const int qi = w->qb == 16 ? 0 : 1;
  if (!attr_done[qi]) {
    const cudaError_t e = qi == 0
        ? cudaFuncSetAttribute(gemm_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
        : cudaFuncSetAttribute(gemm_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    attr_done[qi] = true;
  }
  void* gargs[] = {&a};
  const int grid = p.ntiles * p.mtiles * p.splits;
  int e = qi == 0 ? launch_ex(gemm_tc_kernel<16>, grid, kGThreads, smem, pdl, st, gargs)
                  : launch_ex(gemm_tc_kernel<32>, grid, kGThreads, smem, pdl, st, gargs);
  if (e || p.splits == 1) return e;
  int splits = p.splits, Mi = M, Mp = p.Mpad, Ni = N;
  void* rargs[] = {&part, &splits, &Mi, &Mp, &Ni, &y};
  int rgrid = (int)(((size_t)M * N + 255) / 256);
  if (rgrid > 4096) rgrid = 4096;
  return launch_ex(gemm_reduce_kernel, rgrid, 256, 0, pdl, st, rargs);
}
