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
// accumulates W_hi X_hi + W_hi X_lo + W_lo X_hi in fp32 TMEM (the dropped
// W_lo X_lo is below 2^-22 relative) and undoes both scales exactly in the
// epilogue: results agree with the fp32 GEMV to ~1e-6 (normwise).
//
// Design (sm_100a).  The weights are the MMA's M side (128 rows of a tile,
// one per TMEM lane) and the tokens its N side (N = tokens rounded up to 16,
// at most 128 a tile), so a 16-token decode step issues 1/8 of the tensor
// work of a 128-token prefill chunk and both stream the same weight bytes.
// A persistent grid (one CTA per SM) walks work units (tile, K slice):
//   * warp 0 streams the raw GGUF blocks of its units' rows, 8 blocks (4 K
//     chunks of 64) a row per stage: one TMA tensor load of the 128 x 128-byte
//     quant box (two for Q8_0), swizzled 128B, and one of the 128 x 16-byte
//     scale box, into a shared-memory ring (mbarrier complete_tx).  Weights
//     depend on nothing, so the ring fills before the previous kernel has
//     finished;
//   * warps 2..17, four groups of four each taking every fourth K chunk,
//     turn the raw blocks into the fp16 hi / lo A operands in tensor memory
//     (one row a thread, the row in the TMEM lane of that number,
//     tcgen05.st), a ring of A stages of 64 columns beside the accumulators.
//     The tensor cores then read only the activations from shared memory:
//     with A there too, its writes and the MMAs' reads of both operands
//     (~76 KB a chunk at 16 tokens) made a chunk shared-memory bound;
//   * warp 22 bulk-copies the prepared activation parts (the B tiles) into
//     their own ring, ahead of the MMAs: for up to 32 tokens one copy covers
//     the four chunks of a weight stage (an L2-to-shared copy takes ~1.5 us
//     whatever its size, so small tiles need many chunks in flight);
//   * warp 1: one elected thread issues the tcgen05.mma into one of two TMEM
//     accumulators and commits each chunk back.  Up to 64 tokens (where the
//     MMA count, not the tensor pipe, sets the pace) the X_hi and X_lo parts
//     form one N = 2 NB operand: 2 MMAs per 16-wide K step, W_hi [X_hi X_lo]
//     and W_lo [X_hi X_lo], the two column halves added in the epilogue;
//     beyond that 3 MMAs per step (W_hi X_hi, W_hi X_lo, W_lo X_hi);
//   * warps 18..21 (epilogue) read the accumulator of the previous unit
//     (tcgen05.ld) while the next one accumulates, unscale it and store it.
// Every CTA first runs the same number of whole tiles; the tiles left over
// are cut into K slices whose partial tiles a second kernel adds in slice
// order (deterministic).
// Q4_0 chunks are dequantised in a permuted K order (word e of every 16-byte
// group holds elements e and e + 4, the order in which two mask operations
// take the nibbles out of a 32-bit word); the activation prep writes the
// same order, so the products are unchanged.  Every wait is bounded and
// reports through *err; TMEM is always released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

constexpr int kWR = 128;                  // weight rows per tile (MMA M, TMEM lanes)
constexpr int kTok = 128;                 // most tokens per tile (MMA N)
constexpr int kBK = 64;                   // K per chunk: one 128-byte fp16 row
constexpr int kRawBlk = 8;                // GGUF blocks a row per raw stage
constexpr int kRawCh = kRawBlk / 2;       // K chunks per raw stage
constexpr int kDqWarps = 4;               // dequantising warps per group (one per TMEM lane quarter)
constexpr int kDqGroups = 4;              // groups, each on every fourth K chunk
constexpr int kEpWarps = 4;
constexpr int kDq0 = 2;                                  // first dequantising warp
constexpr int kEp0 = kDq0 + kDqGroups * kDqWarps;        // first epilogue warp
constexpr int kBw = kEp0 + kEpWarps;                     // activation copy warp
constexpr int kGThreads = 32 * (kBw + 1);                // 736: six warps on some SM
                                                         // sub-partitions, 80 registers a thread
constexpr int kMaxSA = 7;                 // A stages in TMEM (weight hi/lo of one chunk)
constexpr int kMaxSB = 8;                 // B stages (activation hi/lo of one chunk)
constexpr int kMaxR = 8;                  // raw stages
constexpr int kHdrBytes = 512;
constexpr int kMaxSmem = 227 * 1024;
static_assert(kEp0 % 4 == 2, "the epilogue warps cover the four TMEM lane quarters");
static_assert((2 * kMaxR + 2 * kMaxSA + 2 * kMaxSB + 5) * 8 + 8 <= kHdrBytes, "header");

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
// M = 128; N (a multiple of 16, 16..256) goes to bits 17..22 as N / 8.
constexpr uint32_t kIdescM128 = (1u << 4) | ((uint32_t)(kWR >> 4) << 24);
__host__ __device__ constexpr uint32_t idesc_n(int n) { return kIdescM128 | ((uint32_t)(n >> 3) << 17); }

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same MMA with A (128 rows x 16 fp16) in tensor memory: lane m holds
// row m, column j its K elements 2j and 2j + 1 (low half first).
__device__ __forceinline__ void umma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
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

// 16 consecutive fp32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers
// (completion: tmem_st_wait).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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
// exact for weights (at most 19 bits in all) and keeps 11 more bits of an
// activation.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi2, uint32_t& lo2) {
  const float ta = __fmul_rn(a, 8193.0f), tb = __fmul_rn(b, 8193.0f);
  const float ha = __fsub_rn(ta, __fsub_rn(ta, a)), hb = __fsub_rn(tb, __fsub_rn(tb, b));
  const __half2 H = __floats2half2_rn(ha, hb);
  const __half2 L = __floats2half2_rn(__fsub_rn(a, ha), __fsub_rn(b, hb));
  hi2 = *reinterpret_cast<const uint32_t*>(&H);
  lo2 = *reinterpret_cast<const uint32_t*>(&L);
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<const __half2*>(&u); }

struct GemmArgs {
  CUtensorMap tq;       // weight quants [N][nb * qb] bytes: 128-byte x 128-row boxes, swizzled 128B
  CUtensorMap ts;       // weight scales [N][nbp] fp16: 8 x 128 boxes
  const float* rws;     // per-row power-of-two weight scales [N]
  int nb, nbp, N, K, nkc;
  const uint8_t* xa;    // prepared activations [mtiles][nkc][hi, lo][NB rows x 128 B]
  const float* xs;      // per-row inverse activation scales [mtiles * NB]
  float* y;             // Y [M][N] (epi 0), the residual stream [M][N] (epi 1) or H [M][N / 2] (epi 2)
  int epi;              // epilogue: 0 store, 1 add to y (residual), 2 SiLU(row 2j) * row 2j+1 into y
  float* part;          // K-slice partials [splits][M][N]
  int M, NB, mtiles, ntiles, splits, kcps, units;
  int full;             // tiles 0..full-1 run whole; the rest in `splits` K slices each
  int SA, SB, R;        // A, B and raw stages in the rings
  int bcs;              // chunks per B stage: kRawCh (one copy per weight stage) or 1
  int cat;              // 1: [X_hi X_lo] as one operand, accumulators of 2 NB columns
  uint32_t b_bytes, raw_bytes, tcols;   // b_bytes: one B stage; tcols: TMEM columns allocated
  uint32_t acols;       // TMEM columns of one accumulator (NB, or 2 NB with cat)
  uint32_t aoff;        // first TMEM column of the A stages (64 columns each: hi, lo)
  int* err;
};

// One work unit: a 128-row weight tile, a token tile and a K slice (ns
// slices of that tile in all; ns == 1 for a whole tile).  Its nst raw stages
// (4 chunks each, the last one possibly shorter) run in the order
// rot, rot + 1, ..., nst - 1, 0, ..., rot - 1 with rot = tile % nst, so CTAs
// that run units at the same time read different activation chunks (one
// order for all of them piles every CTA onto the same L2 lines); the order
// depends on the tile only, so results are the same run to run.
struct Unit {
  int mt, tile, split, ns, n0, kc0, nk, ntok, nst, rot;
};
__device__ __forceinline__ Unit unit_of(const GemmArgs& a, int u) {
  Unit w;
  if (u < a.full) {
    w.tile = u;
    w.split = 0;
    w.ns = 1;
    w.kc0 = 0;
    w.nk = a.nkc;
  } else {
    const int v = u - a.full;
    w.tile = a.full + v / a.splits;
    w.split = v % a.splits;
    w.ns = a.splits;
    w.kc0 = w.split * a.kcps;
    w.nk = min(a.nkc, w.kc0 + a.kcps) - w.kc0;
  }
  const int nt = w.tile % a.ntiles;
  w.mt = w.tile / a.ntiles;
  w.n0 = nt * kWR;
  w.ntok = min(a.NB, (a.M - w.mt * kTok + 15) & ~15);
  w.nst = (w.nk + kRawCh - 1) / kRawCh;
  w.rot = w.tile % w.nst;
  return w;
}

// First chunk (relative to kc0) and chunk count of the q-th raw stage run.
__device__ __forceinline__ int stage_c0(const Unit& w, int q) {
  const int st = q + w.rot < w.nst ? q + w.rot : q + w.rot - w.nst;
  return kRawCh * st;
}

// ---------------------------------------------------------------------------
// prep: X[M][K] fp32 -> per-row power-of-two scale s (stored as 1/s, exact)
// and fp16 hi/lo parts of X*s in the swizzled K-major layout, token tiles of
// NB rows (rows beyond M are zero).  perm: the Q4_0 K order (word e of a
// 16-byte group = elements e and e + 4 of its eight) instead of the natural
// one.  Grid: (prepared row, part of K); every CTA of a row finds the row's
// maximum, then converts its part.  nw non-null: the row is first RMS-
// normalised as llm_rmsnorm does (llm.c:416-452: ss = 1/sqrt(sum x^2 / K +
// eps), then (x ss) w) with a fixed-order tree sum of squares, so the norm
// feeding a GEMM needs no launch of its own.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) gemm_prep_kernel(const float* __restrict__ x, int M, int K, int NB,
                                                        int perm, uint8_t* __restrict__ xa,
                                                        float* __restrict__ xs, const float* __restrict__ nw,
                                                        float eps) {
  __shared__ float red[4];
  __shared__ float s_ss;
  pdl_wait();
  pdl_trigger();
  const int p = blockIdx.x;            // prepared row
  const int mt = p / NB, r = p % NB;
  const int m = mt * kTok + r;
  const int nkc = K / kBK;
  const bool valid = m < M;
  const float* xr = x + (size_t)m * K;
  // the row in 16-byte pieces, eight per thread in flight (K is a multiple
  // of 64, rows and norm weights 16-byte aligned)
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  const float4* w4 = reinterpret_cast<const float4*>(nw);
  const int K4 = K / 4, bd = (int)blockDim.x;
  float ss = 1.0f;
  if (nw) {
    float acc = 0.0f;
    if (valid)
      for (int i0 = threadIdx.x; i0 < K4; i0 += 8 * bd) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = i0 + u * bd < K4 ? x4[i0 + u * bd] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          acc = fmaf(v[u].w, v[u].w, fmaf(v[u].z, v[u].z, fmaf(v[u].y, v[u].y, fmaf(v[u].x, v[u].x, acc))));
      }
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      const float t = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
      s_ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), eps)));
    }
    __syncthreads();
    ss = s_ss;
  }
  // an element of the (normalised) row
  auto nval = [&](float xv, float wv) { return nw ? __fmul_rn(__fmul_rn(xv, ss), wv) : xv; };
  float mx = 0.0f;
  if (valid)
    for (int i0 = threadIdx.x; i0 < K4; i0 += 8 * bd) {
      float4 v[8], wv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const bool in = i0 + u * bd < K4;
        v[u] = in ? x4[i0 + u * bd] : make_float4(0.f, 0.f, 0.f, 0.f);
        wv[u] = in && nw ? w4[i0 + u * bd] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        mx = fmaxf(fmaxf(fmaxf(mx, fabsf(nval(v[u].x, wv[u].x))), fabsf(nval(v[u].y, wv[u].y))),
                   fmaxf(fabsf(nval(v[u].z, wv[u].z)), fabsf(nval(v[u].w, wv[u].w))));
    }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float s = pow2_to_2p13(mx);
  if (threadIdx.x == 0 && blockIdx.y == 0) xs[p] = 1.0f / s;
  const size_t part = (size_t)NB * 128;
  const int ng = K / 8;
  const int g1 = (int)(((long long)(blockIdx.y + 1) * ng) / gridDim.y);
  // one 16-byte group (8 elements) per thread and step
  for (int q = (int)(((long long)blockIdx.y * ng) / gridDim.y) + threadIdx.x; q < g1; q += blockDim.x) {
    const int kc = q / 8, c = q % 8;
    float g8[8];   // elements 8q .. 8q + 7, normalised
    if (valid) {
      const float4 a = x4[2 * q], b = x4[2 * q + 1];
      const float4 wa = nw ? w4[2 * q] : make_float4(1.f, 1.f, 1.f, 1.f);
      const float4 wb = nw ? w4[2 * q + 1] : make_float4(1.f, 1.f, 1.f, 1.f);
      g8[0] = nval(a.x, wa.x); g8[1] = nval(a.y, wa.y); g8[2] = nval(a.z, wa.z); g8[3] = nval(a.w, wa.w);
      g8[4] = nval(b.x, wb.x); g8[5] = nval(b.y, wb.y); g8[6] = nval(b.z, wb.z); g8[7] = nval(b.w, wb.w);
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i0 = perm ? e : 2 * e, i1 = perm ? e + 4 : 2 * e + 1;
      const float v0 = valid ? __fmul_rn(g8[i0], s) : 0.0f;
      const float v1 = valid ? __fmul_rn(g8[i1], s) : 0.0f;
      split2(v0, v1, hi[e], lo[e]);
    }
    uint8_t* blk = xa + ((size_t)mt * nkc + kc) * 2 * part;
    *reinterpret_cast<uint4*>(blk + sw128_off(r, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(blk + part + sw128_off(r, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// Q4_0 block (16 quant bytes; byte j = elements 2j (low nibble) and 2j + 1
// (high nibble), llm.c:162-165) times d*ws into fp16 hi / lo words, in the
// permuted K order: words 4k..4k+3 cover elements 8k..8k+7 as (e, e + 4).
// D = d*ws (11 significant bits, exact) = Dh (top 7 bits) + Dl (4 bits);
// (n - 8) Dh and (n - 8) Dl are exact in fp16.  A nibble n becomes 1024 + n
// (or 1024 + 16 n for a high nibble, paired with Dh/16 and Dl/16) through
// the 0x6400 exponent, so one subtraction gives (n - 8) (or 16 (n - 8)).
__device__ __forceinline__ void dequant_q4(const uint4 q, float d, float ws, uint32_t (&hi)[16],
                                           uint32_t (&lo)[16]) {
  const float D = __fmul_rn(d, ws);
  const float Dh = __uint_as_float(__float_as_uint(D) & ~((1u << 17) - 1u));
  const float Dl = __fsub_rn(D, Dh);
  const __half2 h1 = __float2half2_rn(Dh), l1 = __float2half2_rn(Dl);
  const __half2 h16 = __float2half2_rn(__fmul_rn(Dh, 0.0625f));
  const __half2 l16 = __float2half2_rn(__fmul_rn(Dl, 0.0625f));
  const __half2 k1032 = __float2half2_rn(1032.0f), k1152 = __float2half2_rn(1152.0f);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w8 = w[k] >> 8;
    const __half2 v0 = __hsub2(u2h((w[k] & 0x000F000Fu) | 0x64006400u), k1032);   // elements 0, 4
    const __half2 v1 = __hsub2(u2h((w[k] & 0x00F000F0u) | 0x64006400u), k1152);   // 1, 5 (x16)
    const __half2 v2 = __hsub2(u2h((w8 & 0x000F000Fu) | 0x64006400u), k1032);     // 2, 6
    const __half2 v3 = __hsub2(u2h((w8 & 0x00F000F0u) | 0x64006400u), k1152);     // 3, 7 (x16)
    hi[4 * k + 0] = h2u(__hmul2(v0, h1));
    lo[4 * k + 0] = h2u(__hmul2(v0, l1));
    hi[4 * k + 1] = h2u(__hmul2(v1, h16));
    lo[4 * k + 1] = h2u(__hmul2(v1, l16));
    hi[4 * k + 2] = h2u(__hmul2(v2, h1));
    lo[4 * k + 2] = h2u(__hmul2(v2, l1));
    hi[4 * k + 3] = h2u(__hmul2(v3, h16));
    lo[4 * k + 3] = h2u(__hmul2(v3, l16));
  }
}

// Q8_0 block (32 int8 quants, llm.c:199-200) times d*ws into fp16 hi / lo
// pairs in the natural K order (19 significant bits, split 11 + 8).
__device__ __forceinline__ void dequant_q8(const uint4 q0, const uint4 q1, float d, float ws,
                                           uint32_t (&hi)[16], uint32_t (&lo)[16]) {
  const float ds = __fmul_rn(d, ws);   // exact (power-of-two ws)
  const float kM = 8388736.0f;         // 2^23 + 128
  const uint32_t w[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u, q0.w ^ 0x80808080u,
                         q1.x ^ 0x80808080u, q1.y ^ 0x80808080u, q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t word = w[j >> 1];
    const uint32_t b0 = (uint32_t)((2 * j) & 3), b1 = (uint32_t)((2 * j + 1) & 3);
    const float e0 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | b0)), kM);
    const float e1 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | b1)), kM);
    split2(__fmul_rn(e0, ds), __fmul_rn(e1, ds), hi[j], lo[j]);
  }
}

// Every lane of the warp waits (each acquires the barrier's phase); the warp
// continues only if all of them saw it complete.
// 2-D TMA tensor load into this CTA's shared memory, completion counted on
// `bar` in bytes.  No multicast.  x (innermost, in elements) times the
// element size is a multiple of 16 at every call site.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// True in exactly one lane of a full warp (the lowest).
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(e));
  return e != 0;
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const bool good = mbar_wait(bar, parity, err, code);
  return __all_sync(0xffffffffu, good);
}

template <int QB>
__global__ void __launch_bounds__(kGThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ uint8_t gsm[];
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(gsm);   // [R]: raw stage landed
  uint64_t* raw_empty = raw_full + kMaxR;                  // [R]: every dequantising warp is done with it
  uint64_t* a_full = raw_empty + kMaxR;                    // [SA]: the chunk's A parts written
  uint64_t* a_empty = a_full + kMaxSA;                     // [SA]: the chunk's MMAs have read them
  uint64_t* b_full = a_empty + kMaxSA;                     // [SB]: the chunk's B parts landed
  uint64_t* b_empty = b_full + kMaxSB;                     // [SB]: the chunk's MMAs have read them
  uint64_t* tm_full = b_empty + kMaxSB;                    // [2]: accumulator final
  uint64_t* tm_empty = tm_full + 2;                        // [2]: accumulator read out
  uint64_t* drain = tm_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const uint32_t sbase = (smem_u32(gsm) + kHdrBytes + 1023) & ~1023u;
  uint8_t* bring = gsm + (sbase - smem_u32(gsm));
  uint8_t* raws = bring + (size_t)a.SB * a.b_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.R; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kDqGroups * kDqWarps);
    }
    for (int s = 0; s < a.SA; ++s) {
      mbar_init(&a_full[s], kDqWarps);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < a.SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], kEpWarps);
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, a.tcols);   // two accumulators, then the A stages
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ---------------- raw weight stages: TMA boxes of 128 rows x 8 blocks ----------------
    // (rows past N and blocks past the row end read as zeros)
    constexpr int kQBoxes = QB / 16;
    if (lane == 0) {
      int j = 0;
      for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
        const Unit w = unit_of(a, u);
        bool ok = true;
        for (int q = 0; q < w.nst; ++q, ++j) {
          const int slot = j % a.R;
          if (j >= a.R && !mbar_wait(&raw_empty[slot], ((j / a.R) - 1) & 1, a.err, 21)) {
            ok = false;
            break;
          }
          const int b0 = 2 * (w.kc0 + stage_c0(w, q));   // a multiple of 8: every box starts 16-byte aligned
          uint8_t* rq = raws + (size_t)slot * a.raw_bytes;
          mbar_arrive_expect_tx(&raw_full[slot], (uint32_t)(kQBoxes * 16384 + 2048));
#pragma unroll
          for (int qb = 0; qb < kQBoxes; ++qb)
            tma_load_2d(rq + 16384 * qb, &a.tq, b0 * QB + 128 * qb, w.n0, &raw_full[slot]);
          tma_load_2d(rq + 16384 * kQBoxes, &a.ts, b0, w.n0, &raw_full[slot]);
        }
        if (!ok) break;
      }
      // loads still in flight land before the CTA leaves (each slot's last
      // stage is the newest phase of its barrier)
      for (int jj = max(0, j - a.R); jj < j; ++jj) mbar_wait(&raw_full[jj % a.R], (jj / a.R) & 1, a.err, 28);
    }
  } else if (warp == kBw) {
    // ---------------- activation (B) parts: one bulk copy per B stage ----------------
    if (lane == 0) {
      pdl_wait();   // the prepared activations come from the prep kernel
      const uint32_t cbytes = 2u * (uint32_t)a.NB * 128u;   // hi and lo parts of one chunk
      int i = 0;    // B stages issued
      for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
        const Unit w = unit_of(a, u);
        bool ok = true;
        for (int q = 0; q < w.nst && ok; ++q) {
          const int c0 = stage_c0(w, q), cn = min(kRawCh, w.nk - c0);
          for (int c = c0; c < c0 + cn; c += a.bcs, ++i) {
            const int s = i % a.SB;
            if (i >= a.SB && !mbar_wait(&b_empty[s], ((i / a.SB) - 1) & 1, a.err, 29)) {
              ok = false;
              break;
            }
            const uint32_t bytes = (uint32_t)min(a.bcs, c0 + cn - c) * cbytes;
            mbar_arrive_expect_tx(&b_full[s], bytes);
            bulk_g2s(bring + (size_t)s * a.b_bytes, a.xa + ((size_t)w.mt * a.nkc + w.kc0 + c) * cbytes, bytes,
                     &b_full[s]);
          }
        }
        if (!ok) break;
      }
      for (int ii = max(0, i - a.SB); ii < i; ++ii) mbar_wait(&b_full[ii % a.SB], (ii / a.SB) & 1, a.err, 30);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    // The whole warp runs the loop, so the descriptors are warp-uniform;
    // one elected lane (always lane 0) issues the MMAs and their commits.
    int i = 0, v = 0, jb = 0;   // chunks, units and B stages so far
    bool ok = true, issued = false;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x, ++v) {
      const Unit w = unit_of(a, u);
      const int buf = v & 1;
      if (v >= 2 && !warp_wait(&tm_empty[buf], ((v >> 1) - 1) & 1, a.err, 22)) break;
      tc_fence_after();
      const uint32_t idesc = a.cat ? idesc_n(2 * a.NB) : idesc_n(w.ntok);
      const uint32_t d = taddr + (uint32_t)buf * a.acols;
      int c = 0;   // chunks of this unit so far (run order)
      for (int q = 0; q < w.nst && ok; ++q) {
       const int cn = min(kRawCh, w.nk - stage_c0(w, q));
       for (int cc = 0; cc < cn; ++cc, ++c, ++i) {
        const int sa = i % a.SA;
        const bool bfirst = cc % a.bcs == 0, blast = cc % a.bcs == a.bcs - 1 || cc == cn - 1;
        const int sb = jb % a.SB;
        if (!warp_wait(&a_full[sa], (i / a.SA) & 1, a.err, 23) ||
            (bfirst && !warp_wait(&b_full[sb], (jb / a.SB) & 1, a.err, 23))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ah0 = taddr + a.aoff + 64u * (uint32_t)sa, al0 = ah0 + 32u;   // A hi / lo in TMEM
        const uint32_t bh0 = smem_u32(bring + (size_t)sb * a.b_bytes) + (uint32_t)(cc % a.bcs) * 256u * a.NB;
        const uint32_t bl0 = bh0 + (uint32_t)a.NB * 128u;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t ah = ah0 + 8u * kk, al = al0 + 8u * kk;   // 16 K elements = 8 columns
            const uint64_t bh = sw128_desc(bh0 + 32 * kk), bl = sw128_desc(bl0 + 32 * kk);
            umma_f16_ta(d, ah, bh, idesc, (c > 0 || kk > 0) ? 1u : 0u);   // c counts chunks in run order
            if (a.cat) {
              umma_f16_ta(d, al, bh, idesc, 1u);   // bh spans the hi and the lo rows
            } else {
              umma_f16_ta(d, ah, bl, idesc, 1u);
              umma_f16_ta(d, al, bh, idesc, 1u);
            }
          }
          umma_commit(&a_empty[sa]);   // the chunk's operands may be refilled once read
          if (blast) umma_commit(&b_empty[sb]);
        }
        __syncwarp();
        issued = true;
        if (blast) ++jb;
       }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&tm_full[buf]);   // this unit's accumulator is final
      __syncwarp();
    }
    if (issued) {
      if (elect_one()) umma_commit(drain);   // nothing of this warp is in flight past here
      __syncwarp();
      mbar_wait(drain, 0, a.err, 27);
    }
  } else if (warp < kEp0) {
    // ---------------- dequantisation: group g takes the chunks i with i % kDqGroups == g ----------------
    // a warp reaches only TMEM lanes 32 (warp % 4) .. + 31, so it takes those
    // rows (the group's four warps cover the four lane quarters); a thread
    // dequantises both blocks of its row in the chunk
    const int g = (warp - kDq0) / kDqWarps;
    const int r = 32 * (warp & 3) + lane;   // weight row in the tile
    const uint32_t tlane = taddr + ((uint32_t)(32 * (warp & 3)) << 16) + a.aoff;
    int i = 0, j = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
      const Unit w = unit_of(a, u);
      const bool valid = w.n0 + r < a.N;
      const float ws = valid ? a.rws[w.n0 + r] : 1.0f;
      for (int q = 0; q < w.nst; ++q, ++j) {
        const int slot = j % a.R;
        if (!warp_wait(&raw_full[slot], (j / a.R) & 1, a.err, 24)) {
          ok = false;
          break;
        }
        const uint8_t* rq = raws + (size_t)slot * a.raw_bytes;
        const uint16_t* rs = reinterpret_cast<const uint16_t*>(rq + 16384 * (QB / 16));
        const int cn = min(kRawCh, w.nk - stage_c0(w, q));
        for (int c = 0; c < cn; ++c, ++i) {
          if (i % kDqGroups != g) continue;
          const int s = i % a.SA;
          if (i >= a.SA && !warp_wait(&a_empty[s], ((i / a.SA) - 1) & 1, a.err, 25)) {
            ok = false;
            break;
          }
          tc_fence_after();   // the MMAs that read this A stage are complete
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {   // the chunk's two blocks
            uint32_t hi[16], lo[16];
            if (valid) {
              const int blk = 2 * c + h;    // block of the raw stage, 0..7
              const float dd = h2f(rs[8 * r + blk]);
              if constexpr (QB == 16) {
                dequant_q4(*reinterpret_cast<const uint4*>(rq + sw128_off(r, blk)), dd, ws, hi, lo);
              } else {
                const uint8_t* box = rq + 16384 * (blk >> 2);
                dequant_q8(*reinterpret_cast<const uint4*>(box + sw128_off(r, 2 * (blk & 3))),
                           *reinterpret_cast<const uint4*>(box + sw128_off(r, 2 * (blk & 3) + 1)), dd, ws, hi, lo);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) hi[e] = lo[e] = 0u;
            }
            // row r's K elements 32 h .. 32 h + 31 of the chunk: columns 16 h ..
            // 16 h + 15 of the stage's hi and lo parts
            const uint32_t ta = tlane + 64u * (uint32_t)s + 16u * (uint32_t)h;
            tmem_st16(ta, hi);
            tmem_st16(ta + 32u, lo);
          }
          tmem_st_wait();
          tc_fence_before();   // ordered before the MMA warp's issue
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[s]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[slot]);
      }
    }
  } else {
    // ---------------- epilogue: warp q reads TMEM lanes 32q..32q+31 ----------------
    pdl_wait();   // Y and the partials: after the previous kernels
    const int q = warp & 3;
    const int r = 32 * q + lane;
    int v = 0;
    for (int u = blockIdx.x; u < a.units; u += gridDim.x, ++v) {
      const Unit w = unit_of(a, u);
      const int buf = v & 1;
      if (!warp_wait(&tm_full[buf], (v >> 1) & 1, a.err, 26)) break;
      tc_fence_after();
      const int n = w.n0 + r;
      const bool vn = n < a.N;
      const float inv_ws = vn ? 1.0f / a.rws[n] : 0.0f;   // exact: power of two
      const int m0 = w.mt * kTok;
      const int mend = min(a.M, m0 + w.ntok);
      const uint32_t tcol = taddr + ((uint32_t)(32 * q) << 16) + (uint32_t)buf * a.acols;
      // a whole tile goes to Y; a K slice to its partial plane (added by
      // the slice-sum kernel)
      float* dst = w.ns == 1 ? a.y : a.part + (size_t)w.split * a.M * a.N;
      for (int c0 = 0; c0 < w.ntok; c0 += 16) {
        float vv[16];
        tmem_ld16(tcol + (uint32_t)c0, vv);
        if (a.cat) {
          float vl[16];
          tmem_ld16(tcol + (uint32_t)(a.NB + c0), vl);
#pragma unroll
          for (int e = 0; e < 16; ++e) vv[e] = __fadd_rn(vv[e], vl[e]);
        }
        if (w.ns > 1 || a.epi == 0) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int m = m0 + c0 + e;
            if (vn && m < mend) dst[(size_t)m * a.N + n] = __fmul_rn(__fmul_rn(vv[e], a.xs[m]), inv_ws);
          }
        } else if (a.epi == 1) {
          // residual (llm.c:717-718, 732-733): x + y, as pf_add_kernel
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int m = m0 + c0 + e;
            if (vn && m < mend) {
              float* px = a.y + (size_t)m * a.N + n;
              *px = __fadd_rn(*px, __fmul_rn(__fmul_rn(vv[e], a.xs[m]), inv_ws));
            }
          }
        } else {
          // gate|up rows interleaved (2j gate, 2j + 1 up, in lanes r, r ^ 1):
          // h = SiLU(gate) * up (llm.c:726-729), as pf_swiglu_kernel
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int m = m0 + c0 + e;
            const float v = m < mend ? __fmul_rn(__fmul_rn(vv[e], a.xs[m]), inv_ws) : 0.0f;
            const float up = __shfl_xor_sync(0xffffffffu, v, 1);
            if (vn && m < mend && (n & 1) == 0) a.y[(size_t)m * (a.N >> 1) + (n >> 1)] = __fmul_rn(ref_silu(v), up);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tm_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(taddr, a.tcols);
  }
}

// ---------------------------------------------------------------------------
// Q4_0 at up to 16 tokens: exact integer block products on the tensor cores
// (tcgen05.mma kind::i8).
//
// Every 32-element block of an activation row becomes X_i = rint(x_i / s),
// s a power of two per (token, block) with max |X_i| <= 2^22 (the FAST
// GEMV's fixed point, gemv_fastmath.cuh), written as three signed byte limbs
// X = L0 + 2^8 L1 + 2^16 L2.  The weights enter as n - 8 (signed bytes, no
// scale), so one MMA of K = 32 per block (N = 48: limb l of token t in
// column 16 l + t) gives the exact sums S_l = sum_k (n_k - 8) L_l,k
// (|S_l| <= 2^15), and Y = S_0 + 2^8 S_1 + 2^16 S_2 is the block's exact
// integer value, the FAST GEMV's block value before its two roundings.  The
// warps that read the accumulators add float(Y) * (d * s) into per-row fp32
// sums.  Against the fp16 hi / lo form: one MMA per block instead of four,
// and a weight operand that is a nibble expansion (no scale, no split).
//
// Warps: 0 raw weight stages (TMA, as gemm_tc_kernel); 1 MMA issue; 2..17
// dequantise and accumulate: two groups of eight, group g taking the chunks
// (4 blocks, K = 128) i with i % 2 == g, each warp its TMEM lane quarter and
// two blocks (half h) of the chunk; 18 activation chunks (bulk copies).  A
// group owns one A stage (32 TMEM columns) and one accumulator (4 x 48
// columns): it reads out chunk i's sums, then writes chunk i + 2's weights,
// so its A-stage arrival also frees the accumulator.  At the end of a unit
// the four partial sums of a row (two groups x two halves) are added in a
// fixed order (deterministic) and the epilogue of gemm_tc_kernel runs.
// ---------------------------------------------------------------------------
constexpr int kI8Tok = 16;                                     // tokens (MMA N / 3)
constexpr int kI8N = 3 * kI8Tok;                               // MMA N
constexpr int kI8BK = 128;                                     // K per chunk: one 128-byte B row
constexpr int kI8RawCh = 2;                                    // chunks per raw stage (8 blocks)
constexpr int kI8W0 = 2;                                       // first dequantising warp
constexpr int kI8Heavy = 16;                                   // dequantising warps
constexpr int kI8Bw = kI8W0 + kI8Heavy;                        // activation copy warp
constexpr int kI8Threads = 32 * (kI8Bw + 1);                   // 608
constexpr int kI8MaxSB = 8;
constexpr int kI8MaxR = 8;
constexpr uint32_t kI8BChunk = kI8N * 128 + 4 * kI8Tok * 4;    // 6400: limb rows, then s[4 blocks][16 tokens]
constexpr uint32_t kI8BStage = 7168;                           // a B stage in shared memory (1024-aligned)
constexpr uint32_t kI8RawBytes = 16384 + 2048;                 // quant box, scale box
constexpr uint32_t kI8Acc = 4 * kI8N;                          // accumulator columns of a chunk (192)
constexpr uint32_t kI8ACols = 4 * 8;                           // A columns of a chunk (K = 32 bytes a block)
constexpr uint32_t kI8RedBytes = 3 * kI8Tok * kWR * 4;         // three partial sums [3][16][128]
static_assert(2 * kI8Acc + 2 * kI8ACols <= 512, "TMEM");
static_assert((2 * kI8MaxR + 2 * kI8MaxSB + 7) * 8 + 8 <= kHdrBytes, "header");

// Instruction descriptor: s32 accumulate, signed 8-bit A and B, both
// K-major, M = 128, N = 48.
constexpr uint32_t kIdescI8 =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kI8N >> 3) << 17) | ((uint32_t)(kWR >> 4) << 24);

// D = A B with A (128 rows x 32 signed bytes) in tensor memory: lane m holds
// row m, column j its K elements 4j .. 4j + 3 (lowest byte first).
__device__ __forceinline__ void umma_i8_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(0u)
      : "memory");
}

// 16 consecutive 32-bit accumulator columns of this warp's 32 TMEM lanes
// (completion: tmem_ld_wait).
__device__ __forceinline__ void tmem_ld16_raw(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// A Q4_0 quant word (bytes b = elements 2b (low nibble) and 2b + 1) as two
// words of signed bytes n - 8: the low nibbles (elements 0, 2, 4, 6 of the
// word's eight) and the high ones (1, 3, 5, 7).  n + 120 stays inside its
// byte; flipping bit 7 then gives n - 8 in two's complement.
__device__ __forceinline__ void q4_to_s8(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = ((w & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
  hi = (((w >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
}

struct GemmI8Args {
  CUtensorMap tq;       // weight quants, as GemmArgs
  CUtensorMap ts;       // weight scales, as GemmArgs
  const uint8_t* xb;    // prepared activation chunks [nkc][kI8BChunk]
  float* y;             // as GemmArgs
  int epi;
  float* part;          // K-slice partials [splits][M][N]
  int N, K, nkc, M, ntiles, splits, kcps, units, full;
  int* err;
};

// Work unit: a 128-row tile and a K slice (chunks of 128), its raw stages
// (two chunks each) in the rotated order of unit_of.
struct UnitI8 {
  int tile, split, ns, n0, kc0, nk, nst, rot;
};
__device__ __forceinline__ UnitI8 unit_i8(const GemmI8Args& a, int u) {
  UnitI8 w;
  if (u < a.full) {
    w.tile = u;
    w.split = 0;
    w.ns = 1;
    w.kc0 = 0;
    w.nk = a.nkc;
  } else {
    const int v = u - a.full;
    w.tile = a.full + v / a.splits;
    w.split = v % a.splits;
    w.ns = a.splits;
    w.kc0 = w.split * a.kcps;
    w.nk = min(a.nkc, w.kc0 + a.kcps) - w.kc0;
  }
  w.n0 = w.tile * kWR;
  w.nst = (w.nk + kI8RawCh - 1) / kI8RawCh;
  w.rot = w.tile % w.nst;
  return w;
}
__device__ __forceinline__ int stage_c0_i8(const UnitI8& w, int q) {
  const int st = q + w.rot < w.nst ? q + w.rot : q + w.rot - w.nst;
  return kI8RawCh * st;
}

// prep for gemm_i8_kernel: X[M][K] fp32 (RMS-normalised first when nw is
// given, exactly as gemm_prep_kernel) -> chunk c (K elements 128 c ..): 48
// K-major rows of 128 bytes, SWIZZLE_128B (row 16 l + t: limb l of token t),
// then s[4 blocks][16 tokens].  Inside each group of eight elements the K
// order is q4_to_s8's: positions 0..3 hold elements 0, 2, 4, 6 and 4..7 hold
// 1, 3, 5, 7.  Tokens t >= M are zeros with s = 0; a block holding a
// non-finite value gets X = 0 and s = NaN (as make_xfix).  Grid (16 tokens,
// parts of K); four consecutive threads make one block.
__global__ void __launch_bounds__(128) gemm_prep_i8_kernel(const float* __restrict__ x, int M, int K,
                                                           uint8_t* __restrict__ xb,
                                                           const float* __restrict__ nw, float eps) {
  __shared__ float red[4];
  __shared__ float s_ss;
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const bool valid = t < M;
  const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)(valid ? t : 0) * K);
  const float4* w4 = reinterpret_cast<const float4*>(nw);
  const int K4 = K / 4, bd = (int)blockDim.x;
  float ss = 1.0f;
  if (nw) {
    float acc = 0.0f;
    if (valid)
      for (int i0 = threadIdx.x; i0 < K4; i0 += 8 * bd) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = i0 + u * bd < K4 ? x4[i0 + u * bd] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          acc = fmaf(v[u].w, v[u].w, fmaf(v[u].z, v[u].z, fmaf(v[u].y, v[u].y, fmaf(v[u].x, v[u].x, acc))));
      }
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      const float tt = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
      s_ss = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tt, (float)K), eps)));
    }
    __syncthreads();
    ss = s_ss;
  }
  const int nblk = K / 32;
  const int g0 = 4 * (int)(((long long)blockIdx.y * nblk) / gridDim.y);
  const int g1 = 4 * (int)(((long long)(blockIdx.y + 1) * nblk) / gridDim.y);
  for (int base = g0; base < g1; base += bd) {   // g0 and bd are multiples of 4
    const int q = base + threadIdx.x;              // 8-element group: elements 8q .. 8q + 7
    const bool in = q < g1;
    float g8[8];
    if (valid && in) {
      const float4 va = x4[2 * q], vb = x4[2 * q + 1];
      g8[0] = va.x; g8[1] = va.y; g8[2] = va.z; g8[3] = va.w;
      g8[4] = vb.x; g8[5] = vb.y; g8[6] = vb.z; g8[7] = vb.w;
      if (nw) {
        const float4 wa = w4[2 * q], wb = w4[2 * q + 1];
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) g8[e] = __fmul_rn(__fmul_rn(g8[e], ss), wv[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) g8[e] = 0.0f;
    }
    float m = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(g8[e]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int eb = (int)((__float_as_uint(m) >> 23) & 0xFF);
    const int e = max(eb - 127 - 21, -126);   // max / 2^e < 2^22
    const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
    const bool fin = eb != 255;
    const float s = !valid ? 0.0f : fin ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x7FC00000u);
    uint32_t lw[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int X = valid && fin ? __float_as_int(fmaf(g8[j], inv, 12582912.0f)) - 0x4B400000 : 0;
      const int l0 = (int)(signed char)(X & 0xFF);
      const int r1 = (X - l0) >> 8;
      const int l1 = (int)(signed char)(r1 & 0xFF);
      const int l2 = (r1 - l1) >> 8;   // |l2| <= 65
      const int p = (j & 1) ? 4 + (j >> 1) : (j >> 1);   // K position of element j
      lw[0][p >> 2] |= ((uint32_t)l0 & 0xFFu) << (8 * (p & 3));
      lw[1][p >> 2] |= ((uint32_t)l1 & 0xFFu) << (8 * (p & 3));
      lw[2][p >> 2] |= ((uint32_t)l2 & 0xFFu) << (8 * (p & 3));
    }
    if (in) {
      const int kpos = 8 * q;
      const int o = kpos & (kI8BK - 1);
      uint8_t* ch = xb + (size_t)(kpos / kI8BK) * kI8BChunk;
#pragma unroll
      for (int l = 0; l < 3; ++l)
        *reinterpret_cast<uint2*>(ch + sw128_off(kI8Tok * l + t, o >> 4) + (o & 15)) = make_uint2(lw[l][0], lw[l][1]);
      if ((q & 3) == 0) reinterpret_cast<float*>(ch + kI8N * 128)[kI8Tok * (o >> 5) + t] = s;
    }
  }
}

__global__ void __launch_bounds__(kI8Threads, 1) gemm_i8_kernel(const __grid_constant__ GemmI8Args a) {
  extern __shared__ uint8_t gsm[];
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(gsm);   // [R]: raw stage landed
  uint64_t* raw_empty = raw_full + kI8MaxR;                // [R]: every dequantising warp is done with it
  uint64_t* b_full = raw_empty + kI8MaxR;                  // [SB]: activation chunk landed
  uint64_t* b_empty = b_full + kI8MaxSB;                   // [SB]: its group has read its sums and scales
  uint64_t* a_full = b_empty + kI8MaxSB;                   // [2]: group's A stage written, accumulator free
  uint64_t* acc_full = a_full + 2;                         // [2]: group's chunk MMAs complete
  uint64_t* red_full = acc_full + 2;                       // partial sums of a unit written
  uint64_t* red_empty = red_full + 1;                      // ... and read
  uint64_t* drain = red_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const uint32_t sbase = (smem_u32(gsm) + kHdrBytes + 1023) & ~1023u;
  uint8_t* bring = gsm + (sbase - smem_u32(gsm));
  uint8_t* raws = bring + (size_t)kI8MaxSB * kI8BStage;
  float* red = reinterpret_cast<float*>(raws + (size_t)kI8MaxR * kI8RawBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kI8MaxR; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kI8Heavy);
    }
    for (int s = 0; s < kI8MaxSB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], kI8Heavy / 2);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&a_full[g], kI8Heavy / 2);
      mbar_init(&acc_full[g], 1);
    }
    mbar_init(red_full, 12);   // the warps of halves 1..3
    mbar_init(red_empty, 4);   // the warps of half 0
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);   // two accumulators, then two A stages
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ---------------- raw weight stages: TMA boxes of 128 rows x 8 blocks ----------------
    if (lane == 0) {
      int j = 0;
      for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
        const UnitI8 w = unit_i8(a, u);
        bool ok = true;
        for (int q = 0; q < w.nst; ++q, ++j) {
          const int slot = j % kI8MaxR;
          if (j >= kI8MaxR && !mbar_wait(&raw_empty[slot], ((j / kI8MaxR) - 1) & 1, a.err, 41)) {
            ok = false;
            break;
          }
          const int b0 = 4 * (w.kc0 + stage_c0_i8(w, q));   // a multiple of 8: 16-byte aligned boxes
          uint8_t* rq = raws + (size_t)slot * kI8RawBytes;
          mbar_arrive_expect_tx(&raw_full[slot], kI8RawBytes);
          tma_load_2d(rq, &a.tq, b0 * 16, w.n0, &raw_full[slot]);
          tma_load_2d(rq + 16384, &a.ts, b0, w.n0, &raw_full[slot]);
        }
        if (!ok) break;
      }
      for (int jj = max(0, j - kI8MaxR); jj < j; ++jj) mbar_wait(&raw_full[jj % kI8MaxR], (jj / kI8MaxR) & 1, a.err, 42);
    }
  } else if (warp == kI8Bw) {
    // ---------------- activation chunks: one bulk copy each ----------------
    if (lane == 0) {
      pdl_wait();   // the prepared chunks come from the prep kernel
      int i = 0;
      for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
        const UnitI8 w = unit_i8(a, u);
        bool ok = true;
        for (int q = 0; q < w.nst && ok; ++q) {
          const int c0 = stage_c0_i8(w, q), cn = min(kI8RawCh, w.nk - c0);
          for (int c = c0; c < c0 + cn; ++c, ++i) {
            const int s = i % kI8MaxSB;
            if (i >= kI8MaxSB && !mbar_wait(&b_empty[s], ((i / kI8MaxSB) - 1) & 1, a.err, 43)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&b_full[s], kI8BChunk);
            bulk_g2s(bring + (size_t)s * kI8BStage, a.xb + (size_t)(w.kc0 + c) * kI8BChunk, kI8BChunk, &b_full[s]);
          }
        }
        if (!ok) break;
      }
      for (int ii = max(0, i - kI8MaxSB); ii < i; ++ii) mbar_wait(&b_full[ii % kI8MaxSB], (ii / kI8MaxSB) & 1, a.err, 44);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue: four MMAs (one a block) a chunk ----------------
    int i = 0;
    bool ok = true, issued = false;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
      const UnitI8 w = unit_i8(a, u);
      for (int q = 0; q < w.nst && ok; ++q) {
        const int cn = min(kI8RawCh, w.nk - stage_c0_i8(w, q));
        for (int cc = 0; cc < cn; ++cc, ++i) {
          const int g = i & 1, sb = i % kI8MaxSB;
          if (!warp_wait(&a_full[g], (i >> 1) & 1, a.err, 45) || !warp_wait(&b_full[sb], (i / kI8MaxSB) & 1, a.err, 46)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d0 = taddr + (uint32_t)g * kI8Acc;
          const uint32_t a0 = taddr + 2u * kI8Acc + (uint32_t)g * kI8ACols;
          const uint32_t b0 = smem_u32(bring + (size_t)sb * kI8BStage);
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              umma_i8_ta(d0 + (uint32_t)(kI8N * j), a0 + 8u * (uint32_t)j, sw128_desc(b0 + 32u * (uint32_t)j), kIdescI8);
            umma_commit(&acc_full[g]);
          }
          __syncwarp();
          issued = true;
        }
      }
    }
    if (issued) {
      if (elect_one()) umma_commit(drain);   // nothing of this warp is in flight past here
      __syncwarp();
      mbar_wait(drain, 0, a.err, 47);
    }
  } else {
    // ---------------- dequantise, accumulate, epilogue ----------------
    const int hw = warp - kI8W0;
    const int g = hw >> 3;             // group: chunks i with i % 2 == g
    const int h = (hw >> 2) & 1;       // blocks 2h, 2h + 1 of a chunk
    const int gh = hw >> 2;            // which of a row's four partial sums
    const int qd = warp & 3;           // TMEM lane quarter
    const int r = 32 * qd + lane;      // weight row in the tile
    const uint32_t tl = taddr + ((uint32_t)(32 * qd) << 16);
    const uint32_t accb = tl + (uint32_t)g * kI8Acc + (uint32_t)(2 * h * kI8N);
    const uint32_t ab = tl + 2u * kI8Acc + (uint32_t)g * kI8ACols + 16u * (uint32_t)h;
    float acc[kI8Tok];
    bool pend = false;
    int pi = 0;
    float pd0 = 0.0f, pd1 = 0.0f;
    // add the pending chunk's two blocks: float(Y) * (d * s) per token
    auto take = [&]() -> bool {
      if (!warp_wait(&acc_full[g], (pi >> 1) & 1, a.err, 48)) return false;
      tc_fence_after();
      const float* sc = reinterpret_cast<const float*>(bring + (size_t)(pi % kI8MaxSB) * kI8BStage + kI8N * 128);
#pragma unroll
      for (int jb = 0; jb < 2; ++jb) {
        uint32_t v[kI8N];
        tmem_ld16_raw(accb + (uint32_t)(kI8N * jb), v);
        tmem_ld16_raw(accb + (uint32_t)(kI8N * jb + 16), v + 16);
        tmem_ld16_raw(accb + (uint32_t)(kI8N * jb + 32), v + 32);
        tmem_ld_wait();
        const float dd = jb ? pd1 : pd0;
        const float4* s4 = reinterpret_cast<const float4*>(sc + kI8Tok * (2 * h + jb));
#pragma unroll
        for (int t4 = 0; t4 < kI8Tok / 4; ++t4) {
          const float4 sv = s4[t4];
          const float s[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 4 * t4 + e;
            const int Y = (int)(v[t] + (v[16 + t] << 8) + (v[32 + t] << 16));
            acc[t] = fmaf((float)Y, __fmul_rn(dd, s[e]), acc[t]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_empty[pi % kI8MaxSB]);
      return true;
    };
    int i = 0, j = 0, v = 0;   // chunks, raw stages, units
    bool ok = true;
    for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x, ++v) {
      const UnitI8 w = unit_i8(a, u);
#pragma unroll
      for (int t = 0; t < kI8Tok; ++t) acc[t] = 0.0f;
      for (int q = 0; q < w.nst; ++q, ++j) {
        const int slot = j % kI8MaxR;
        if (!warp_wait(&raw_full[slot], (j / kI8MaxR) & 1, a.err, 49)) {
          ok = false;
          break;
        }
        const uint8_t* rq = raws + (size_t)slot * kI8RawBytes;
        const uint16_t* rs = reinterpret_cast<const uint16_t*>(rq + 16384);
        const int cn = min(kI8RawCh, w.nk - stage_c0_i8(w, q));
        for (int c = 0; c < cn; ++c, ++i) {
          if ((i & 1) != g) continue;
          if (pend && !take()) {
            ok = false;
            break;
          }
          // blocks 4c + 2h, 4c + 2h + 1 of the raw stage into this group's A stage
          uint32_t wv[16];
          float dv[2];
#pragma unroll
          for (int jb = 0; jb < 2; ++jb) {
            const int blk = 4 * c + 2 * h + jb;
            const uint4 qv = *reinterpret_cast<const uint4*>(rq + sw128_off(r, blk));
            dv[jb] = h2f(rs[8 * r + blk]);
            q4_to_s8(qv.x, wv[8 * jb + 0], wv[8 * jb + 1]);
            q4_to_s8(qv.y, wv[8 * jb + 2], wv[8 * jb + 3]);
            q4_to_s8(qv.z, wv[8 * jb + 4], wv[8 * jb + 5]);
            q4_to_s8(qv.w, wv[8 * jb + 6], wv[8 * jb + 7]);
          }
          tmem_st16(ab, wv);
          tmem_st_wait();
          tc_fence_before();   // ordered before the MMA warp's issue
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[g]);
          pend = true;
          pi = i;
          pd0 = dv[0];
          pd1 = dv[1];
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[slot]);
      }
      if (!ok) break;
      if (pend) {
        if (!take()) break;
        pend = false;
      }
      // the row's four partial sums, added in a fixed order, then the epilogue
      pdl_wait();   // Y and the partial planes: after the previous kernels
      if (gh != 0) {
        if (v > 0 && !warp_wait(red_empty, (v - 1) & 1, a.err, 50)) break;
        float* rp = red + (size_t)(gh - 1) * kI8Tok * kWR;
#pragma unroll
        for (int t = 0; t < kI8Tok; ++t) rp[t * kWR + r] = acc[t];
        __syncwarp();
        if (lane == 0) mbar_arrive(red_full);
        continue;
      }
      if (!warp_wait(red_full, v & 1, a.err, 51)) break;
      const int n = w.n0 + r;
      const bool vn = n < a.N;
      float* dst = w.ns == 1 ? a.y : a.part + (size_t)w.split * a.M * a.N;
#pragma unroll
      for (int t = 0; t < kI8Tok; ++t) {
        const float y = __fadd_rn(__fadd_rn(__fadd_rn(acc[t], red[t * kWR + r]), red[(kI8Tok + t) * kWR + r]),
                                  red[(2 * kI8Tok + t) * kWR + r]);
        if (w.ns > 1 || a.epi == 0) {
          if (vn && t < a.M) dst[(size_t)t * a.N + n] = y;
        } else if (a.epi == 1) {
          if (vn && t < a.M) {
            float* px = a.y + (size_t)t * a.N + n;
            *px = __fadd_rn(*px, y);
          }
        } else {
          const float up = __shfl_xor_sync(0xffffffffu, y, 1);
          if (vn && t < a.M && (n & 1) == 0) a.y[(size_t)t * (a.N >> 1) + (n >> 1)] = __fmul_rn(ref_silu(y), up);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(red_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(taddr, 512);
  }
}

// The K slices of the tiles past `full`, added in slice order, then the
// epilogue of gemm_tc_kernel (epi 2: one thread per row pair).
__global__ void __launch_bounds__(256) gemm_slice_sum_kernel(const float* __restrict__ part, int splits, int M,
                                                             int N, int NB, int full, int ntiles, int rem,
                                                             int epi, float* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int pw = epi == 2 ? 2 : 1;        // columns a thread covers
  const size_t per = (size_t)NB * kWR / pw;   // threads of one tile (tokens x columns)
  const size_t total = (size_t)rem * per;
  auto sum = [&](int m, int n) {
    float acc = part[(size_t)m * N + n];
    for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, part[((size_t)s * M + m) * N + n]);
    return acc;
  };
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = full + (int)(i / per);
    const int wi = (int)(i % per);
    const int m = (t / ntiles) * kTok + wi / (kWR / pw);
    const int n = (t % ntiles) * kWR + pw * (wi % (kWR / pw));
    if (m >= M || n >= N) continue;
    if (epi == 0) y[(size_t)m * N + n] = sum(m, n);
    else if (epi == 1) y[(size_t)m * N + n] = __fadd_rn(y[(size_t)m * N + n], sum(m, n));
    else y[(size_t)m * (N >> 1) + (n >> 1)] = __fmul_rn(ref_silu(sum(m, n)), sum(m, n + 1));
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
  int mtiles, ntiles, nkc, NB, splits, kcps, units, grid, SA, SB, R, full, bcs, cat;
  uint32_t b_bytes, raw_bytes, tcols, acols, aoff;
  size_t off_xs, off_part, bytes, smem;
};

size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

// Ring sizes from the token tile, then the schedule: every CTA first runs
// the same number of whole tiles, then the tiles left over (fewer than the
// SMs) are cut into K slices so that they spread over the grid.  The slice
// count trades idle SMs in that last round against the slices' reduction.
// A chunk costs the slowest of its weight bytes at the per-SM share of HBM
// bandwidth, its MMAs' tensor time, their issue and its dequantisation; the
// slice sum costs a launch and its traffic (estimates in ns).
// Deterministic in (M, N, K, qb) on a given device.
GemmPlan gemm_plan(int M, int N, int K, int qb) {
  GemmPlan p = {};
  p.mtiles = (M + kTok - 1) / kTok;
  p.NB = min(kTok, (M + 15) & ~15);
  p.ntiles = (N + kWR - 1) / kWR;
  p.nkc = K / kBK;
  p.raw_bytes = (uint32_t)(16384 * (qb / 16) + 2048);   // quant box(es), then the scale box
  p.bcs = p.NB <= 32 ? kRawCh : 1;
  p.b_bytes = (uint32_t)(2 * p.NB * 128 * p.bcs);
  p.cat = p.NB <= 64 ? 1 : 0;
  // TMEM (512 columns, one CTA per SM): two accumulators, then the A
  // stages of 64 columns (hi and lo parts of a 64-wide K chunk)
  p.tcols = 512;
  p.acols = (uint32_t)(p.cat ? 2 * p.NB : p.NB);
  p.aoff = 2 * p.acols;
  p.SA = (int)min((uint32_t)kMaxSA, (p.tcols - p.aoff) / 64u);
  p.SB = p.NB <= 32 ? 4 : p.NB >= 96 ? 3 : 4;
  const size_t avail = (size_t)kMaxSmem - kHdrBytes - 1024;
  for (;; --p.SB) {
    const size_t used = (size_t)p.SB * p.b_bytes;
    p.R = used < avail ? (int)min((size_t)kMaxR, (avail - used) / p.raw_bytes) : 0;
    if (p.R >= 2 || p.SB == 2) break;
  }
  p.smem = (size_t)kHdrBytes + 1024 + (size_t)p.SB * p.b_bytes + (size_t)p.R * p.raw_bytes;

  const int tiles = p.mtiles * p.ntiles;
  const int sms = tosk_num_sms();
  const double t_mem = 256.0 * (qb + 2) / (6500.0 / sms);
  const double t_mma = 3.0 * kWR * p.NB * kBK / 5600.0;
  const double t_dq = qb == 16 ? 95.0 : 250.0;
  // the tensor core's pace for a chunk's MMAs (measured: ~0.75 us a chunk at
  // 16 tokens, 8 MMAs of N = 32; ~1.4 us at 128, 12 MMAs of N = 128)
  const double t_issue = p.cat ? 8 * 90.0 : 12 * 115.0;
  const double tc = fmax(fmax(t_mem, t_issue), fmax(t_mma, t_dq));
  const int rounds = tiles / sms;
  const int rem = tiles - rounds * sms;
  p.full = rounds * sms;
  p.kcps = (p.nkc + 3) & ~3;
  p.splits = 1;
  double best = 1e300;
  if (rem > 0) {
    for (int kcps = 4; kcps <= ((p.nkc + 3) & ~3); kcps += 4) {
      const int splits = (p.nkc + kcps - 1) / kcps;
      if (splits > 64) continue;
      const int last = (rem * splits + sms - 1) / sms;
      const double red = splits > 1 ? 2500.0 + (splits + 1.0) * rem * p.NB * kWR * 4.0 / 6500.0 : 0.0;
      const double t = last * (min(kcps, p.nkc) * tc + 200.0) + red;
      if (t < best * 0.999) {
        best = t;
        p.kcps = kcps;
        p.splits = splits;
      }
    }
  }
  p.units = p.full + rem * p.splits;
  p.grid = min(sms, p.units);
  const size_t part = (size_t)p.NB * 128;
  p.off_xs = up256((size_t)p.mtiles * p.nkc * 2 * part);
  p.off_part = up256(p.off_xs + (size_t)p.mtiles * p.NB * 4);
  p.bytes = p.off_part + (p.splits > 1 ? (size_t)p.splits * M * N * 4 : 0);
  return p;
}

struct GemmI8Plan {
  int nkc, ntiles, splits, kcps, units, full, grid, SB, R;
  size_t off_part, bytes, smem;
};

// Schedule of gemm_i8_kernel, as gemm_plan: every CTA first runs the same
// number of whole tiles, the tiles left over are cut into K slices of an
// even number of chunks.  A chunk (4 blocks of 128 rows) costs about its
// weight bytes at the per-SM share of HBM bandwidth; a unit adds its
// pipeline fill (estimates in ns).
GemmI8Plan gemm_plan_i8(int M, int N, int K) {
  GemmI8Plan p = {};
  p.nkc = K / kI8BK;
  p.ntiles = (N + kWR - 1) / kWR;
  p.SB = kI8MaxSB;
  const size_t fixed = (size_t)kHdrBytes + 1024 + (size_t)p.SB * kI8BStage + kI8RedBytes;
  p.R = (int)min((size_t)kI8MaxR, ((size_t)kMaxSmem - fixed) / kI8RawBytes);
  p.smem = fixed + (size_t)p.R * kI8RawBytes;
  const int sms = tosk_num_sms();
  const double tc = 4.0 * 18.0 * kWR / (6500.0 / sms);
  const int rounds = p.ntiles / sms;
  const int rem = p.ntiles - rounds * sms;
  p.full = rounds * sms;
  p.kcps = (p.nkc + 1) & ~1;
  p.splits = 1;
  double best = 1e300;
  if (rem > 0) {
    for (int kcps = 2; kcps <= ((p.nkc + 1) & ~1); kcps += 2) {
      const int splits = (p.nkc + kcps - 1) / kcps;
      if (splits > 64) continue;
      const int last = (rem * splits + sms - 1) / sms;
      const double red = splits > 1 ? 2500.0 + (splits + 1.0) * rem * kI8Tok * kWR * 4.0 / 6500.0 : 0.0;
      const double t = last * (min(kcps, p.nkc) * tc + 1000.0) + red;
      if (t < best * 0.999) {
        best = t;
        p.kcps = kcps;
        p.splits = splits;
      }
    }
  }
  p.units = p.full + rem * p.splits;
  p.grid = min(sms, p.units);
  p.off_part = up256((size_t)p.nkc * kI8BChunk);
  p.bytes = p.off_part + (p.splits > 1 ? (size_t)p.splits * M * N * 4 : 0);
  return p;
}

template <typename Kern>
int launch_ex(Kern kern, dim3 grid, int threads, size_t smem, int pdl, cudaStream_t st, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependency on the driver library).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// Largest workspace of any call with at most M rows (a caller sizes the
// workspace once for its longest batch and then runs shorter ones).
extern "C" size_t tosk_gemm_ws_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % kBK) return 0;
  size_t best = 0;
  for (int m = 16;; m += 16) {
    const int mm = min(m, M);
    for (int qb = 16; qb <= 32; qb += 16) {
      const size_t b = gemm_plan(mm, N, K, qb).bytes;
      if (b > best) best = b;
    }
    if (mm <= kI8Tok && K % kI8BK == 0) best = max(best, gemm_plan_i8(mm, N, K).bytes);
    if (mm == M) break;
  }
  return best;
}

namespace {
// Tensor maps of the two weight planes (host-side encoding, no device work):
// quants in 128-byte x 128-row boxes (SWIZZLE_128B), scales in 8 x 128 boxes.
int weight_maps(const tosk_qmat_t* w, CUtensorMap* tq, CUtensorMap* ts) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return (int)cudaErrorNotSupported;
  const int N = w->rows;
  const cuuint32_t es[2] = {1, 1};
  const cuuint64_t qdim[2] = {(cuuint64_t)w->nb * w->qb, (cuuint64_t)N};
  const cuuint64_t qstr[1] = {(cuuint64_t)w->nb * w->qb};
  const cuuint32_t qbox[2] = {128, (cuuint32_t)kWR};
  const cuuint64_t sdim[2] = {(cuuint64_t)w->nbp, (cuuint64_t)N};
  const cuuint64_t sstr[1] = {(cuuint64_t)w->nbp * 2};
  const cuuint32_t sbox[2] = {(cuuint32_t)kRawBlk, (cuuint32_t)kWR};
  if (enc(tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)w->qs, qdim, qstr, qbox, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      enc(ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void*)w->sc, sdim, sstr, sbox, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return (int)cudaErrorInvalidValue;
  return 0;
}

// Q4_0 at up to 16 tokens (gemm_i8_kernel): prep, GEMM, and the slice sum
// when the last tiles were cut into K slices.
int gemm_i8(const tosk_qmat_t* w, const float* x, const float* nw, float eps, int M, float* y, int epi, void* ws,
            size_t ws_bytes, int* err, int pdl, cudaStream_t st) {
  const int N = w->rows, K = w->cols;
  const GemmI8Plan p = gemm_plan_i8(M, N, K);
  // the kernel's rings are compile-time sized (no division by a ring size in its loops)
  if (ws_bytes < p.bytes || p.R != kI8MaxR || p.SB != kI8MaxSB || p.smem > (size_t)kMaxSmem)
    return (int)cudaErrorInvalidValue;
  uint8_t* xb = (uint8_t*)ws;
  float* part = (float*)((uint8_t*)ws + p.off_part);
  {
    int Mi = M, Ki = K;
    float epsv = eps;
    void* args[] = {(void*)&x, &Mi, &Ki, &xb, (void*)&nw, &epsv};
    const int kparts = max(1, min(K / 32 / 32, (4 * tosk_num_sms() + kI8Tok - 1) / kI8Tok));
    const int e = launch_ex(gemm_prep_i8_kernel, dim3(kI8Tok, kparts), 128, 0, pdl, st, args);
    if (e) return e;
  }
  GemmI8Args a = {};
  if (const int e = weight_maps(w, &a.tq, &a.ts)) return e;
  a.xb = xb;
  a.y = y;
  a.epi = epi;
  a.part = part;
  a.N = N;
  a.K = K;
  a.nkc = p.nkc;
  a.M = M;
  a.ntiles = p.ntiles;
  a.splits = p.splits;
  a.kcps = p.kcps;
  a.units = p.units;
  a.full = p.full;
  a.err = err;
  static bool attr_done = false;
  if (!attr_done) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return (int)e;
    attr_done = true;
  }
  void* gargs[] = {&a};
  const int e = launch_ex(gemm_i8_kernel, p.grid, kI8Threads, p.smem, pdl, st, gargs);
  if (e || p.splits == 1 || p.ntiles == p.full) return e;
  int sp = p.splits, Mi = M, Ni = N, NBi = kI8Tok, full = p.full, nti = p.ntiles, rem = p.ntiles - p.full, ep = epi;
  void* rargs[] = {&part, &sp, &Mi, &Ni, &NBi, &full, &nti, &rem, &ep, &y};
  const size_t total = (size_t)rem * kI8Tok * kWR;
  const int rgrid = (int)min((size_t)tosk_num_sms() * 8, (total + 255) / 256);
  return launch_ex(gemm_slice_sum_kernel, rgrid, 256, 0, pdl, st, rargs);
}

int gemm_q(const tosk_qmat_t* w, const float* x, const float* nw, float eps, int M, float* y, int epi, void* ws,
           size_t ws_bytes, int* err, int pdl, cudaStream_t st) {
  if (!w || !x || !y || !ws || M <= 0 || (w->qb != 16 && w->qb != 32)) return (int)cudaErrorInvalidValue;
  const int N = w->rows, K = w->cols;
  if (epi == 2 && (N & 1)) return (int)cudaErrorInvalidValue;
  if (K % kBK || (reinterpret_cast<uintptr_t>(ws) & 255)) return (int)cudaErrorInvalidValue;
  if (w->qb == 16 && M <= kI8Tok && K % kI8BK == 0) return gemm_i8(w, x, nw, eps, M, y, epi, ws, ws_bytes, err, pdl, st);
  const GemmPlan p = gemm_plan(M, N, K, w->qb);
  if (ws_bytes < p.bytes || p.R < 2 || p.smem > (size_t)kMaxSmem) return (int)cudaErrorInvalidValue;
  uint8_t* xa = (uint8_t*)ws;
  float* xs = (float*)((uint8_t*)ws + p.off_xs);
  float* part = (float*)((uint8_t*)ws + p.off_part);
  {
    int Mi = M, Ki = K, NBi = p.NB, perm = w->qb == 16 ? 1 : 0;
    float epsv = eps;
    void* args[] = {(void*)&x, &Mi, &Ki, &NBi, &perm, &xa, &xs, (void*)&nw, &epsv};
    const int rows = p.mtiles * p.NB;
    const int kparts = max(1, min(K / 8 / 128, (4 * tosk_num_sms() + rows - 1) / rows));
    const int e = launch_ex(gemm_prep_kernel, dim3(rows, kparts), 128, 0, pdl, st, args);
    if (e) return e;
  }
  GemmArgs a = {};
  if (const int e = weight_maps(w, &a.tq, &a.ts)) return e;
  a.rws = w->rws;
  a.nb = w->nb;
  a.nbp = w->nbp;
  a.N = N;
  a.K = K;
  a.nkc = p.nkc;
  a.xa = xa;
  a.xs = xs;
  a.y = y;
  a.epi = epi;
  a.part = part;
  a.M = M;
  a.NB = p.NB;
  a.mtiles = p.mtiles;
  a.ntiles = p.ntiles;
  a.splits = p.splits;
  a.kcps = p.kcps;
  a.units = p.units;
  a.full = p.full;
  a.SA = p.SA;
  a.SB = p.SB;
  a.bcs = p.bcs;
  a.cat = p.cat;
  a.R = p.R;
  a.b_bytes = p.b_bytes;
  a.raw_bytes = p.raw_bytes;
  a.tcols = p.tcols;
  a.acols = p.acols;
  a.aoff = p.aoff;
  a.err = err;
  static bool attr_done[2] = {false, false};
  const int qi = w->qb == 16 ? 0 : 1;
  if (!attr_done[qi]) {
    const cudaError_t e = qi == 0
        ? cudaFuncSetAttribute(gemm_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem)
        : cudaFuncSetAttribute(gemm_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return (int)e;
    attr_done[qi] = true;
  }
  void* gargs[] = {&a};
  const int e = qi == 0 ? launch_ex(gemm_tc_kernel<16>, p.grid, kGThreads, p.smem, pdl, st, gargs)
                        : launch_ex(gemm_tc_kernel<32>, p.grid, kGThreads, p.smem, pdl, st, gargs);
  const int tiles = p.mtiles * p.ntiles;
  if (e || p.splits == 1 || tiles == p.full) return e;
  int sp = p.splits, Mi = M, Ni = N, NBi = p.NB, full = p.full, nti = p.ntiles, rem = tiles - p.full, ep = epi;
  void* rargs[] = {&part, &sp, &Mi, &Ni, &NBi, &full, &nti, &rem, &ep, &y};
  const size_t total = (size_t)rem * p.NB * kWR;
  const int rgrid = (int)min((size_t)tosk_num_sms() * 8, (total + 255) / 256);
  return launch_ex(gemm_slice_sum_kernel, rgrid, 256, 0, pdl, st, rargs);
}
}  // namespace

extern "C" int tosk_gemm_q(const tosk_qmat_t* w, const float* x, int M, float* y, void* ws, size_t ws_bytes,
                           int* err, int pdl, cudaStream_t st) {
  return gemm_q(w, x, nullptr, 0.0f, M, y, 0, ws, ws_bytes, err, pdl, st);
}

extern "C" int tosk_gemm_q_norm(const tosk_qmat_t* w, const float* x, const float* norm_w, float eps, int M,
                                float* y, void* ws, size_t ws_bytes, int* err, int pdl, cudaStream_t st) {
  if (!norm_w) return (int)cudaErrorInvalidValue;
  return gemm_q(w, x, norm_w, eps, M, y, 0, ws, ws_bytes, err, pdl, st);
}

extern "C" int tosk_gemm_q_residual(const tosk_qmat_t* w, const float* x, int M, float* res, void* ws,
                                    size_t ws_bytes, int* err, int pdl, cudaStream_t st) {
  return gemm_q(w, x, nullptr, 0.0f, M, res, 1, ws, ws_bytes, err, pdl, st);
}

extern "C" int tosk_gemm_q_norm_swiglu(const tosk_qmat_t* w, const float* x, const float* norm_w, float eps,
                                       int M, float* h, void* ws, size_t ws_bytes, int* err, int pdl,
                                       cudaStream_t st) {
  if (!norm_w) return (int)cudaErrorInvalidValue;
  return gemm_q(w, x, norm_w, eps, M, h, 2, ws, ws_bytes, err, pdl, st);
}
