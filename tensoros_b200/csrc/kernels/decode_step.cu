// decode_step.cu - the whole greedy decode step of one token in one
// persistent kernel (TensorOS runtime/nn llm_forward_token, llm.c:641-743,
// and llm_argmax, llm.c:1129-1140), FAST arithmetic.
//
// Why one kernel: a batch-1 decode step is ~160 dependent GEMVs and attention
// passes, each a few microseconds long.  As separate launches every one pays
// its CTA start-up and the DRAM latency of its first weight stage, and the
// next launch cannot prefetch (its CTAs need the shared memory the previous
// kernel still holds).  Here one CTA per SM stays resident for the token:
//
//   * warp 0 (the producer) streams the weight planes of EVERY projection of
//     the step, in execution order, through a 3-slot shared-memory ring of
//     41.5 KB stages (cp.async.bulk with an L2 evict-first policy, mbarrier
//     complete_tx).  Weights depend on nothing, so the producer only waits
//     for free slots: while the other warps wait at a grid barrier or run
//     attention, the next projection's rows are already landing.
//   * warps 4..15 (compute) stage the phase's input vector in shared memory
//     (coalesced cp.async, every chunk once per CTA); thread (b, g) then
//     turns block b (RMSNorm weight applied) into a fixed-point record in
//     registers and evaluates block b of rows g, g + rg, ... of
//     each ring stage as the FAST GEMV does (integer dp4a dot products on
//     24-bit fixed-point x, gemv_fastmath.cuh) into a partials tile;
//   * warps 1..3 (chain) compute a RMSNorm phase's 1/rms from the whole
//     input vector, add each row's partials in a fixed tree order, scale
//     the row by 1/rms and run the fused epilogue (RoPE + KV store, residual
//     add, SiLU*up, logits with a running argmax); during the q|k|v
//     projection they prefetch into L2 the K and V rows the CTA's attention
//     reads next;
//   * between dependent phases all 148 CTAs meet at a grid barrier (an
//     atomic counter in global memory, release/acquire at GPU scope, every
//     wait bounded).  Attention runs on the 15 worker warps: up to 1024
//     positions one CTA per head in one phase, beyond that the split-K
//     scores / softmax*V passes of attention.cu's FAST mode.
//
// Each CTA owns the same contiguous row range of a given projection in every
// layer, so the residual rows it adds to are the rows it wrote (no extra
// barrier for the residual), and every vector another CTA wrote is read
// through L2 (ld.global.cg, cp.async.cg).
//
// Numerics: FAST (tolerance 1e-4 normwise to the reference, greedy ids equal
// to the exact path on every tested configuration).  Block values and the
// fixed-point conversion are those of the FAST GEMV; row sums, the RMSNorm
// sum of squares and the attention passes use fixed tree orders, so results
// are deterministic run to run.
//
// Launch: cooperative (all CTAs co-resident), one per SM.  Every wait is
// bounded (tos::kWaitCycles); a wait that runs out records a code in the
// step's error word and the CTAs leave together at the next grid barrier.
#include <cuda_runtime.h>

#include "gemv_common.cuh"
#include "gemv_fastmath.cuh"

namespace tos {
namespace step {

// 16 warps (four per SM sub-partition) leave 128 registers a thread: room
// for four rows of block values in flight per compute thread
constexpr int kThreads = 512;            // warp 0 producer, 1..3 chain, 4..15 compute
constexpr int kChain = 3;
constexpr int kCompute = 12;
constexpr int kWorkers = kThreads - 32;  // chain + compute threads
constexpr int kSlot = 41472;             // ring slot: 18 rows of a 4096-column Q4_0 matrix
constexpr int kSlots = 3;
constexpr int kHdr = 2048;
constexpr int kPreRows = 128;           // residual rows a CTA can stage for its epilogue
constexpr int kXBytes = 58368;           // the phase's input vector and norm weights; attention scratch
constexpr int kPBytes = 28512;           // partials tile (also attention scratch)
constexpr int kSmem = kHdr + kXBytes + kPBytes + kSlots * kSlot;
static_assert(kSmem <= 227 * 1024, "shared memory");
constexpr int kGW = 5;                   // worker warps per long-context attention group
constexpr int kGroups = kWorkers / 32 / kGW;   // three groups: all fifteen worker warps
constexpr int kChunk = 16 * kGW;         // attention positions per chunk (16 per warp)
constexpr int kMaxHd = 256;
constexpr int kMaxGrid = 1024;
constexpr int kHeadMaxN = 1024;          // longest context of the one-phase-per-head attention
constexpr int kNW = kWorkers / 32;       // worker warps
enum { K_QKV = 0, K_O = 1, K_GU = 2, K_D = 3, K_LM = 4, K_N = 5 };
// named barriers (0 is __syncthreads)
enum { B_COMPUTE = 1, B_WORKERS = 2, B_CHAIN = 3, B_GROUP0 = 4, B_STAGED = 4 + kWorkers / 32 / 4 };
static_assert(B_STAGED <= 15, "named barriers");

// Geometry of one projection (the same in every layer).
struct Geo {
  int R, nb, nbp, qb, unit, tr, pstride, sc_off;
};

struct Params {
  tosk_step_t s;
  int ll;          // vectors handed between phases as exchange words (peer_ll set; always when sharded)
  Geo g[K_N];
  float* S;        // attention workspace (the FAST attention layout)
  float* cmax;
  float* lsum;
  float* opart;
  int* cnt;
  int maxc;
};

struct Hdr {
  uint64_t full[kSlots];
  uint64_t empty[kSlots];
  uint64_t pfull[kChain];
  uint64_t pempty[kChain];
  int abort;
  int tok, pos, skip;
  unsigned ebase;   // epoch of the last cross-GPU barrier before this step (sharded)
  unsigned efinal;  // epoch of this step's argmax exchange (sharded)
  float cpart[kChain];   // the chain warps' partial sums of squares (RMSNorm)
  float av[kChain];
  int ai[kChain];
  // epilogue operands the chain warps stage while the compute warps stage
  // the input vector: this CTA's residual rows, RoPE (cos, sin) of pos
  float res[kPreRows];
  float2 cs[kMaxHd / 2];
};
static_assert(sizeof(Hdr) <= kHdr, "header");

// Attention scratch of one group inside the partials area (floats).
// es[kChunk] | red[12] (kGW maxima, kGW sums; 16-byte padded) | wpart[kGW][kMaxHd] | s_last
constexpr int kGroupFloats = kChunk + 12 + kGW * kMaxHd + 8;
static_assert((kChunk + 12) % 4 == 0 && kGroupFloats % 4 == 0 && 2 * kGW <= 12, "attention scratch alignment");
static_assert(B_GROUP0 + kGroups <= B_STAGED, "named barriers");
static_assert(kGroups * kGroupFloats * 4 <= kPBytes, "attention scratch");
static_assert((1024 + (kWorkers / 32) * kMaxHd + 32) * 4 <= kXBytes, "per-head attention scratch");

// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or ~the hint passes) instead of spinning, so the producer and
// the chain warps, which wait most of the time, leave the issue slots to the
// compute warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool wait_mb(uint64_t* bar, uint32_t parity, int* err, int code,
                                        volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (int i = 0;; ++i) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 15) == 0) {
      if (*abort) return false;
      if (clock64() - t0 > kWaitCycles) {
        atomicCAS(err, 0, code);
        *abort = 1;
        return false;
      }
    }
  }
}

// L2 policies: weights are read once per token (evict first, so they do
// not push out the KV rows and vectors the step reuses); KV rows prefetched
// for the coming attention stay (evict last).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// bulk copy global -> shared with an L2 policy (no multicast)
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// prefetch [src, src + bytes) into L2 (bytes a multiple of 16, 16-byte aligned)
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(pol)
               : "memory");
}

// 16-byte asynchronous copy global -> shared through L2 (cp.async.cg)
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier for the worker threads of every CTA: the k-th call waits for
// the counter to reach k * gridDim.x.  The CTA's writes are ordered before
// its arrival by the CTA barrier and the release reduction (cumulative), and
// the acquire load that sees the count orders the other CTAs' writes before
// everything after the closing CTA barrier.  Returns false, in every worker
// thread of the CTA alike, when the step must stop (an error here or
// elsewhere).
__device__ __forceinline__ bool grid_sync(Hdr* h, unsigned* bar, unsigned target, int* err) {
  named_sync(B_WORKERS, kWorkers);
  if (threadIdx.x == 32 && !*reinterpret_cast<volatile int*>(&h->abort)) {
    red_release_add(bar, 1u);
    const long long t0 = clock64();
    for (int i = 0;; ++i) {
      if (ld_acquire(bar) >= target) break;
      __nanosleep(32);
      if ((i & 7) == 7) {
        if (*reinterpret_cast<volatile int*>(err)) {
          h->abort = 1;
          break;
        }
        if (clock64() - t0 > kWaitCycles) {
          atomicCAS(err, 0, 20);
          h->abort = 1;
          break;
        }
      }
    }
  }
  named_sync(B_WORKERS, kWorkers);
  return !*reinterpret_cast<volatile int*>(&h->abort);
}

// Exchange words of a sharded step: {value bits, epoch} as one 8-byte
// access, so a reader that sees the epoch sees the value with it (no fence
// between them; the same idea as NCCL's low-latency protocol).  Volatile
// accesses: every poll goes to L2, where the peers' NVLink stores land.
__device__ __forceinline__ void ll_store(unsigned long long* p, uint32_t v, uint32_t e) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v), "r"(e) : "memory");
}
__device__ __forceinline__ void ll_store2(unsigned long long* p, uint32_t v0, uint32_t v1, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v0), "r"(e), "r"(v1), "r"(e)
               : "memory");
}
// two words (16-byte aligned): x, z values; y, w epochs
__device__ __forceinline__ uint4 ll_load2(const unsigned long long* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// A projection's geometry in registers: read once from the kernel
// parameters and kept opaque to the compiler, which would otherwise reload
// it inside the stage loops (a constant load with a computed index issues
// on the narrow ADU pipe).
__device__ __forceinline__ Geo geo_regs(const Params& p, int kind) {
  Geo g = p.g[kind];
  asm volatile("" : "+r"(g.R), "+r"(g.nb), "+r"(g.nbp), "+r"(g.qb), "+r"(g.unit), "+r"(g.tr), "+r"(g.pstride),
               "+r"(g.sc_off));
  return g;
}

__device__ __forceinline__ void row_range(const Geo& G, int& rb, int& re, int& nst) {
  const int NU = (G.R + G.unit - 1) / G.unit;
  const int u0 = (int)(((long long)blockIdx.x * NU) / gridDim.x);
  const int u1 = (int)(((long long)(blockIdx.x + 1) * NU) / gridDim.x);
  rb = u0 * G.unit;
  re = min(u1 * G.unit, G.R);
  nst = re > rb ? (re - rb + G.tr - 1) / G.tr : 0;
}

__device__ __forceinline__ void planes(const Params& p, int kind, int layer, const uint8_t*& qs,
                                       const uint16_t*& sc) {
  if (kind == K_LM) {
    qs = p.s.lm_qs;
    sc = p.s.lm_sc;
  } else {
    const tosk_step_layer_t& L = p.s.layers[layer];
    qs = L.qs[kind];
    sc = L.sc[kind];
  }
}

// The phases of one token in order: per layer q|k|v, scores, softmax*V, o,
// gate|up, down; then the LM head.  Weight-streaming phases only.
__device__ __forceinline__ int gemv_kind_of(int i, int n_layers, int& layer) {
  if (i >= 4 * n_layers) {
    layer = n_layers;
    return K_LM;
  }
  layer = i >> 2;
  return i & 3;
}

// (value, index) order of llm_argmax (llm.c:1129-1140) for partial results:
// a larger value wins, equal values go to the lower index, NaNs never win
// (index -1 marks "no candidate").  Associative and commutative, so the
// result does not depend on the order partial results are combined in.
__device__ __forceinline__ void arg_better(float& v, int& i, float v2, int i2) {
  if (i2 < 0) return;
  if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// Word offsets of the exchange area (the same on every rank): attention
// output [q_full], residual after o [dim], SwiGLU output [ff], residual
// after down [dim], argmax pairs [2 * TOSK_MAX_WORLD].
enum { X_ATT = 0, X_XO = 1, X_H = 2, X_XD = 3 };
__device__ __forceinline__ size_t ll_off(const Params& p, int kind) {
  const size_t q = (size_t)p.s.q_full, d = (size_t)p.s.dim, f = (size_t)p.s.ff;
  switch (kind) {
    case X_ATT: return 0;
    case X_XO: return q;
    case X_H: return q + d;
    case X_XD: return q + d + f;
    default: return q + 2 * d + f;   // pairs
  }
}
// Epoch of exchange `kind` of layer `layer` in this step.
__device__ __forceinline__ uint32_t ll_epoch(const Hdr* h, int layer, int kind) {
  return h->ebase + 4u * (uint32_t)layer + (uint32_t)kind + 1u;
}
// Element i of an exchanged vector into every rank's area.
__device__ __forceinline__ void ll_store_all(const Params& p, int kind, size_t i, float v, uint32_t e) {
  const size_t w = ll_off(p, kind) + i;
  for (int r = 0; r < p.s.world; ++r) ll_store(p.s.peer_ll[r] + w, __float_as_uint(v), e);
}
// Waits (bounded) until both words of a pair carry epoch e; false when the
// step must stop.  (Out of line: the spin is the rare path.)
__device__ __noinline__ bool ll_wait(const unsigned long long* w, uint4& v, uint32_t e, Hdr* h, int* err) {
  const long long t0 = clock64();
  for (int i = 0;; ++i) {
    __nanosleep(20);
    v = ll_load2(w);
    if (v.y == e && v.w == e) return true;
    if ((i & 15) == 15) {
      if (*reinterpret_cast<volatile int*>(&h->abort)) return false;
      if (clock64() - t0 > kWaitCycles) {
        atomicCAS(err, 0, 21);
        h->abort = 1;
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool ll_ready(const unsigned long long* w, uint4& v, uint32_t e, Hdr* h, int* err) {
  return (v.y == e && v.w == e) || ll_wait(w, v, e, h, err);
}
// Every worker thread of this CTA (the phases of a sharded step hand their
// vectors over through the exchange words, not through grid barriers);
// false, in all of them alike, when the step must stop.
__device__ __forceinline__ bool cta_sync(Hdr* h) {
  named_sync(B_WORKERS, kWorkers);
  const bool ok = !*reinterpret_cast<volatile int*>(&h->abort);
  named_sync(B_WORKERS, kWorkers);
  return ok;
}

// ---------------------------------------------------------------------------
// producer: every weight stage of the step, in order
// ---------------------------------------------------------------------------
__device__ __forceinline__ void producer(const Params& p, Hdr* h, uint8_t* ring) {
  int* err = p.s.io + 3;
  int gs = 0;
  bool ok = true;
  const uint64_t pol = policy_evict_first();
  const int nphase = 4 * p.s.n_layers + 1;
  for (int i = 0; i < nphase && ok; ++i) {
    int layer;
    const int kind = gemv_kind_of(i, p.s.n_layers, layer);
    const Geo G = geo_regs(p, kind);
    const uint8_t* qs;
    const uint16_t* sc;
    planes(p, kind, layer, qs, sc);
    int rb, re, nst;
    row_range(G, rb, re, nst);
    for (int it = 0; it < nst; ++it) {
      const int s = gs % kSlots;
      if (gs >= kSlots && !wait_mb(&h->empty[s], ((gs / kSlots) - 1) & 1, err, 1, &h->abort)) {
        ok = false;
        break;
      }
      if (*reinterpret_cast<volatile int*>(&h->abort)) {
        ok = false;
        break;
      }
      const int r0 = rb + it * G.tr;
      const int n = min(G.tr, re - r0);
      const uint32_t bq = (uint32_t)(n * G.nb * G.qb);
      const uint32_t bs = (uint32_t)(n * G.nbp * 2);
      uint8_t* dst = ring + (size_t)s * kSlot;
      mbar_arrive_expect_tx(&h->full[s], bq + bs);
      bulk_g2s_hint(dst, qs + (size_t)r0 * G.nb * G.qb, bq, &h->full[s], pol);
      bulk_g2s_hint(dst + G.sc_off, sc + (size_t)r0 * G.nbp, bs, &h->full[s], pol);
      ++gs;
    }
  }
  // the copies of the last stages land before the CTA may exit
  for (int j = max(0, gs - kSlots); j < gs; ++j) mbar_wait(&h->full[j % kSlots], (j / kSlots) & 1, nullptr, 0);
}

// ---------------------------------------------------------------------------
// compute warps: the phase's input block in fixed point, then block values
// ---------------------------------------------------------------------------
// Chunk q (elements 4q .. 4q+3) of token tok's embedding row (llm.c:365-410;
// the arithmetic of embed_kernel: (n - 8) * d, q * d, fp16 widening, a copy).
__device__ __forceinline__ float4 embed_chunk(const void* embd, int type, int dim, int tok, int q) {
  const int nb = dim / 32, blk = q >> 3, c = q & 7;
  float4 v;
  if (type == TOSK_Q4_0) {
    const uint8_t* b = reinterpret_cast<const uint8_t*>(embd) + ((size_t)tok * nb + blk) * 18;
    const float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
    const int b0 = b[2 + 2 * c], b1 = b[3 + 2 * c];
    v.x = __fmul_rn((float)((b0 & 0x0F) - 8), d);
    v.y = __fmul_rn((float)((b0 >> 4) - 8), d);
    v.z = __fmul_rn((float)((b1 & 0x0F) - 8), d);
    v.w = __fmul_rn((float)((b1 >> 4) - 8), d);
  } else if (type == TOSK_Q8_0) {
    const uint8_t* b = reinterpret_cast<const uint8_t*>(embd) + ((size_t)tok * nb + blk) * 34 + 2 + 4 * c;
    const float d = h2f((uint16_t)(b[-2 - 4 * c] | (b[-1 - 4 * c] << 8)));
    v.x = __fmul_rn((float)(int8_t)b[0], d);
    v.y = __fmul_rn((float)(int8_t)b[1], d);
    v.z = __fmul_rn((float)(int8_t)b[2], d);
    v.w = __fmul_rn((float)(int8_t)b[3], d);
  } else if (type == TOSK_F16) {
    const uint16_t* e = reinterpret_cast<const uint16_t*>(embd) + (size_t)tok * dim + 4 * q;
    v = make_float4(h2f(e[0]), h2f(e[1]), h2f(e[2]), h2f(e[3]));
  } else {
    const float* e = reinterpret_cast<const float*>(embd) + (size_t)tok * dim + 4 * q;
    v = make_float4(e[0], e[1], e[2], e[3]);
  }
  return v;
}

// Shared-memory slot of 16-byte chunk q of the phase's input vector: chunk j
// of block k at 8 k + (j ^ (k & 7)), so the compute threads, each reading
// the eight chunks of its own block, spread over all banks.
__device__ __forceinline__ int xsw(int q) { return (q & ~7) | ((q ^ (q >> 3)) & 7); }

// Sharded step: the phase's input vector from every rank's exchange words
// into X4 (nq 16-byte chunks): four rounds of chunks in flight per thread, a
// chunk read again until its words carry the exchange's epoch.  Out of line,
// so its registers do not weigh on the block-value loop.
__device__ __noinline__ void ll_input(const Params& p, Hdr* h, float4* X4, int nq, int xk, int el, int ct, int* err) {
  const unsigned long long* ll = p.s.peer_ll[p.s.rank] + ll_off(p, xk);
  const uint32_t ep = ll_epoch(h, el, xk);
  for (int qb = ct; qb < nq; qb += 4 * 32 * kCompute) {
    uint4 w[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = qb + u * 32 * kCompute;
      if (q < nq) {
        w[u][0] = ll_load2(ll + 4 * (size_t)q);
        w[u][1] = ll_load2(ll + 4 * (size_t)q + 2);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = qb + u * 32 * kCompute;
      if (q < nq) {
        ll_ready(ll + 4 * (size_t)q, w[u][0], ep, h, err);
        ll_ready(ll + 4 * (size_t)q + 2, w[u][1], ep, h, err);
        X4[xsw(q)] = make_float4(__uint_as_float(w[u][0].x), __uint_as_float(w[u][0].z), __uint_as_float(w[u][1].x),
                                 __uint_as_float(w[u][1].z));
      }
    }
  }
}

// The RMSNorm weights of a phase (null: no norm).
__device__ __forceinline__ const float* norm_weights(const Params& p, int kind, int layer) {
  return kind == K_QKV ? p.s.layers[layer].norm_att
       : kind == K_GU  ? p.s.layers[layer].norm_ffn
       : kind == K_LM  ? p.s.norm_out : nullptr;
}

// ---------------------------------------------------------------------------
// compute warps: the phase's input block in fixed point, then block values
// ---------------------------------------------------------------------------
// The compute warps copy the phase's input vector (and a RMSNorm's weights)
// into shared memory, every chunk once per CTA in coalesced 16-byte copies
// (the vector is read by all CTAs, so L2 requests, not bytes, set the time);
// after one barrier with the chain warps, compute thread (b, g) turns its
// block b into a fixed-point record in registers (make_xfix) and evaluates
// block b of rows g, g + rg, ... of every stage.  The RMSNorm's scalar 1/rms
// is applied to the row sums by the chain warps (chain_gemv).
template <int QB, bool kLL>
__device__ __forceinline__ void compute_gemv(const Params& p, Hdr* h, float* Xs, float* P, const uint8_t* ring,
                                             int kind, int layer, int& gs) {
  const Geo G = geo_regs(p, kind);
  int* err = p.s.io + 3;
  const int ct = (int)threadIdx.x - 32 * (1 + kChain);   // 0 .. 32 * kCompute - 1
  const int lane = threadIdx.x & 31;
  const int nwb = (G.nb + 31) >> 5;
  int rg = kCompute / nwb;
  if (rg < 1) rg = 1;
  if (rg > G.tr) rg = G.tr;
  const int bw = nwb * 32;
  const int b = ct % bw, g = ct / bw;
  const bool active = b < G.nb && g < rg;
  int rb, re, nst;
  row_range(G, rb, re, nst);

  const float* nw = norm_weights(p, kind, layer);
  const int nq = G.nb * 8;   // 16-byte chunks
  float4* X4 = reinterpret_cast<float4*>(Xs);
  float4* W4 = X4 + nq;
  const bool stage_w = nw && 2 * nq * 16 <= kXBytes;
  {
    const float4* src4 = reinterpret_cast<const float4*>((kind == K_O) ? p.s.att : (kind == K_D) ? p.s.h : p.s.x);
    if (kind == K_QKV && layer == 0) {
      int orb, ore, ons;
      row_range(p.g[K_O], orb, ore, ons);
      for (int q = ct; q < nq; q += 32 * kCompute) {
        const float4 v = embed_chunk(p.s.embd, p.s.embd_type, p.s.dim, h->tok, q);
        // the residual stream starts as the embedding: this CTA writes the
        // rows it owns in the o / down phases (their residual adds are its own)
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int lr = 4 * q + i - p.s.row0;   // the o phase's local row
          if (lr >= orb && lr < ore) p.s.x[4 * q + i] = e[i];
        }
        X4[xsw(q)] = v;
      }
    } else if (kLL) {
      const int xk = kind == K_O ? X_ATT : kind == K_GU ? X_XO : kind == K_D ? X_H : X_XD;
      ll_input(p, h, X4, nq, xk, (kind == K_QKV || kind == K_LM) ? layer - 1 : layer, ct, err);
    } else {
      for (int q = ct; q < nq; q += 32 * kCompute) cp_async16(X4 + xsw(q), src4 + q);
    }
    if (stage_w)
      for (int q = ct; q < nq; q += 32 * kCompute) cp_async16(W4 + xsw(q), reinterpret_cast<const float4*>(nw) + q);
    cp_async_wait_all();
  }
  named_sync(B_COMPUTE, 32 * kCompute);   // the vector is in shared memory
  if (nw) named_arrive(B_STAGED, kWorkers);   // ... for the chain warps' sum of squares too
  XFix xf;
  if (active) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 e = X4[8 * b + (j ^ (b & 7))];
      v[4 * j] = e.x; v[4 * j + 1] = e.y; v[4 * j + 2] = e.z; v[4 * j + 3] = e.w;
    }
    if (nw) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 e = stage_w ? W4[8 * b + (j ^ (b & 7))] : __ldg(reinterpret_cast<const float4*>(nw) + 8 * b + j);
        v[4 * j] = __fmul_rn(v[4 * j], e.x);
        v[4 * j + 1] = __fmul_rn(v[4 * j + 1], e.y);
        v[4 * j + 2] = __fmul_rn(v[4 * j + 2], e.z);
        v[4 * j + 3] = __fmul_rn(v[4 * j + 3], e.w);
      }
    }
    make_xfix<QB>(v, xf);
  }

  for (int it = 0; it < nst; ++it, ++gs) {
    const int s = gs % kSlots;
    if (!wait_mb(&h->full[s], (gs / kSlots) & 1, err, 2, &h->abort)) return;
    const int c = gs % kChain;
    if (gs >= kChain && !wait_mb(&h->pempty[c], ((gs / kChain) & 1) ^ 1, err, 3, &h->abort)) return;
    const int n = min(G.tr, re - (rb + it * G.tr));
    const uint8_t* stq = ring + (size_t)s * kSlot;
    const uint16_t* sts = reinterpret_cast<const uint16_t*>(stq + G.sc_off);
    float* Pc = P + c * G.tr * G.pstride;
    if (active) {
      int r = g;
      for (; r + 3 * rg < n; r += 4 * rg) {   // four rows in flight
        const float y0 = block_value_fast<QB>(stq, sts, r, b, G.nb, G.nbp, xf);
        const float y1 = block_value_fast<QB>(stq, sts, r + rg, b, G.nb, G.nbp, xf);
        const float y2 = block_value_fast<QB>(stq, sts, r + 2 * rg, b, G.nb, G.nbp, xf);
        const float y3 = block_value_fast<QB>(stq, sts, r + 3 * rg, b, G.nb, G.nbp, xf);
        Pc[r * G.pstride + b] = y0;
        Pc[(r + rg) * G.pstride + b] = y1;
        Pc[(r + 2 * rg) * G.pstride + b] = y2;
        Pc[(r + 3 * rg) * G.pstride + b] = y3;
      }
      for (; r + rg < n; r += 2 * rg) {
        const float y0 = block_value_fast<QB>(stq, sts, r, b, G.nb, G.nbp, xf);
        const float y1 = block_value_fast<QB>(stq, sts, r + rg, b, G.nb, G.nbp, xf);
        Pc[r * G.pstride + b] = y0;
        Pc[(r + rg) * G.pstride + b] = y1;
      }
      if (r < n) Pc[r * G.pstride + b] = block_value_fast<QB>(stq, sts, r, b, G.nb, G.nbp, xf);
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&h->pfull[c]);
      mbar_arrive(&h->empty[s]);
    }
  }
}

// ---------------------------------------------------------------------------
// chain warps: row sums and the fused epilogues
// ---------------------------------------------------------------------------
// Lane i (< n) holds the sum of row r0 + i.  Paired epilogues see both rows
// of a pair in lanes i, i ^ 1 (stages and row ranges start at even rows).
template <int ESZ, bool kLL>
__device__ __forceinline__ void epilogue(const Params& p, const Hdr* h, int kind, int layer, float y, int r0, int n,
                                         int lane, int pos, int rb, bool pre_res, float& bv, int& bi) {
  const int r = r0 + lane;
  const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
  if (lane >= n) return;
  if (kind == K_QKV) {
    const int qr = p.s.n_heads * p.s.hd, kr = p.s.n_kv * p.s.hd, hd = p.s.hd;
    float v = y;
    if (r < qr + kr) {
      // llm.c:488-492: RoPE on q and k rows (adjacent pairs)
      const int i = (r < qr ? r : r - qr) % hd;
      const float2 cs = h->cs[i >> 1];
      if ((i & 1) == 0)
        v = __fsub_rn(__fmul_rn(y, cs.x), __fmul_rn(partner, cs.y));
      else
        v = __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(y, cs.x));
    }
    if (r < qr) {
      p.s.q[r] = v;
    } else {
      // llm.c:673-681: k, v of this position into the cache
      const bool is_k = r < qr + kr;
      const int e = is_k ? r - qr : r - qr - kr;
      const tosk_step_layer_t& L = p.s.layers[layer];
      const size_t idx = (size_t)pos * kr + e;
      if constexpr (ESZ == 2)
        reinterpret_cast<uint16_t*>(is_k ? L.k_cache : L.v_cache)[idx] = f2h(v);
      else
        reinterpret_cast<float*>(is_k ? L.k_cache : L.v_cache)[idx] = v;
    }
  } else if (kind == K_O || kind == K_D) {
    const int gr = p.s.row0 + r;   // residual row (all of x on one GPU)
    const float v = __fadd_rn(pre_res ? h->res[r - rb] : __ldcg(p.s.x + gr), y);   // llm.c:717-718, 732-733
    p.s.x[gr] = v;
    if (kLL) ll_store_all(p, kind == K_O ? X_XO : X_XD, gr, v, ll_epoch(h, layer, kind == K_O ? X_XO : X_XD));
  } else if (kind == K_GU) {
    if ((r & 1) == 0) {
      const float v = __fmul_rn(ref_silu(y), partner);   // llm.c:726-729
      if (kLL) ll_store_all(p, X_H, p.s.ff0 + (r >> 1), v, ll_epoch(h, layer, X_H));
      else p.s.h[r >> 1] = v;
    }
  } else {
    p.s.logits[r] = y;
    if (!(y != y)) arg_better(bv, bi, y, p.s.vocab0 + r);
  }
}

// Chain warps after the LM head: the CTA's (value, index), then the last CTA
// to finish reduces all of them and writes the greedy token.
template <bool kLL>
__device__ __forceinline__ void argmax_finish(const Params& p, Hdr* h, float bv, int bi) {
  const int cw = (int)(threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_down_sync(0xffffffffu, bv, o);
    const int i2 = __shfl_down_sync(0xffffffffu, bi, o);
    arg_better(bv, bi, v2, i2);
  }
  if (lane == 0) {
    h->av[cw] = bv;
    h->ai[cw] = bi;
  }
  named_sync(B_CHAIN, 32 * kChain);
  if (threadIdx.x >= 64) return;   // warp 1 finishes
  int* pairs = reinterpret_cast<int*>(p.s.sync + 64);
  int last = 0;
  if (threadIdx.x == 32) {
    float v = h->av[0];
    int i = h->ai[0];
    for (int c = 1; c < kChain; ++c) arg_better(v, i, h->av[c], h->ai[c]);
    pairs[2 * blockIdx.x] = __float_as_int(v);
    pairs[2 * blockIdx.x + 1] = i;
    __threadfence();
    last = atomicAdd(p.s.sync + 1, 1u) == gridDim.x - 1;
    if (last) __threadfence();
  }
  if (!__shfl_sync(0xffffffffu, last, 0)) return;
  // the last CTA: the warp loads the CTAs' pairs side by side and reduces
  // them (arg_better is associative and commutative, so the order of the
  // combination does not change the result)
  float best = 0.0f;
  int idx = -1;
  for (unsigned k = lane; k < gridDim.x; k += 32)
    arg_better(best, idx, __int_as_float(__ldcg(pairs + 2 * k)), __ldcg(pairs + 2 * k + 1));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_down_sync(0xffffffffu, best, o);
    const int i2 = __shfl_down_sync(0xffffffffu, idx, o);
    arg_better(best, idx, v2, i2);
  }
  if (lane != 0) return;
  // llm.c:1130: x[0] is the starting candidate; it stays when NaN or unbeaten
  // (logit 0 is the first row of rank 0's slice)
  const bool x0_nan = p.s.rank == 0 && __ldcg(p.s.logits) != __ldcg(p.s.logits);
  int* io = p.s.io;
  if (kLL) {   // sharded
    // every rank's (value, index) pair into every rank's pair words (rank 0
    // marks a NaN logit 0 with index -2) with the step's final epoch; every
    // rank then reduces the same pairs in rank order
    const size_t pw = ll_off(p, 4);
    for (int r = 0; r < p.s.world; ++r)
      ll_store2(p.s.peer_ll[r] + pw + 2 * p.s.rank, __float_as_uint(best), (uint32_t)(x0_nan ? -2 : idx), h->efinal);
    const unsigned long long* mine = p.s.peer_ll[p.s.rank] + pw;
    best = 0.0f;
    idx = -1;
    bool nan0 = false;
    for (int r = 0; r < p.s.world; ++r) {
      uint4 v = ll_load2(mine + 2 * r);
      if (!ll_ready(mine + 2 * r, v, h->efinal, h, io + 3)) break;
      const int pi = (int)v.z;
      if (pi == -2) nan0 = true;
      else arg_better(best, idx, __uint_as_float(v.x), pi);
    }
    if (nan0 || idx < 0) idx = 0;
  } else if (x0_nan || idx < 0) {
    idx = 0;
  }
  // the next step's exchange words carry later epochs than every word of
  // this one
  if (kLL) io[5] = (int)h->efinal;
  io[2] = idx;
  if (p.s.chained) {
    const int k = io[4];
    p.s.ring[k] = idx;
    io[4] = k + 1;
    io[1] = io[1] + 1;
  }
  // every CTA is past its last grid barrier: reset the counters for the next step
  atomicExch(p.s.sync, 0u);
  atomicExch(p.s.sync + 1, 0u);
}

// RMSNorm scale 1/sqrt(mean(x^2) + eps) of the phase's input (llm.c:416-442)
// by the chain warps from the shared-memory copy, while the compute warps
// evaluate block values: chain thread t sums the squares of chunks t, t + 96,
// ... in order, then a butterfly per warp and the three warps in order (the
// same order in every instance, so a sharded step's scale equals the one-GPU
// step's).
__device__ __noinline__ float norm_scale(const Params& p, Hdr* h, const float4* X4) {
  const int ct = (int)threadIdx.x - 32, lane = threadIdx.x & 31;
  const int nq = p.s.dim / 4;
  float acc = 0.0f;
  for (int q = ct; q < nq; q += 32 * kChain) {
    const float4 v = X4[xsw(q)];
    acc = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, acc))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) h->cpart[ct >> 5] = acc;
  named_sync(B_CHAIN, 32 * kChain);
  float s2 = 0.0f;
  for (int c = 0; c < kChain; ++c) s2 += h->cpart[c];
  named_sync(B_CHAIN, 32 * kChain);   // cpart is read before the next phase writes it
  return 1.0f / sqrtf(s2 / (float)p.s.dim + p.s.eps);
}

template <int ESZ, bool kLL>
__device__ __forceinline__ void chain_gemv(const Params& p, Hdr* h, const float* Xs, const float* P, int kind,
                                           int layer, int& gs) {
  float bv = 0.0f;   // LM head: this lane's running (value, index) of llm_argmax
  int bi = -1;
  const Geo G = geo_regs(p, kind);
  int* err = p.s.io + 3;
  const int cw = (int)(threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
  int rb, re, nst;
  row_range(G, rb, re, nst);
  const int gs0 = gs;
  gs += nst;
  // lane = row * nseg + segment; each lane sums its segment of the row's
  // partials with four running sums, then a butterfly over the segments
  const int tr = G.tr;
  int nseg = 1;
  while (nseg * 2 * tr <= 32) nseg <<= 1;
  const int row = min(lane / nseg, tr - 1), seg = lane % nseg;
  const int L = ((G.nb + nseg - 1) / nseg + 3) & ~3;
  const int j0 = min(G.nb, seg * L), j1 = min(G.nb, seg * L + L);
  const int pos = h->pos;
  const bool pre_res = (kind == K_O || kind == K_D) && re - rb <= kPreRows;
  const bool nrm = norm_weights(p, kind, layer) != nullptr;
  float ss = 1.0f;
  {
    const int ct = (int)threadIdx.x - 32;   // 0 .. 32 * kChain - 1
    if (pre_res)
      for (int i = ct; i < re - rb; i += 32 * kChain) h->res[i] = __ldcg(p.s.x + p.s.row0 + rb + i);
    if (kind == K_QKV) {
      for (int i = ct; i < (p.s.hd >> 1); i += 32 * kChain) h->cs[i] = p.s.rope[(size_t)pos * (p.s.hd >> 1) + i];
      if (pos + 1 <= kHeadMaxN) {
        // the heads this CTA attends to next: their K and V rows of the
        // earlier positions go to L2 while the projection runs
        const tosk_step_layer_t& Ly = p.s.layers[layer];
        const int hd = p.s.hd, group = p.s.n_heads / p.s.n_kv, kv_dim = p.s.n_kv * hd;
        const uint32_t rowb = (uint32_t)(hd * ESZ);
        const uint64_t keep = policy_evict_last();
        for (int hh = blockIdx.x; hh < p.s.n_heads; hh += gridDim.x) {
          const size_t off = (size_t)(hh / group) * hd * ESZ;
          for (int t = ct; t < 2 * pos; t += 32 * kChain) {
            const uint8_t* base = reinterpret_cast<const uint8_t*>(t < pos ? Ly.k_cache : Ly.v_cache);
            prefetch_l2(base + (size_t)(t < pos ? t : t - pos) * kv_dim * ESZ + off, rowb, keep);
          }
        }
      }
    }
    named_sync(B_CHAIN, 32 * kChain);
  }
  if (nrm) {
    named_sync(B_STAGED, kWorkers);   // the compute warps have staged the input vector
    ss = norm_scale(p, h, reinterpret_cast<const float4*>(Xs));
  }
  for (int it = ((cw - gs0) % kChain + kChain) % kChain; it < nst; it += kChain) {
    const int gsi = gs0 + it;
    if (!wait_mb(&h->pfull[cw], (gsi / kChain) & 1, err, 4, &h->abort)) break;
    const int r0 = rb + it * tr;
    const int n = min(tr, re - r0);
    const float* Prow = P + (cw * tr + row) * G.pstride;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int j = j0;
    for (; j + 4 <= j1; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(Prow + j);
      s0 += v.x; s1 += v.y; s2 += v.z; s3 += v.w;
    }
    for (; j < j1; ++j) s0 += Prow[j];
    float t = (s0 + s1) + (s2 + s3);
    for (int o = 1; o < nseg; o <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    float y = __shfl_sync(0xffffffffu, t, min(lane, tr - 1) * nseg);
    if (nrm) y = __fmul_rn(y, ss);   // RMSNorm's 1/rms (llm.c:416-442), applied to the row
    __syncwarp();
    if (lane == 0) mbar_arrive(&h->pempty[cw]);
    epilogue<ESZ, kLL>(p, h, kind, layer, y, r0, n, lane, pos, rb, pre_res, bv, bi);
  }
  if (kind == K_LM) argmax_finish<kLL>(p, h, bv, bi);
}

// ---------------------------------------------------------------------------
// attention (llm.c:683-714), FAST: split-K over 64-position chunks
// ---------------------------------------------------------------------------
// Four consecutive cache elements as loaded (fp16: two packed words) and as
// floats.
template <int ESZ> struct RawT { using type = float4; };
template <> struct RawT<2> { using type = uint2; };
template <int ESZ>
__device__ __forceinline__ typename RawT<ESZ>::type ldraw(const uint8_t* p) {
  return __ldcg(reinterpret_cast<const typename RawT<ESZ>::type*>(p));
}
__device__ __forceinline__ float4 unraw2(uint2 u) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <int ESZ>
__device__ __forceinline__ float4 unraw(typename RawT<ESZ>::type r) {
  if constexpr (ESZ == 2) return unraw2(r);
  else return r;
}

__device__ __forceinline__ float warp_max_f(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

// Scores of one (kv head, chunk) item per group of kGW warps: a warp per 16
// positions, lane l covering d = 128 s + 4 l .. +3, all 16 rows in flight,
// then a shuffle reduce-scatter; per-chunk maxima for the softmax pass.
template <int ESZ>
__device__ __forceinline__ void attn_scores(const Params& p, Hdr* h, float* P, int layer) {
  const int w = (int)(threadIdx.x >> 5) - 1;
  const int grp = w / kGW, gw = w % kGW, lane = threadIdx.x & 31;
  float* wmax = P + grp * kGroupFloats + kChunk;
  const int n = h->pos + 1;
  const int n_heads = p.s.n_heads, n_kv = p.s.n_kv, hd = p.s.hd;
  if (blockIdx.x == 0)
    for (int i = (int)threadIdx.x - 32; i < n_heads; i += kWorkers) p.cnt[i] = 0;   // the pv pass's counters
  if (grp >= kGroups) return;
  const int group = n_heads / n_kv, kv_dim = n_kv * hd;
  const int nchunk = (n + kChunk - 1) / kChunk;
  const int items = n_kv * nchunk;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const uint8_t* kc = reinterpret_cast<const uint8_t*>(p.s.layers[layer].k_cache);
  for (int item = blockIdx.x * kGroups + grp; item < items; item += gridDim.x * kGroups) {
    // kv head fastest: the groups that run together read every head of the
    // same positions, i.e. whole cache rows
    const int kvh = item % n_kv, c = item / n_kv;
    const int tw = c * kChunk + gw * 16;
    for (int gi = 0; gi < group; ++gi) {
      const int hh = kvh * group + gi;
      float v[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) v[q] = 0.0f;
#pragma unroll
      for (int sl = 0; sl < kMaxHd / 128; ++sl) {
        const int d = 128 * sl + 4 * lane;
        if (d < hd) {
          const float4 qv = __ldcg(reinterpret_cast<const float4*>(p.s.q + (size_t)hh * hd + d));
          typename RawT<ESZ>::type kr[16];   // all 16 rows in flight (fp16 packed)
#pragma unroll
          for (int q = 0; q < 16; ++q)
            kr[q] = tw + q < n ? ldraw<ESZ>(kc + ((size_t)(tw + q) * kv_dim + (size_t)kvh * hd + d) * ESZ)
                               : typename RawT<ESZ>::type{};
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float4 kv = unraw<ESZ>(kr[q]);
            v[q] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, v[q]))));
          }
        }
      }
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
      float m = -INFINITY;
      if (t < n) {
        m = dot * scale;
        if ((lane & 1) == 0) p.S[(size_t)hh * p.s.max_seq + t] = m;
      }
      m = warp_max_f(m);
      named_sync(B_GROUP0 + grp, 32 * kGW);
      if (lane == 0) wmax[gw] = m;
      named_sync(B_GROUP0 + grp, 32 * kGW);
      if (gw == 0 && lane == 0) {
        float cm = wmax[0];
        for (int i = 1; i < kGW; ++i) cm = fmaxf(cm, wmax[i]);
        p.cmax[(size_t)hh * p.maxc + c] = cm;
      }
    }
  }
}

// e_t = llm_expf(s_t - max) with the head's global max (llm.c:509-517), the
// chunk's e-sum and sum_t e_t v_t; the last chunk of a head to finish adds
// the chunks in order and divides by the sum (llm.c:519-521, 703-712).
template <int ESZ, bool kLL>
__device__ __forceinline__ void attn_pv(const Params& p, Hdr* h, float* P, int layer) {
  constexpr int kGT = 32 * kGW;   // threads of a group
  const int w = (int)(threadIdx.x >> 5) - 1;
  const int grp = w / kGW, gw = w % kGW, lane = threadIdx.x & 31;
  const int gt = gw * 32 + lane;
  float* es = P + grp * kGroupFloats;
  float* red = es + kChunk;
  float* wpart = es + kChunk + 12;
  int* s_last = reinterpret_cast<int*>(wpart + kGW * kMaxHd);
  if (grp >= kGroups) return;
  const int n = h->pos + 1;
  const int n_heads = p.s.n_heads, n_kv = p.s.n_kv, hd = p.s.hd;
  const int group = n_heads / n_kv, kv_dim = n_kv * hd;
  const int nchunk = (n + kChunk - 1) / kChunk;
  const int items = n_heads * nchunk;
  const uint8_t* vc = reinterpret_cast<const uint8_t*>(p.s.layers[layer].v_cache);
  for (int item = blockIdx.x * kGroups + grp; item < items; item += gridDim.x * kGroups) {
    const int hh = item % n_heads, c = item / n_heads;   // head fastest (whole cache rows together)
    const int kvh = hh / group;
    const int t0 = c * kChunk, cn = min(kChunk, n - t0);
    float m = -INFINITY;
    for (int i = gt; i < nchunk; i += kGT) m = fmaxf(m, __ldcg(p.cmax + (size_t)hh * p.maxc + i));
    m = warp_max_f(m);
    named_sync(B_GROUP0 + grp, kGT);
    if (lane == 0) red[gw] = m;
    named_sync(B_GROUP0 + grp, kGT);
    float M = red[0];
    for (int i = 1; i < kGW; ++i) M = fmaxf(M, red[i]);
    float e = 0.0f;
    if (gt < kChunk) {
      if (gt < cn) e = ref_expf(__fsub_rn(__ldcg(p.S + (size_t)hh * p.s.max_seq + t0 + gt), M));
      es[gt] = e;
    }
    float l = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    named_sync(B_GROUP0 + grp, kGT);
    if (lane == 0) red[kGW + gw] = l;
    const int tw = gw * 16;
#pragma unroll
    for (int sl = 0; sl < kMaxHd / 128; ++sl) {
      const int d = 128 * sl + 4 * lane;
      if (d < hd) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        typename RawT<ESZ>::type vr[16];   // all 16 rows in flight (fp16 packed)
#pragma unroll
        for (int q = 0; q < 16; ++q)
          vr[q] = tw + q < cn ? ldraw<ESZ>(vc + ((size_t)(t0 + tw + q) * kv_dim + (size_t)kvh * hd + d) * ESZ)
                              : typename RawT<ESZ>::type{};
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float ep = es[tw + q];
          const float4 vv = unraw<ESZ>(vr[q]);
          acc.x = fmaf(ep, vv.x, acc.x);
          acc.y = fmaf(ep, vv.y, acc.y);
          acc.z = fmaf(ep, vv.z, acc.z);
          acc.w = fmaf(ep, vv.w, acc.w);
        }
        *reinterpret_cast<float4*>(&wpart[gw * kMaxHd + d]) = acc;
      }
    }
    named_sync(B_GROUP0 + grp, kGT);
    float* op = p.opart + ((size_t)hh * p.maxc + c) * kMaxHd;
    for (int d = gt; d < hd; d += kGT) {
      float o = wpart[d];
      for (int i = 1; i < kGW; ++i) o += wpart[i * kMaxHd + d];
      op[d] = o;
    }
    if (gt == 0) {
      float lc = red[kGW];
      for (int i = 1; i < kGW; ++i) lc += red[kGW + i];
      p.lsum[(size_t)hh * p.maxc + c] = lc;
    }
    __threadfence();
    named_sync(B_GROUP0 + grp, kGT);
    if (gt == 0) *s_last = atomicAdd(p.cnt + hh, 1) == nchunk - 1;
    named_sync(B_GROUP0 + grp, kGT);
    if (*s_last) {
      __threadfence();
      // chunk order, eight chunks' loads in flight
      const float* ls = p.lsum + (size_t)hh * p.maxc;
      const float* op = p.opart + (size_t)hh * p.maxc * kMaxHd;
      float Ls = 0.0f;
      for (int i0 = 0; i0 < nchunk; i0 += 8) {
        float lv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) lv[k] = i0 + k < nchunk ? __ldcg(ls + i0 + k) : 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (i0 + k < nchunk) Ls += lv[k];
      }
      const float inv = 1.0f / (Ls + 1e-10f);
      for (int d = gt; d < hd; d += kGT) {
        float o = 0.0f;
        for (int i0 = 0; i0 < nchunk; i0 += 8) {
          float ov[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) ov[k] = i0 + k < nchunk ? __ldcg(op + (size_t)(i0 + k) * kMaxHd + d) : 0.0f;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (i0 + k < nchunk) o += ov[k];
        }
        if (kLL) ll_store_all(p, X_ATT, p.s.q0 + (size_t)hh * hd + d, o * inv, ll_epoch(h, layer, X_ATT));
        else p.s.att[(size_t)hh * hd + d] = o * inv;
      }
    }
    named_sync(B_GROUP0 + grp, kGT);   // es / red / wpart / s_last are reused by the next item
  }
}

// Short contexts (n <= kHeadMaxN positions): one CTA per head does the whole
// attention of that head in one phase, scores and e_t in shared memory, so
// no grid barrier separates the max from the exponentials.  Worker warp w
// takes positions w, w + kNW, ... eight at a time (all eight K or V rows in
// flight); the eight dot products of a warp meet in one reduce-scatter.

template <int ESZ, bool kLL>
__device__ __forceinline__ void attn_head(const Params& p, Hdr* h, float* smf, int layer) {
  // rows in flight per warp: sixteen fp16 rows (two registers each), eight fp32
  using KRaw = typename RawT<ESZ>::type;
  constexpr int kRows = ESZ == 2 ? 16 : 8;
  constexpr int kLow = ESZ == 2 ? 1 : 2;   // lane bits left to sum after the reduce-scatter
  const int w = (int)(threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
  const int wt = (int)threadIdx.x - 32;
  const int n = h->pos + 1;
  const int hd = p.s.hd, n_heads = p.s.n_heads, group = n_heads / p.s.n_kv, kv_dim = p.s.n_kv * hd;
  float* sc = smf;                              // [n]: scores, then e_t
  float* part = smf + kHeadMaxN;                // [kNW][kMaxHd] PV partials
  float* red = part + kNW * kMaxHd;             // [32]
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(p.s.layers[layer].k_cache);
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(p.s.layers[layer].v_cache);
  for (int hh = blockIdx.x; hh < n_heads; hh += gridDim.x) {
    const int kvh = hh / group;
    const uint8_t* kc = kbase + (size_t)kvh * hd * ESZ;
    const uint8_t* vc = vbase + (size_t)kvh * hd * ESZ;
    float4 qv[kMaxHd / 128];
#pragma unroll
    for (int sl = 0; sl < kMaxHd / 128; ++sl) {
      const int d = 128 * sl + 4 * lane;
      qv[sl] = d < hd ? __ldcg(reinterpret_cast<const float4*>(p.s.q + (size_t)hh * hd + d))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // scores (llm.c:686-692), kRows positions per warp per pass (all their
    // K rows in flight; fp16 rows stay packed until used)
    for (int t0 = w; t0 < n; t0 += kRows * kNW) {
      float v[kRows];
#pragma unroll
      for (int u = 0; u < kRows; ++u) v[u] = 0.0f;
#pragma unroll 1
      for (int sl = 0; sl < kMaxHd / 128; ++sl) {
        const int d = 128 * sl + 4 * lane;
        if (d < hd) {
          KRaw kr[kRows];
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
            const int t = t0 + u * kNW;
            kr[u] = t < n ? ldraw<ESZ>(kc + ((size_t)t * kv_dim + d) * ESZ) : KRaw{};
          }
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
            const float4 kv = unraw<ESZ>(kr[u]);
            v[u] = fmaf(qv[sl].x, kv.x, fmaf(qv[sl].y, kv.y, fmaf(qv[sl].z, kv.z, fmaf(qv[sl].w, kv.w, v[u]))));
          }
        }
      }
      // reduce-scatter over the lane bits from 4 down: lane l ends with
      // position (l >> kLow) % kRows summed over those bits; the kLow low
      // bits finish the sum
#pragma unroll
      for (int half = kRows / 2, o = 16; half >= 1; half >>= 1, o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float keep = up ? v[half + i] : v[i];
          const float send = up ? v[i] : v[half + i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      float dot = v[0];
#pragma unroll
      for (int o = 1 << (kLow - 1); o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      const int t = t0 + ((lane >> kLow) & (kRows - 1)) * kNW;
      if ((lane & ((1 << kLow) - 1)) == 0 && t < n) sc[t] = dot * scale;
    }
    named_sync(B_WORKERS, kWorkers);
    // llm.c:509-521: max, e_t = llm_expf(s_t - max), sum (tree), 1/(sum + 1e-10)
    float m = -INFINITY;
    for (int t = wt; t < n; t += kWorkers) m = fmaxf(m, sc[t]);
    m = warp_max_f(m);
    if (lane == 0) red[w] = m;
    named_sync(B_WORKERS, kWorkers);
    float M = red[0];
    for (int i = 1; i < kNW; ++i) M = fmaxf(M, red[i]);
    float l = 0.0f;
    for (int t = wt; t < n; t += kWorkers) {
      const float e = ref_expf(__fsub_rn(sc[t], M));
      sc[t] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    named_sync(B_WORKERS, kWorkers);   // every thread has read red (the max) and written its e_t
    if (lane == 0) red[w] = l;
    // sum_t e_t v_t[d] (llm.c:703-712): warp w over its positions, lane l four d
#pragma unroll 1
    for (int sl = 0; sl < kMaxHd / 128; ++sl) {
      const int d = 128 * sl + 4 * lane;
      if (d < hd) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int t0 = w; t0 < n; t0 += kRows * kNW) {
          KRaw vr[kRows];
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
            const int t = t0 + u * kNW;
            vr[u] = t < n ? ldraw<ESZ>(vc + ((size_t)t * kv_dim + d) * ESZ) : KRaw{};
          }
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
            const int t = t0 + u * kNW;
            const float e = t < n ? sc[t] : 0.0f;
            const float4 vv = unraw<ESZ>(vr[u]);
            acc.x = fmaf(e, vv.x, acc.x);
            acc.y = fmaf(e, vv.y, acc.y);
            acc.z = fmaf(e, vv.z, acc.z);
            acc.w = fmaf(e, vv.w, acc.w);
          }
        }
        *reinterpret_cast<float4*>(part + w * kMaxHd + d) = acc;
      }
    }
    named_sync(B_WORKERS, kWorkers);
    float L = red[0];
    for (int i = 1; i < kNW; ++i) L += red[i];
    const float inv = 1.0f / (L + 1e-10f);
    for (int d = wt; d < hd; d += kWorkers) {
      float o = part[d];
      for (int i = 1; i < kNW; ++i) o += part[i * kMaxHd + d];
      if (kLL) ll_store_all(p, X_ATT, p.s.q0 + (size_t)hh * hd + d, o * inv, ll_epoch(h, layer, X_ATT));
      else p.s.att[(size_t)hh * hd + d] = o * inv;
    }
    named_sync(B_WORKERS, kWorkers);   // scratch is reused by the next head
  }
}

// ---------------------------------------------------------------------------
// the step
// ---------------------------------------------------------------------------
template <int ESZ, bool kLL>
__device__ __forceinline__ void gemv_phase(const Params& p, Hdr* h, float* Xs, float* P, const uint8_t* ring,
                                           int kind, int layer, int& gs) {
  if ((threadIdx.x >> 5) <= kChain)
    chain_gemv<ESZ, kLL>(p, h, Xs, P, kind, layer, gs);
  else if (p.g[kind].qb == 16)
    compute_gemv<16, kLL>(p, h, Xs, P, ring, kind, layer, gs);
  else
    compute_gemv<32, kLL>(p, h, Xs, P, ring, kind, layer, gs);
}

template <int ESZ, bool kLL>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ Params p) {
  // kLL: the phases hand their vectors over as exchange words (a sharded
  // step); otherwise through grid barriers.  Two instances, so that the
  // one-GPU step carries none of the exchange code.
  extern __shared__ __align__(1024) uint8_t smem[];
  Hdr* h = reinterpret_cast<Hdr*>(smem);
  float* A = reinterpret_cast<float*>(smem + kHdr);   // input vector / attention scratch
  float* P = reinterpret_cast<float*>(smem + kHdr + kXBytes);
  uint8_t* ring = smem + kHdr + kXBytes + kPBytes;
  int* err = p.s.io + 3;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&h->full[s], 1);
      mbar_init(&h->empty[s], kCompute);
    }
    for (int c = 0; c < kChain; ++c) {
      mbar_init(&h->pfull[c], kCompute);
      mbar_init(&h->pempty[c], 1);
    }
    h->abort = 0;
    // an earlier step whose bounded wait ran out leaves the error word set:
    // then nothing runs (the host reports it and resets the step)
    h->skip = *reinterpret_cast<volatile int*>(err) != 0;
    h->pos = p.s.io[1];
    h->tok = p.s.chained ? p.s.io[2] : p.s.io[0];
    // four cross-GPU barriers a layer (after attention, o, gate|up, down),
    // then the argmax exchange
    h->ebase = (unsigned)p.s.io[5];
    h->efinal = h->ebase + 4u * (unsigned)p.s.n_layers + 1u;
    mbar_fence_init();
  }
  __syncthreads();
  if (h->skip) return;
  if (threadIdx.x < 32) {
    if (threadIdx.x == 0) producer(p, h, ring);
    return;
  }
  int gs = 0;
  // per layer: q|k|v, attention (one phase per head for short contexts,
  // else split-K scores then softmax*V), o, gate|up, down; then the LM head.
  // One call site per role keeps every role inlined once.
  const bool short_ctx = h->pos + 1 <= kHeadMaxN;
  unsigned nsync = 0;
  const int nph = 6 * p.s.n_layers + 1;
  for (int ph = 0; ph < nph; ++ph) {
    const int l = ph / 6, r = ph - 6 * l;
    if (l == p.s.n_layers || r == 0 || r >= 3) {
      const int kind = l == p.s.n_layers ? K_LM : r == 0 ? K_QKV : r == 3 ? K_O : r == 4 ? K_GU : K_D;
      gemv_phase<ESZ, kLL>(p, h, A, P, ring, kind, l, gs);
      if (kind == K_LM) break;
    } else if (short_ctx) {
      if (r == 2) continue;
      attn_head<ESZ, kLL>(p, h, A, l);
    } else if (r == 1) {
      attn_scores<ESZ>(p, h, P, l);
    } else {
      attn_pv<ESZ, kLL>(p, h, P, l);
    }
    // with exchange words, the vectors the next phase reads in full
    // (attention output, residual, SwiGLU output; from every rank when
    // sharded) carry their own readiness, which the readers wait on; only
    // the q|k|v -> attention and scores -> softmax*V hand-offs (q, the KV
    // rows, the scores) need the grid barrier
    const bool grid = !kLL || r == 0 || (r == 1 && !short_ctx);
    if (grid) {
      if (!grid_sync(h, p.s.sync, (++nsync) * gridDim.x, err)) return;
    } else if (!cta_sync(h)) {
      return;
    }
  }
}

}  // namespace step
}  // namespace tos

using namespace tos;
using namespace tos::step;

extern "C" size_t tosk_step_sync_bytes(void) { return 256 + (size_t)kMaxGrid * 8; }

extern "C" size_t tosk_step_ll_words(int q_full, int dim, int ff) {
  return (size_t)q_full + 2 * (size_t)dim + (size_t)ff + 2 * TOSK_MAX_WORLD;
}

static inline int round_up_i(int v, int a) { return (v + a - 1) / a * a; }
static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

static int make_geo(int R, int cols, int qtype, int unit, Geo& G) {
  if (R <= 0 || cols <= 0 || cols % 32 != 0 || R % unit != 0) return (int)cudaErrorInvalidValue;
  if (qtype != TOSK_Q4_0 && qtype != TOSK_Q8_0) return (int)cudaErrorNotSupported;
  G.R = R;
  G.nb = cols / 32;
  // a block per compute thread; the input vector staged in shared memory
  if (G.nb > 32 * kCompute || G.nb * 128 > kXBytes) return (int)cudaErrorNotSupported;
  G.nbp = round_up_i(G.nb, 8);
  G.qb = qtype == TOSK_Q4_0 ? 16 : 32;
  G.unit = unit;
  G.pstride = round_up_i(G.nb, 8) + 4;
  int tr = 32;
  while (tr > 0 && (round_up_i(tr * G.nb * G.qb, 16) + tr * G.nbp * 2 > kSlot ||
                    kChain * tr * G.pstride * 4 > kPBytes))
    --tr;
  if (unit == 2) tr &= ~1;
  if (tr < unit) return (int)cudaErrorNotSupported;
  G.tr = tr;
  G.sc_off = round_up_i(tr * G.nb * G.qb, 16);
  return 0;
}

template <int ESZ, bool kLL>
static int prepare_kernel(int* occ) {
  static int done = 0, occ_v = 0;
  if (!done) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_step_kernel<ESZ, kLL>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return (int)e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_v, decode_step_kernel<ESZ, kLL>, kThreads, kSmem);
    if (e != cudaSuccess) return (int)e;
    done = 1;
  }
  *occ = occ_v;
  return 0;
}

static int plan(const tosk_step_t* s, Params* p) {
  if (!s || !s->layers || !s->io || !s->sync || !s->attn_ws || s->n_layers <= 0) return (int)cudaErrorInvalidValue;
  if (s->n_heads <= 0 || s->n_kv <= 0 || s->n_heads % s->n_kv != 0 || s->hd <= 0 || s->max_seq <= 0)
    return (int)cudaErrorInvalidValue;
  if (s->kv_type != TOSK_F16 && s->kv_type != TOSK_F32) return (int)cudaErrorNotSupported;
  const int esz = s->kv_type == TOSK_F16 ? 2 : 4;
  if (s->hd > kMaxHd || s->hd % 4 != 0 || (s->hd * esz) % 16 != 0) return (int)cudaErrorNotSupported;
  if (s->dim % 32 != 0 || s->ff % 32 != 0) return (int)cudaErrorNotSupported;
  const int q_dim = s->n_heads * s->hd, kv_dim = s->n_kv * s->hd;
  if (q_dim % 32 != 0) return (int)cudaErrorNotSupported;
  // 16-byte aligned vectors (float4 block loads)
  const void* vecs[] = {s->x, s->q, s->att, s->h, s->logits};
  for (const void* v : vecs)
    if (!v || (reinterpret_cast<uintptr_t>(v) & 15)) return (int)cudaErrorInvalidValue;
  memset(p, 0, sizeof(*p));
  p->s = *s;
  tosk_step_t& t = p->s;
  if (t.world <= 1) {
    // one GPU: every row is local, every vector has only its own copy
    t.world = 1;
    t.rank = 0;
    t.n_rows = s->dim;
    t.n_ff = s->ff;
    t.q_full = q_dim;
    t.q0 = t.row0 = t.ff0 = t.vocab0 = 0;
  } else {
    if (t.world > TOSK_MAX_WORLD || t.rank < 0 || t.rank >= t.world) return (int)cudaErrorInvalidValue;
    if (t.n_rows <= 0 || t.n_ff <= 0 || t.q_full < q_dim || t.q0 < 0 || t.q0 + q_dim > t.q_full ||
        t.row0 < 0 || t.row0 + t.n_rows > s->dim || t.ff0 < 0 || t.ff0 + t.n_ff > s->ff || t.vocab0 < 0 ||
        t.q_full % 32 != 0)
      return (int)cudaErrorInvalidValue;
    for (int r = 0; r < t.world; ++r)
      if (!t.peer_ll[r] || (reinterpret_cast<uintptr_t>(t.peer_ll[r]) & 15)) return (int)cudaErrorInvalidValue;
  }
  if (t.world == 1 && t.peer_ll[0] && (reinterpret_cast<uintptr_t>(t.peer_ll[0]) & 15)) return (int)cudaErrorInvalidValue;
  p->ll = t.peer_ll[0] != nullptr;
  int e = make_geo(q_dim + 2 * kv_dim, s->dim, s->wtype, 2, p->g[K_QKV]);
  if (!e) e = make_geo(t.n_rows, t.q_full, s->wtype, 1, p->g[K_O]);
  if (!e) e = make_geo(2 * t.n_ff, s->dim, s->wtype, 2, p->g[K_GU]);
  if (!e) e = make_geo(t.n_rows, s->ff, s->wtype, 1, p->g[K_D]);
  if (!e) e = make_geo(s->vocab, s->dim, s->lm_type, 1, p->g[K_LM]);
  if (e) return e;
  p->maxc = (s->max_seq + kChunk - 1) / kChunk;
  char* ws = reinterpret_cast<char*>(s->attn_ws);
  p->S = reinterpret_cast<float*>(ws);
  p->cmax = reinterpret_cast<float*>(ws + al256((size_t)s->n_heads * s->max_seq * 4));
  p->lsum = reinterpret_cast<float*>(reinterpret_cast<char*>(p->cmax) + al256((size_t)s->n_heads * p->maxc * 4));
  p->opart = reinterpret_cast<float*>(reinterpret_cast<char*>(p->lsum) + al256((size_t)s->n_heads * p->maxc * 4));
  p->cnt = reinterpret_cast<int*>(reinterpret_cast<char*>(p->opart) +
                                  al256((size_t)s->n_heads * p->maxc * kMaxHd * 4));
  int occ = 0;
  e = esz == 2 ? (p->ll ? prepare_kernel<2, true>(&occ) : prepare_kernel<2, false>(&occ))
               : (p->ll ? prepare_kernel<4, true>(&occ) : prepare_kernel<4, false>(&occ));
  if (e) return e;
  // every CTA must be resident at once (grid barriers): one per SM
  if (occ < 1 || tosk_num_sms() > kMaxGrid) return (int)cudaErrorNotSupported;
  return 0;
}

extern "C" int tosk_step_check(const tosk_step_t* s) {
  Params p;
  return plan(s, &p);
}

extern "C" int tosk_step_launch(const tosk_step_t* s, cudaStream_t st) {
  Params p;
  int e = plan(s, &p);
  if (e) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tosk_num_sms());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (s->kv_type == TOSK_F16)
    return (int)(p.ll ? cudaLaunchKernelEx(&cfg, decode_step_kernel<2, true>, p)
                      : cudaLaunchKernelEx(&cfg, decode_step_kernel<2, false>, p));
  return (int)(p.ll ? cudaLaunchKernelEx(&cfg, decode_step_kernel<4, true>, p)
                    : cudaLaunchKernelEx(&cfg, decode_step_kernel<4, false>, p));
}
