// gemv_common.cuh - GEMV launch arguments, the bulk-copy stage issue, a
// named barrier and the fused output epilogues.
#pragma once
#include <cuda_runtime.h>

#include "tos_dev.cuh"
#include "tos_kernels.h"

namespace tos {

struct GemvArgs {
  const uint8_t* qs;
  const uint16_t* sc;
  const float* x;
  const float* norm_w;
  float eps;
  float* out;
  int* err;
  int R, nb, nbp, cols;
  int unit;      // CTA row ranges are multiples of `unit` rows
  int S;         // ring depth
  int pstride;   // EXACT: partials row stride (floats)
  int nwb, rg;   // compute warps per row of blocks, row groups
  int tr;        // rows per stage
  uint32_t off_x, off_w, off_p, off_st, stage_bytes, stage_sc_off;
  tosk_epi_t epi;
};

// Issues stage `it` of a CTA's row range into ring slot s: the quants and the
// scales of up to tr rows, both counted on full[s].
template <int QB>
__device__ __forceinline__ void issue_stage(const GemvArgs& a, uint8_t* stages, uint64_t* full, int it,
                                            int s, int rb, int re) {
  const int r0 = rb + it * a.tr;
  const int n = min(a.tr, re - r0);
  const uint32_t bq = (uint32_t)(n * a.nb * QB);
  const uint32_t bs = (uint32_t)(n * a.nbp * 2);
  uint8_t* st = stages + (size_t)s * a.stage_bytes;
  mbar_arrive_expect_tx(&full[s], bq + bs);
  bulk_g2s(st, a.qs + (size_t)r0 * a.nb * QB, bq, &full[s]);
  bulk_g2s(st + a.stage_sc_off, a.sc + (size_t)r0 * a.nbp, bs, &full[s]);
}

// CTA named barrier over n threads.  The non-.aligned form: threads of one
// warp may reach it from divergent paths (e.g. the lanes that ran a serial
// chain and those that did not); callers still reconverge with __syncwarp.
__device__ __forceinline__ void named_sync(int id, int n) {
  __syncwarp();
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Arrive on named barrier id (n threads in all) without waiting: the
// producer side of a producer / consumer hand-off (its earlier writes are
// visible to the threads that wait on the barrier with named_sync).
__device__ __forceinline__ void named_arrive(int id, int n) {
  __syncwarp();
  asm volatile("barrier.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Output epilogue of one stage, run by a full warp: lane i (< n) holds the
// row sum y of row r0 + i.  Paired epilogues (RoPE, SiLU*up) rely on stages
// and row ranges starting at even rows.
template <int kEpi>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, float y, int r0, int n, int lane,
                                              int pos) {
  const int r = r0 + lane;
  if constexpr (kEpi == TOSK_EPI_STORE) {
    if (lane < n) a.out[r] = y;
  } else if constexpr (kEpi == TOSK_EPI_RESID) {
    if (lane < n) a.out[r] = __fadd_rn(a.epi.resid[r], y);  // llm.c:599-614
  } else if constexpr (kEpi == TOSK_EPI_SWIGLU) {
    // llm.c:726-729: g = silu(g); g *= u
    const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
    if (lane < n && (r & 1) == 0) a.out[r >> 1] = __fmul_rn(ref_silu(y), partner);
  } else if constexpr (kEpi == TOSK_EPI_QKV) {
    const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
    const int qr = a.epi.q_rows, kr = a.epi.kv_rows, hd = a.epi.hd;
    if (lane < n) {
      float v = y;
      if (r < qr + kr) {
        // llm.c:488-492 (RoPE on q and k rows, adjacent pairs)
        const int i = (r < qr ? r : r - qr) % hd;
        const float2 cs = a.epi.rope_cs[(size_t)pos * (hd >> 1) + (i >> 1)];
        if ((i & 1) == 0)
          v = __fsub_rn(__fmul_rn(y, cs.x), __fmul_rn(partner, cs.y));
        else
          v = __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(y, cs.x));
      }
      if (r < qr) {
        a.out[r] = v;
      } else {
        // llm.c:673-681: store k, v at [pos][kv_dim]
        const bool is_k = r < qr + kr;
        const int e = is_k ? r - qr : r - qr - kr;
        void* cache = is_k ? a.epi.k_cache : a.epi.v_cache;
        const size_t idx = (size_t)pos * kr + e;
        if (a.epi.kv_type == TOSK_F16)
          reinterpret_cast<uint16_t*>(cache)[idx] = f2h(v);
        else
          reinterpret_cast<float*>(cache)[idx] = v;
      }
    }
  }
}

}  // namespace tos
