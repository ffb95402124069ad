// tos_dev.cuh - device helpers shared by the sm_100a kernels.
//
// All arithmetic that must reproduce the reference bit for bit is written with
// the IEEE round-to-nearest intrinsics (__fadd_rn, __fmul_rn, __fdiv_rn,
// __fsqrt_rn) so that no FMA contraction can change a rounding; the library is
// additionally compiled with -fmad=false.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace tos {

// ---------------------------------------------------------------------------
// Reference scalar math (restated from runtime/nn/llm.c)
// ---------------------------------------------------------------------------

// llm.c:123-131: (1 + x/256)^256 by eight squarings, clamped at +-88.
// x/256 is exact division by a power of two; written as a correctly rounded
// division so that subnormal results round exactly as the reference does.
__device__ __forceinline__ float ref_expf(float x) {
  if (x > 88.0f) return 3.4e38f;
  if (x < -88.0f) return 0.0f;
  float y = __fadd_rn(1.0f, __fdiv_rn(x, 256.0f));
#pragma unroll
  for (int i = 0; i < 8; ++i) y = __fmul_rn(y, y);
  return y;
}

// llm.c:538-544: s = 1/(1 + exp(-x)); x*s
__device__ __forceinline__ float ref_silu(float x) {
  float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, ref_expf(-x)));
  return __fmul_rn(x, s);
}

// Packed fp32 product that is never fused with the add consuming it.
// The compiler contracts __fmul2_rn followed by __fadd2_rn into a packed FMA
// (one rounding instead of two) even without -fmad; passing the product
// through an opaque register barrier keeps the reference's two roundings.
// Bit-exactness of every user is covered by the GPU parity tests.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  const float2 m = __fmul2_rn(a, b);
  unsigned long long u =
      (unsigned long long)__float_as_uint(m.x) | ((unsigned long long)__float_as_uint(m.y) << 32);
  asm volatile("" : "+l"(u));
  return make_float2(__uint_as_float((unsigned)u), __uint_as_float((unsigned)(u >> 32)));
}

__device__ __forceinline__ float h2f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f2h(float f) {
  return __half_as_ushort(__float2half_rn(f));
}

// ---------------------------------------------------------------------------
// Shared-memory addressing, mbarriers and bulk copies (sm_90+ PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait limit: about two seconds of SM clock at 1.9 GHz.  A wait that runs out
// records `code` in *err and returns false; the caller then leaves its loop.
constexpr long long kWaitCycles = 4000000000ll;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kWaitCycles) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes.  No multicast.  Both addresses 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: wait for the preceding kernel's writes /
// allow the next kernel to begin its prologue.  No-ops without PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

}  // namespace tos
