// gemv_fastmath.cuh - FAST GEMV arithmetic: integer block dot products on
// 24-bit fixed-point activations (the same products as runtime/nn/llm.c
// q4_0_dot32 / q8_0_dot32, llm.c:148-216, evaluated exactly in integers).
//
// A thread turns its 32 activations into X_i = rint(x_i / s) with a power of
// two s chosen so that max|X_i| <= 2^22 (relative precision ~2^-22 of the
// block maximum), split into three byte limbs X = X0 + 2^8 X1 + 2^16 X2
// (X0, X1 unsigned, X2 signed).  A block value is then exact integer
// arithmetic, 8 dp4a per limb:
//   Q4_0: Y = sum (n_i - 8) X_i = sum n X0 + 2^8 sum n X1 + 2^16 sum n X2 - 8 sum X
//         (|Y| <= 2^30; partial sums may wrap mod 2^32, the total cannot)
//   Q8_0: Y = sum q_i X_i, kept as (sum q X0 + 2^8 sum q X1) and sum q X2
// and the only roundings are float(Y), the scale product and the row sum, so
// a row is within ~1e-7 (normwise) of the exact one.
#pragma once
#include "tos_dev.cuh"

namespace tos {

// Limb words l[limb][w]: Q4_0 word 2k holds the elements of quant word k's
// low nibbles, 2k+1 those of its high nibbles; Q8_0 word j holds elements
// 4j..4j+3.  c = -8 * sum X (Q4_0, wrapping); s = 2^e (NaN for a block
// holding a non-finite value).
struct XFix {
  uint32_t l[3][8];
  int c;
  float s;
};

__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dp4a_us(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dp4a_su(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dp4a_ss(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Six dot-product chains per block (each limb split over the low- and
// high-nibble words, or even and odd words) keep the dependent dp4a runs
// short; the integer total is the same in any order (mod 2^32).
// Q4_0: the high nibbles stay in place (byte value 16 n, no shift per
// word), so the b chains hold 16x their sums.  Each limb's chains are small
// (|a| < 2^16, |b| < 2^20), so s_l = 16 a_l + b_l is exact and a multiple of
// 16, and Y = s0/16 + 2^4 s1 + 2^12 s2 + c (mod 2^32, exact since |Y| <= 2^30).
__device__ __forceinline__ float fast_q4_0(const uint4 q, const float d, const XFix& f) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  uint32_t a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = w[k] & 0x0F0F0F0Fu;
    const uint32_t hi = w[k] & 0xF0F0F0F0u;
    a0 = dp4a_uu(lo, f.l[0][2 * k], a0);
    a1 = dp4a_uu(lo, f.l[1][2 * k], a1);
    a2 = dp4a_us(lo, f.l[2][2 * k], a2);
    b0 = dp4a_uu(hi, f.l[0][2 * k + 1], b0);
    b1 = dp4a_uu(hi, f.l[1][2 * k + 1], b1);
    b2 = dp4a_us(hi, f.l[2][2 * k + 1], b2);
  }
  const uint32_t s0 = a0 * 16u + b0, s1 = a1 * 16u + b1, s2 = a2 * 16u + b2;
  const int y = (int)((s0 >> 4) + (s1 << 4) + (s2 << 12) + (uint32_t)f.c);
  return (float)y * (d * f.s);
}

__device__ __forceinline__ float fast_q8_0(const uint4 qa, const uint4 qb, const float d,
                                           const XFix& f) {
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  uint32_t a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    a0 = dp4a_su(w[j], f.l[0][j], a0);
    a1 = dp4a_su(w[j], f.l[1][j], a1);
    a2 = dp4a_ss(w[j], f.l[2][j], a2);
    b0 = dp4a_su(w[j + 1], f.l[0][j + 1], b0);
    b1 = dp4a_su(w[j + 1], f.l[1][j + 1], b1);
    b2 = dp4a_ss(w[j + 1], f.l[2][j + 1], b2);
  }
  const int lo = (int)((a0 + b0) + ((a1 + b1) << 8));
  return fmaf((float)(int)(a2 + b2), 65536.0f, (float)lo) * (d * f.s);
}

// Byte limbs 0, 1, 2 of four integers, each packed low to high.
__device__ __forceinline__ void pack_limbs(int a, int b, int c, int d, uint32_t& l0, uint32_t& l1,
                                           uint32_t& l2) {
  const uint32_t ab = prmt((uint32_t)a, (uint32_t)b, 0x5140u);   // a0 b0 a1 b1
  const uint32_t cd = prmt((uint32_t)c, (uint32_t)d, 0x5140u);   // c0 d0 c1 d1
  l0 = prmt(ab, cd, 0x5410u);
  l1 = prmt(ab, cd, 0x7632u);
  const uint32_t ab2 = prmt((uint32_t)a, (uint32_t)b, 0x0062u);  // a2 b2 . .
  const uint32_t cd2 = prmt((uint32_t)c, (uint32_t)d, 0x6200u);  // . . c2 d2
  l2 = prmt(ab2, cd2, 0x7610u);
}

template <int QB>
__device__ __forceinline__ void make_xfix(const float (&x)[32], XFix& f) {
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(x[i]));
  const int eb = (int)((__float_as_uint(m) >> 23) & 0xFF);   // biased exponent of the max
  const int e = max(eb - 127 - 21, -126);                      // max / 2^e < 2^22
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
  const bool finite = eb != 255;
  f.s = finite ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x7FC00000u);
  int sum = 0;
  // eight elements at a time (quant word k): rint(x / 2^e) - x * 2^-e is
  // exact and adding 1.5 * 2^23 rounds it to an integer held in the low
  // mantissa bits (|X| <= 2^22); a block with a non-finite value gets X = 0
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int X[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      X[j] = finite ? __float_as_int(fmaf(x[8 * k + j], inv, 12582912.0f)) - 0x4B400000 : 0;
      sum += X[j];
    }
    if constexpr (QB == 16) {
      // quant word k byte p holds elements 8k+2p (low nibble) and 8k+2p+1
      pack_limbs(X[0], X[2], X[4], X[6], f.l[0][2 * k], f.l[1][2 * k], f.l[2][2 * k]);
      pack_limbs(X[1], X[3], X[5], X[7], f.l[0][2 * k + 1], f.l[1][2 * k + 1], f.l[2][2 * k + 1]);
    } else {
      pack_limbs(X[0], X[1], X[2], X[3], f.l[0][2 * k], f.l[1][2 * k], f.l[2][2 * k]);
      pack_limbs(X[4], X[5], X[6], X[7], f.l[0][2 * k + 1], f.l[1][2 * k + 1], f.l[2][2 * k + 1]);
    }
  }
  f.c = -8 * sum;
}

// Cooperative form of make_xfix: eight consecutive lanes (chunk c = lane & 7)
// hold the block's elements 4c..4c+3 in v.  Each lane returns the limb words
// it stores, word index wi of limbs 0..2, and the block's c and s.
template <int QB>
__device__ __forceinline__ void xfix_group(float4 v, int c, uint32_t& w0, uint32_t& w1, uint32_t& w2,
                                           int& wi, int& csum, float& s) {
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  const int eb = (int)((__float_as_uint(m) >> 23) & 0xFF);
  const int e = max(eb - 127 - 21, -126);
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
  s = eb == 255 ? __uint_as_float(0x7FC00000u) : __uint_as_float((uint32_t)(e + 127) << 23);
  int X0 = 0, X1 = 0, X2 = 0, X3 = 0;
  if (eb != 255) {
    X0 = __float_as_int(fmaf(v.x, inv, 12582912.0f)) - 0x4B400000;
    X1 = __float_as_int(fmaf(v.y, inv, 12582912.0f)) - 0x4B400000;
    X2 = __float_as_int(fmaf(v.z, inv, 12582912.0f)) - 0x4B400000;
    X3 = __float_as_int(fmaf(v.w, inv, 12582912.0f)) - 0x4B400000;
  }
  int sum = (X0 + X1) + (X2 + X3);
  sum += __shfl_xor_sync(0xffffffffu, sum, 4);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  csum = -8 * sum;
  if constexpr (QB == 16) {
    // elements 4c..4c+3 = 8k + {0,1,2,3} + 4(c & 1), k = c >> 1: the low-
    // nibble word 2k takes (e0, e2) in half (c & 1), the high-nibble word
    // 2k+1 takes (e1, e3); the partner lane c ^ 1 supplies the other half
    const bool odd = (c & 1) != 0;
    uint32_t out[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      const uint32_t sel = (uint32_t)l | ((uint32_t)(4 + l) << 4);
      const uint32_t h0 = prmt((uint32_t)X0, (uint32_t)X2, sel) & 0xFFFFu;
      const uint32_t h1 = prmt((uint32_t)X1, (uint32_t)X3, sel) & 0xFFFFu;
      const uint32_t r = __shfl_xor_sync(0xffffffffu, odd ? h0 : h1, 1);
      out[l] = odd ? (r | (h1 << 16)) : (h0 | (r << 16));
    }
    w0 = out[0]; w1 = out[1]; w2 = out[2];
    wi = 2 * (c >> 1) + (odd ? 1 : 0);
  } else {
    pack_limbs(X0, X1, X2, X3, w0, w1, w2);   // quant word c = elements 4c..4c+3
    wi = c;
  }
}

// FAST value of block b of row r of a shared-memory stage (quants
// [rows][nb][QB], fp16 scales [rows][nbp]).
template <int QB>
__device__ __forceinline__ float block_value_fast(const uint8_t* stq, const uint16_t* sts, int r, int b,
                                                  int nb, int nbp, const XFix& f) {
  const float d = h2f(sts[r * nbp + b]);
  if constexpr (QB == 16) {
    const uint4 q = *reinterpret_cast<const uint4*>(stq + ((size_t)r * nb + b) * 16);
    return fast_q4_0(q, d, f);
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(stq + ((size_t)r * nb + b) * 32);
    return fast_q8_0(p[0], p[1], d, f);
  }
}

}  // namespace tos
