// Exact fixed-point requantization arithmetic for device code.
//
// The reference defines requantization on a signed 128-bit product
// (quantization/kernels/qa_kernels.cpp:188-205, `mbqm` and `clamp128`):
//
//   p  = (i128)x * (i128)mult
//   ts = 31 + shift
//   ts >  0 : r = (p + 2^(ts-1)) >> ts        (ts capped at 120, arithmetic)
//   ts <= 0 : r = p * 2^(-ts)                 (-ts capped at 60, wraps mod 2^128)
//   out = clamp(r + bias, lo, hi)             (compare on 128 bits)
//
// GPUs have no 128-bit integer type in hardware, so the product is carried
// as two 64-bit halves: the low half from a 64-bit multiply and the high
// half from __mul64hi.  Every step is exact, including the wrapping left
// shift, so the result is bit-identical to the reference for every int64
// input.
//
// `mbqm_fast` is the single-64-bit variant used when the host has proved
// that |x * mult| + 2^(ts-1) < 2^63 and 1 <= ts <= 62 for every value a
// kernel can see; it then computes the same number with one IMAD.WIDE.
#pragma once
#include <cstdint>

namespace qa {

struct I128 {
  uint64_t lo;
  int64_t hi;
};

__device__ __forceinline__ I128 mul_i64_i64(int64_t a, int64_t b) {
  I128 r;
  r.lo = (uint64_t)a * (uint64_t)b;
  r.hi = __mul64hi(a, b);
  return r;
}

__device__ __forceinline__ I128 add_i128_i64(I128 a, int64_t b) {
  I128 r;
  r.lo = a.lo + (uint64_t)b;
  const uint64_t carry = r.lo < a.lo ? 1u : 0u;
  r.hi = (int64_t)((uint64_t)a.hi + (uint64_t)(b >> 63) + carry);
  return r;
}

__device__ __forceinline__ I128 add_i128(I128 a, I128 b) {
  I128 r;
  r.lo = a.lo + b.lo;
  const uint64_t carry = r.lo < a.lo ? 1u : 0u;
  r.hi = (int64_t)((uint64_t)a.hi + (uint64_t)b.hi + carry);
  return r;
}

__device__ __forceinline__ I128 neg_i128(I128 a) {
  I128 r;
  r.lo = ~a.lo + 1u;
  r.hi = (int64_t)(~(uint64_t)a.hi + (r.lo == 0 ? 1u : 0u));
  return r;
}

// Round-half-up arithmetic right shift by ts in [1, 120].
__device__ __forceinline__ I128 round_shift_right(I128 p, int ts) {
  // p + 2^(ts-1)
  const int h = ts - 1;
  if (h < 64) {
    p = add_i128(p, I128{(uint64_t)1 << h, 0});
  } else {
    p.hi = (int64_t)((uint64_t)p.hi + ((uint64_t)1 << (h - 64)));
  }
  I128 r;
  if (ts < 64) {
    r.lo = (p.lo >> ts) | ((uint64_t)p.hi << (64 - ts));
    r.hi = p.hi >> ts;
  } else if (ts == 64) {
    r.lo = (uint64_t)p.hi;
    r.hi = p.hi >> 63;
  } else {
    r.lo = (uint64_t)(p.hi >> (ts - 64));
    r.hi = p.hi >> 63;
  }
  return r;
}

// Wrapping left shift by k in [0, 60].
__device__ __forceinline__ I128 shift_left(I128 p, int k) {
  if (k == 0) return p;
  I128 r;
  r.hi = (int64_t)(((uint64_t)p.hi << k) | (p.lo >> (64 - k)));
  r.lo = p.lo << k;
  return r;
}

// mbqm of qa_kernels.cpp:196-205 on the 128-bit pair.
__device__ __forceinline__ I128 mbqm(int64_t x, int64_t mult, int64_t shift) {
  const I128 p = mul_i64_i64(x, mult);
  int64_t ts = 31 + shift;
  if (ts > 0) {
    if (ts > 120) ts = 120;
    return round_shift_right(p, (int)ts);
  }
  if (ts < -60) ts = -60;
  return shift_left(p, (int)(-ts));
}

// clamp128 of qa_kernels.cpp:188-192.
__device__ __forceinline__ int64_t clamp_i128(I128 v, int64_t lo, int64_t hi) {
  // v < lo  <=>  (v.hi, v.lo) < (sign(lo), lo) lexicographically (signed hi)
  const int64_t lo_hi = lo >> 63, hi_hi = hi >> 63;
  if (v.hi < lo_hi || (v.hi == lo_hi && v.lo < (uint64_t)lo)) return lo;
  if (v.hi > hi_hi || (v.hi == hi_hi && v.lo > (uint64_t)hi)) return hi;
  return (int64_t)v.lo;
}

// clamp(mbqm(x, m, s) + bias, lo, hi): the requantize core.
__device__ __forceinline__ int64_t requant_exact(int64_t x, int64_t m, int64_t s,
                                                 int64_t bias, int64_t lo,
                                                 int64_t hi) {
  return clamp_i128(add_i128_i64(mbqm(x, m, s), bias), lo, hi);
}

// Fast variant; valid only under the host-checked bounds described above.
__device__ __forceinline__ int64_t requant_fast(int64_t x, int64_t m, int ts,
                                                int64_t bias, int64_t lo,
                                                int64_t hi) {
  const int64_t p = x * m;
  int64_t r = ((p + ((int64_t)1 << (ts - 1))) >> ts) + bias;
  r = r < lo ? lo : r;
  return r > hi ? hi : r;
}

// clamp(mbqm(x, m, s) + bias, lo, hi) for 0 <= m < 2^31 and
// 32 <= ts = 31 + s <= 94, exact for every int64 x without 128-bit
// arithmetic.  With x = xh * 2^32 + xl (xl the unsigned low word),
//   x * m + 2^(ts-1) = C * 2^32 + low,  0 <= low < 2^32,
//   C = xh * m + hi32(xl * m) + 2^(ts-33)          (ts >= 33)
// so floor(. / 2^ts) = C >> (ts - 32): the low word cannot move the floor
// when ts >= 32.  |C| < 2^62 + 2^61 + 2^31, so nothing overflows.  At
// ts = 32 the rounding term 2^31 is added to the low product before its
// high word is taken.
__device__ __forceinline__ int64_t requant_hi32(int64_t x, int64_t m, int ts, int64_t bias,
                                                int64_t lo, int64_t hi) {
  // x >> 32 always fits int32 and 0 <= m < 2^31: both partial products are
  // single 32 x 32 -> 64-bit multiplies
  const int32_t xh = (int32_t)(x >> 32);
  const int32_t m32 = (int32_t)m;
  const int64_t a = (int64_t)xh * (int64_t)m32;
  const uint64_t xlm = (uint64_t)(uint32_t)x * (uint64_t)(uint32_t)m32;
  int64_t r;
  if (ts == 32) {
    r = a + (int64_t)((xlm + (1ull << 31)) >> 32);
  } else {
    r = (a + (int64_t)(xlm >> 32) + ((int64_t)1 << (ts - 33))) >> (ts - 32);
  }
  r += bias;
  r = r < lo ? lo : r;
  return r > hi ? hi : r;
}

__device__ __forceinline__ bool hi32_applies(int64_t m, int64_t ts) {
  return m >= 0 && m < ((int64_t)1 << 31) && ts >= 32 && ts <= 94;
}

// mbqm for |x| < 2^31 when |m| < 2^31 and 1 <= ts <= 62 (small_applies):
// |x * m| + 2^(ts-1) < 2^63, so one 64-bit product is exact.
__device__ __forceinline__ int64_t mbqm_small(int64_t x, int64_t m, int ts) {
  return (x * m + ((int64_t)1 << (ts - 1))) >> ts;
}

__device__ __forceinline__ bool small_applies(int64_t m, int64_t s) {
  return m > -((int64_t)1 << 31) && m < ((int64_t)1 << 31) && s >= -30 && s <= 31;
}

}  // namespace qa
