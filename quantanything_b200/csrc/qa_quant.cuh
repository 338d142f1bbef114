// Exact per-tensor quantization of float32 values on the device: the
// reference's qa_quantize_f32 (qa_kernels.cpp:363-386),
//   q = clamp(rint((double)x / scale) + zp, qmin, qmax)
// (NaN -> 0 in the low byte, as x86's truncating conversion leaves it),
// computed through a float product with 1/scale and exact fallbacks.
#pragma once
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>

namespace qa {

// The double-precision definition, for the rare elements the float path
// cannot decide.
__device__ __forceinline__ uint32_t quantize_byte(float xv, double scale, double zp,
                                                  double qmin, double qmax) {
  double v = rint((double)xv / scale) + zp;
  if (v < qmin) v = qmin;
  if (qmax < v) v = qmax;
  return (uint32_t)(int32_t)v & 0xFFu;
}

struct QuantK {
  float inv;  // fl32(1 / scale)
  float zp, qmin, qmax;
  float lo, hi;      // qmin - zp, qmax - zp
  float magic_zp;    // 1.5 * 2^23 + zp
  float t_lo, t_hi;  // 1.5 * 2^23 + qmin, 1.5 * 2^23 + qmax
  int32_t zp_i, qmin_i, qmax_i;
  double scale, zpd, qmind, qmaxd;
};

// Clamp-then-round in the float adder.  With lo = qmin - zp and hi =
// qmax - zp integers of at most 2^10, clamp(rint(d) + zp) ==
// rint(clamp(m, lo, hi)) + zp whenever m = fl32(x * fl32(1/scale)) and the
// double quotient d = x / scale round alike, which holds (|m - d| < 2^-12 on
// that range) unless the clamped product lies within 2^-11 of a
// half-integer; saturated and infinite products clamp to an integer and
// pass.  t = mc + (1.5 * 2^23 + zp) then holds rint(mc) + zp in its low
// mantissa bits, so its low byte is the quantized byte.  `ok` is cleared
// near half-integers, for NaN and when the host could not invert the scale
// (inv = NaN): the caller then uses quantize_byte.
__device__ __forceinline__ uint32_t quantize_bits_try(float xv, const QuantK& k, bool& ok) {
  const float m = __fmul_rn(xv, k.inv);  // no contraction into the adds below
  const float mc = fminf(fmaxf(m, k.lo), k.hi);
  const float t = __fadd_rn(mc, k.magic_zp);
  const float r = __fsub_rn(t, k.magic_zp);
  ok = ok && (fabsf(mc - r) < 0.49951171875f) && (m == m);  // 0.5 - 2^-11
  return __float_as_uint(t);
}

// The quantized byte in six instructions: the product x * inv is rounded to
// an integer inside one FMA, t = fl(x * inv + (1.5 * 2^23 + zp)) =
// 1.5 * 2^23 + zp + rint(x * inv) while |x * inv + zp| < 2^22, and clamped
// as a float to [1.5 * 2^23 + qmin, 1.5 * 2^23 + qmax]; the low byte of the
// clamped word is the byte.  The tie test takes the rounding's residual from
// a second FMA: r = t - (1.5 * 2^23 + zp) is exact, d = fl(x * inv - r) is
// the exact residual rounded once (|d| <= 1/2).
// Error bound: inv = fl32(1 / scale) carries a relative error below
// 2^-24 + 2^-53, so for |q| <= 1025.5 (q = x / scale, the range where the
// clamp can leave the rounding visible: make_quant_k bounds |qmin - zp| and
// |qmax - zp| by 1024) |x * inv - q| < 2^-13.99, and
// |q - r| <= |d| (1 + 2^-23) + 2^-13.99 < 1/2 - 2^-14 whenever
// |d| < 1/2 - 2^-13; the double quotient fl64(q) is within 2^-42 of q, so
// rint(fl64(q)) = r as well and the clamped value is the reference's.  A
// product beyond the clamp is decided by the clamp alone (rounding is
// monotonic and |x * inv - q| < 1/2 there), whatever d says; beyond 2^22,
// where d is no residual, `ok` may go either way.  `ok` is cleared in the
// band (2^-12 of uniform fractions), for NaN and infinite inputs and when
// the host could not invert the scale (inv = NaN); the caller then uses
// quantize_byte_near_tie, which holds for every input.
__device__ __forceinline__ uint32_t quantize_bits_fma(float xv, const QuantK& k, bool& ok) {
  const float t = __fmaf_rn(xv, k.inv, k.magic_zp);
  const float r = __fsub_rn(t, k.magic_zp);
  const float d = __fmaf_rn(xv, k.inv, -r);
  ok = ok & (fabsf(d) < 0.4998779296875f);  // 1/2 - 2^-13; false for NaN
  return __float_as_uint(fminf(fmaxf(t, k.t_lo), k.t_hi));
}

// The byte of an element the float paths could not decide, without a
// division in the common case.  For a finite x with unclamped float product
// m = fl32(x * inv), the exact quotient q = x / scale is within 2^-12 of m,
// so with k = floor(m) the reference's rint(fl64(q)) is k or k + 1 (an
// element that reaches this is near k + 1/2); a product clamped to lo or hi
// leaves k = lo or hi, and the clamp of k or k + 1 is right there as well.
// With scale > 0 the sign of t = fma(k + 1/2, scale, -x) (one rounding of
// the exact (k + 1/2 - q) * scale) says which, unless |t| <= 2^-42 * scale,
// where fl64(q) may round onto the tie itself (|q| < 2^11, so its half ulp
// is below 2^-42).  NaN, a scale the host could not invert, a negative
// scale and those last cases take the double division (quantize_byte).
static __device__ __noinline__ uint32_t quantize_byte_call(float xv, double scale, double zp,
                                                   double qmin, double qmax) {
  return quantize_byte(xv, scale, zp, qmin, qmax);
}

__device__ __forceinline__ uint32_t quantize_byte_near_tie(float xv, const QuantK& k) {
  const float m = __fmul_rn(xv, k.inv);
  if (!(m == m) || !(k.scale > 0.0))
    return quantize_byte_call(xv, k.scale, k.zpd, k.qmind, k.qmaxd);
  const float mc = fminf(fmaxf(m, k.lo), k.hi);
  const float kf = floorf(mc);
  const double t = fma((double)kf + 0.5, k.scale, -(double)xv);
  if (fabs(t) <= k.scale * 0x1p-42) return quantize_byte_call(xv, k.scale, k.zpd, k.qmind, k.qmaxd);
  const int v = (int)kf + (t < 0.0 ? 1 : 0) + k.zp_i;
  return (uint32_t)min(max(v, k.qmin_i), k.qmax_i) & 0xFFu;
}

// The quantized value as an integer (not only its byte).
__device__ __forceinline__ int32_t quantize_value(float xv, const QuantK& k) {
  bool ok = true;
  const uint32_t t = quantize_bits_try(xv, k, ok);
  if (ok) return (int32_t)(t - 0x4B400000u);  // rint(mc) + zp
  const uint32_t b = quantize_byte(xv, k.scale, k.zpd, k.qmind, k.qmaxd);
  return k.qmin_i < 0 ? (int32_t)(int8_t)b : (int32_t)b;
}

// ---- 16-bit outputs (qmin >= -32768, qmax <= 32767): the same FMA
// rounding with the error bound of the wider range.  With |qmin - zp|,
// |qmax - zp| and |zp| at most 2^16 (make_quant_k16), |q| <= 2^16 + 1 where
// the clamp can leave the rounding visible, so |x * inv - q| < 2^-7.99 and
// |d| < 1/2 - 2^-7 proves |q - r| < 1/2 - 2^-9, beyond the 2^-36 half ulp
// of the double quotient there; t keeps its integer form while
// |x * inv + zp| < 2^22.  The value is the low 16 bits of the returned
// word (its mantissa holds 2^22 + value).
__device__ __forceinline__ uint32_t quantize_bits16_fma(float xv, const QuantK& k, bool& ok) {
  const float t = __fmaf_rn(xv, k.inv, k.magic_zp);
  const float r = __fsub_rn(t, k.magic_zp);
  const float d = __fmaf_rn(xv, k.inv, -r);
  ok = ok & (fabsf(d) < 0.4921875f);  // 1/2 - 2^-7; false for NaN
  return __float_as_uint(fminf(fmaxf(t, k.t_lo), k.t_hi));
}

// The reference's value in double precision (NaN converts to 0, whose low
// 16 bits equal those of x86's 0x80000000).
static __device__ __noinline__ int32_t quantize_value_double(float xv, double scale, double zp,
                                                             double qmin, double qmax) {
  double v = rint((double)xv / scale) + zp;
  if (v < qmin) v = qmin;
  if (qmax < v) v = qmax;
  return (int32_t)v;
}

// The value of an element quantize_bits16_fma could not decide: as
// quantize_byte_near_tie, with m = fl32(x * inv) within 2^-7 of q on the
// 16-bit range (so rint(fl64(q)) is floor(m) or floor(m) + 1 for an
// unclamped m) and the double division taken when |k + 1/2 - q| may be
// within the 2^-36 half ulp of fl64(q) (|q| < 2^17).
__device__ __forceinline__ int32_t quantize_value16_near_tie(float xv, const QuantK& k) {
  const float m = __fmul_rn(xv, k.inv);
  if (!(m == m) || !(k.scale > 0.0))
    return quantize_value_double(xv, k.scale, k.zpd, k.qmind, k.qmaxd);
  const float mc = fminf(fmaxf(m, k.lo), k.hi);
  const float kf = floorf(mc);
  const double t = fma((double)kf + 0.5, k.scale, -(double)xv);
  if (fabs(t) <= k.scale * 0x1p-35)
    return quantize_value_double(xv, k.scale, k.zpd, k.qmind, k.qmaxd);
  const int v = (int)kf + (t < 0.0 ? 1 : 0) + k.zp_i;
  return min(max(v, k.qmin_i), k.qmax_i);
}

// Word of four channel bytes from quantize_bits_try results (byte 0 of each).
__device__ __forceinline__ uint32_t pack_bytes(uint32_t b0, uint32_t b1, uint32_t b2,
                                               uint32_t b3) {
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// Four channel bytes of one pixel (channels >= C hold `pad`), exactly; the
// channels are read from `src` at a stride of `plane` floats.
__device__ __noinline__ inline uint32_t quantize_word_exact(const float* src, int64_t plane,
                                                            int C, uint32_t pad,
                                                            const QuantK& k) {
  uint32_t w = 0;
  for (int c = 0; c < 4; ++c)
    w |= (c < C ? quantize_byte(src[c * plane], k.scale, k.zpd, k.qmind, k.qmaxd) : pad)
         << (8 * c);
  return w;
}

// Host side: 1/scale in float, or NaN (every element takes the double
// division) when the scale or the integer bounds are outside the range the
// error bound covers.
inline QuantK make_quant_k(double scale, int64_t zp, int64_t qmin, int64_t qmax) {
  QuantK k;
  k.scale = scale;
  k.zpd = (double)zp;
  k.qmind = (double)qmin;
  k.qmaxd = (double)qmax;
  k.zp = (float)zp;
  k.qmin = (float)qmin;
  k.qmax = (float)qmax;
  k.zp_i = (int32_t)zp;
  k.qmin_i = (int32_t)qmin;
  k.qmax_i = (int32_t)qmax;
  k.lo = (float)(qmin - zp);
  k.hi = (float)(qmax - zp);
  k.magic_zp = 12582912.0f + (float)zp;
  k.t_lo = 12582912.0f + (float)qmin;
  k.t_hi = 12582912.0f + (float)qmax;
  const bool ok = std::fabs(scale) > 1e-30 && std::fabs(scale) < 1e30 &&
                  std::llabs(zp) <= 1024 && std::llabs(qmin - zp) <= 1024 &&
                  std::llabs(qmax - zp) <= 1024 && qmin <= qmax;
  k.inv = ok ? (float)(1.0 / scale) : std::nanf("");
  return k;
}

// make_quant_k for 16-bit outputs: the float path covers |qmin - zp|,
// |qmax - zp| and |zp| up to 2^16 (quantize_bits16_fma's error bound).
inline QuantK make_quant_k16(double scale, int64_t zp, int64_t qmin, int64_t qmax) {
  QuantK k = make_quant_k(scale, zp, qmin, qmax);
  const bool ok = std::fabs(scale) > 1e-30 && std::fabs(scale) < 1e30 &&
                  std::llabs(zp) <= 65536 && std::llabs(qmin - zp) <= 65536 &&
                  std::llabs(qmax - zp) <= 65536 && qmin <= qmax;
  k.inv = ok ? (float)(1.0 / scale) : std::nanf("");
  return k;
}

inline bool byte_range_host(int64_t lo, int64_t hi) { return lo >= -128 && hi <= 255 && lo <= hi; }

}  // namespace qa
