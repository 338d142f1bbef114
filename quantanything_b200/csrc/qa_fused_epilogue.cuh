// The per-element epilogue shared by every fused 8-bit layer kernel: the
// reference's requantize -> LUT -> residual Add -> (Concat rescale) sequence
// on one accumulator, stored as bytes.  See FusedEpilogue in qa_umma.cuh.
#pragma once
#include <cstdint>

#include "qa_fixedpoint.cuh"
#include "qa_umma.cuh"

namespace qa {

__device__ __forceinline__ int64_t stored_byte_value(uint8_t b, int is_signed) {
  return is_signed ? (int64_t)(int8_t)b : (int64_t)b;
}

// acc: exact accumulator of output pixel m, channel n (before bias).
__device__ __forceinline__ void fused_epilogue_store(const FusedEpilogue& e, int64_t acc,
                                                     int64_t m, int n) {
  const int64_t x = acc + (e.bias ? e.bias[n] : 0);
  int64_t q;
  if (e.fast) {
    q = requant_fast(x, e.mult[n], (int)(31 + e.shift[n]), e.zp, e.qmin, e.qmax);
  } else {
    q = requant_exact(x, e.mult[n], e.shift[n], e.zp, e.qmin, e.qmax);
  }
  if (e.lut) {
    int64_t idx = q - e.lut_offset;
    idx = idx < 0 ? 0 : (idx >= e.lut_len ? e.lut_len - 1 : idx);
    q = __ldg(e.lut + idx);
  }
  if (e.res) {
    const int64_t a = stored_byte_value(e.res[m * e.res_pix_stride + n], e.res_signed);
    const I128 ta = mbqm(a - e.za, e.ma, e.sa);
    I128 tb = mbqm(q - e.zb, e.mb, e.sb);
    if (e.sign < 0) tb = neg_i128(tb);
    q = clamp_i128(add_i128_i64(add_i128(ta, tb), e.add_zo), e.add_qmin, e.add_qmax);
  }
  if (e.out) e.out[m * e.out_pix_stride + n] = (uint8_t)q;
  if (e.out2) {
    int64_t q2;
    if (e.r_identity) {
      q2 = q < e.r_qmin ? e.r_qmin : (q > e.r_qmax ? e.r_qmax : q);
    } else {
      q2 = requant_exact(q - e.r_zp_in, e.r_m, e.r_s, e.r_zp_out, e.r_qmin, e.r_qmax);
    }
    e.out2[m * e.out2_pix_stride + n] = (uint8_t)q2;
  }
}

// int16 value of a two-plane tensor element (low byte at p, high byte
// `plane` bytes further on).
__device__ __forceinline__ int64_t plane16_value(const uint8_t* p, int64_t plane) {
  return (int64_t)(int16_t)((uint16_t)p[0] | ((uint16_t)p[plane] << 8));
}

__device__ __forceinline__ void plane16_store(uint8_t* p, int64_t plane, int64_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[plane] = (uint8_t)((v >> 8) & 0xFF);
}

// The same layer sequence on int16 values held as byte planes (16-bit
// graphs).  Requantize, Add and rescale always take the exact 128-bit mbqm:
// int16 accumulators reach 2^40 and more, past the 64-bit fast form.
__device__ __forceinline__ void fused_epilogue_store16(const FusedEpilogue& e, int64_t acc,
                                                       int64_t m, int n) {
  const int64_t x = acc + (e.bias ? e.bias[n] : 0);
  int64_t q = requant_exact(x, e.mult[n], e.shift[n], e.zp, e.qmin, e.qmax);
  if (e.lut) {
    int64_t idx = q - e.lut_offset;
    idx = idx < 0 ? 0 : (idx >= e.lut_len ? e.lut_len - 1 : idx);
    q = __ldg(e.lut + idx);
  }
  if (e.res) {
    const int64_t a = plane16_value(e.res + m * e.res_pix_stride + n, e.res_plane);
    const I128 ta = mbqm(a - e.za, e.ma, e.sa);
    I128 tb = mbqm(q - e.zb, e.mb, e.sb);
    if (e.sign < 0) tb = neg_i128(tb);
    q = clamp_i128(add_i128_i64(add_i128(ta, tb), e.add_zo), e.add_qmin, e.add_qmax);
  }
  if (e.out) plane16_store(e.out + m * e.out_pix_stride + n, e.out_plane, q);
  if (e.out2) {
    int64_t q2;
    if (e.r_identity) {
      q2 = q < e.r_qmin ? e.r_qmin : (q > e.r_qmax ? e.r_qmax : q);
    } else {
      q2 = requant_exact(q - e.r_zp_in, e.r_m, e.r_s, e.r_zp_out, e.r_qmin, e.r_qmax);
    }
    plane16_store(e.out2 + m * e.out2_pix_stride + n, e.out2_plane, q2);
  }
}

}  // namespace qa
