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

// Out-of-line exact forms for the rare channels / layers the 64-bit forms
// do not cover (keeps the unrolled hot loop small).
__device__ __noinline__ inline int64_t requant_exact_cold(int64_t x, int64_t m, int64_t s,
                                                          int64_t bias, int64_t lo,
                                                          int64_t hi) {
  return requant_exact(x, m, s, bias, lo, hi);
}

__device__ __noinline__ inline int64_t add_exact_cold(const FusedEpilogue& e, int64_t a,
                                                      int64_t q) {
  const I128 ta = mbqm(a - e.za, e.ma, e.sa);
  I128 tb = mbqm(q - e.zb, e.mb, e.sb);
  if (e.sign < 0) tb = neg_i128(tb);
  return clamp_i128(add_i128_i64(add_i128(ta, tb), e.add_zo), e.add_qmin, e.add_qmax);
}

// Sixteen consecutive output channels n0 .. n0 + cnt - 1 (cnt <= 16) of
// pixel m: the per-element sequence of fused_epilogue_store16, with the
// residual read and both planes of each output stored 16 bytes at a time
// when the run is complete and 16-byte aligned.
__device__ __forceinline__ bool aligned16(const uint8_t* p, int64_t plane) {
  return ((reinterpret_cast<uintptr_t>(p) | (uint64_t)plane) & 15) == 0;
}

// s_lut: the activation table in shared memory (int16 entries), or null to
// read e.lut from global memory.
// One output channel's requantize parameters staged in shared memory by a
// kernel whose CTA keeps one column tile: bias, multiplier, total shift
// (31 + shift) and whether the high-word form applies.
struct ChanParams16 {
  int64_t bias;
  int64_t mult;
  int32_t ts;
  int32_t hi;
};

__device__ __forceinline__ void fused_epilogue_store16_run(const FusedEpilogue& e,
                                                           const int64_t (&acc)[16], int64_t m,
                                                           int n0, int cnt,
                                                           const int16_t* s_lut = nullptr,
                                                           const ChanParams16* s_par = nullptr,
                                                           bool par_all_hi = false) {
  // Phased so that the independent loads of the sixteen channels are in
  // flight together: channel parameters, then requantize, then the sixteen
  // table lookups, then the residual terms and the stores.  Columns past
  // cnt compute on channel n0's parameters and are not stored.
  const uint8_t* rp = e.res ? e.res + m * e.res_pix_stride + n0 : nullptr;
  uint8_t* op = e.out ? e.out + m * e.out_pix_stride + n0 : nullptr;
  uint8_t* op2 = e.out2 ? e.out2 + m * e.out2_pix_stride + n0 : nullptr;
  const bool full = cnt == 16;
  int64_t q[16];
  if (s_par && par_all_hi) {
    // every staged channel takes the high-word form
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const ChanParams16 c = s_par[j < cnt ? j : 0];
      q[j] = requant_hi32(acc[j] + c.bias, c.mult, c.ts, e.zp, e.qmin, e.qmax);
    }
  } else if (s_par) {
    // s_par[j]: channel n0 + j (columns past cnt hold channel n0's values)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const ChanParams16 c = s_par[j < cnt ? j : 0];
      q[j] = c.hi ? requant_hi32(acc[j] + c.bias, c.mult, c.ts, e.zp, e.qmin, e.qmax)
                  : requant_exact_cold(acc[j] + c.bias, c.mult, (int64_t)c.ts - 31, e.zp,
                                       e.qmin, e.qmax);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = n0 + (j < cnt ? j : 0);
      const int64_t b = e.bias ? __ldg(e.bias + n) : 0;
      const int64_t mv = __ldg(e.mult + n), sv = __ldg(e.shift + n);
      // int16 accumulators pass 2^40: the high-word form when it applies (the
      // usual positive M0 in [2^30, 2^31); e.fast: the host proved it for
      // every channel of the layer), else the 128-bit mbqm
      q[j] = (e.fast || hi32_applies(mv, 31 + sv))
                 ? requant_hi32(acc[j] + b, mv, (int)(31 + sv), e.zp, e.qmin, e.qmax)
                 : requant_exact_cold(acc[j] + b, mv, sv, e.zp, e.qmin, e.qmax);
    }
  }
  if (e.lut) {
    int32_t t[16];
    // q lies in [qmin, qmax] (16-bit): the table index fits 32 bits
    const int32_t off = (int32_t)e.lut_offset, last = (int32_t)e.lut_len - 1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int32_t idx = min(max((int32_t)q[j] - off, 0), last);
      t[j] = s_lut ? (int32_t)s_lut[idx] : __ldg(e.lut + idx);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) q[j] = t[j];
  }
  if (rp) {
    int64_t a[16];
    if (full && aligned16(rp, e.res_plane)) {
      const uint4 rl = *reinterpret_cast<const uint4*>(rp);
      const uint4 rh = *reinterpret_cast<const uint4*>(rp + e.res_plane);
      const uint32_t lw[4] = {rl.x, rl.y, rl.z, rl.w}, hw[4] = {rh.x, rh.y, rh.z, rh.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t l = (lw[j >> 2] >> (8 * (j & 3))) & 0xFF;
        const uint32_t h = (hw[j >> 2] >> (8 * (j & 3))) & 0xFF;
        a[j] = (int64_t)(int16_t)(uint16_t)(l | (h << 8));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) a[j] = plane16_value(rp + (j < cnt ? j : 0), e.res_plane);
    }
    // both terms are int16-range values times multipliers: one 64-bit
    // product each when the multipliers and shifts allow it
    const bool small = small_applies(e.ma, e.sa) && small_applies(e.mb, e.sb) &&
                       e.za > -32768 && e.za < 32768 && e.zb > -32768 && e.zb < 32768;
    if (small) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t ta = mbqm_small(a[j] - e.za, e.ma, (int)(31 + e.sa));
        const int64_t tb = mbqm_small(q[j] - e.zb, e.mb, (int)(31 + e.sb));
        int64_t v = ta + (e.sign < 0 ? -tb : tb) + e.add_zo;
        v = v < e.add_qmin ? e.add_qmin : v;
        q[j] = v > e.add_qmax ? e.add_qmax : v;
      }
    } else {
      for (int j = 0; j < 16; ++j) q[j] = add_exact_cold(e, a[j], q[j]);
    }
  }
  uint32_t wl[4] = {0, 0, 0, 0}, wh[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    wl[j >> 2] |= (uint32_t)(q[j] & 0xFF) << (8 * (j & 3));
    wh[j >> 2] |= (uint32_t)((q[j] >> 8) & 0xFF) << (8 * (j & 3));
  }
  auto put = [&](uint8_t* p, int64_t plane, const uint32_t (&l)[4], const uint32_t (&h)[4]) {
    if (full && aligned16(p, plane)) {
      *reinterpret_cast<uint4*>(p) = make_uint4(l[0], l[1], l[2], l[3]);
      *reinterpret_cast<uint4*>(p + plane) = make_uint4(h[0], h[1], h[2], h[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j < cnt) {
          p[j] = (uint8_t)(l[j >> 2] >> (8 * (j & 3)));
          p[j + plane] = (uint8_t)(h[j >> 2] >> (8 * (j & 3)));
        }
      }
    }
  };
  if (op) put(op, e.out_plane, wl, wh);
  if (op2) {
    uint32_t ml[4] = {0, 0, 0, 0}, mh[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t v = q[j];
      int64_t q2;
      if (e.r_identity) {
        q2 = v < e.r_qmin ? e.r_qmin : (v > e.r_qmax ? e.r_qmax : v);
      } else if (small_applies(e.r_m, e.r_s) && e.r_zp_in > -32768 && e.r_zp_in < 32768) {
        q2 = mbqm_small(v - e.r_zp_in, e.r_m, (int)(31 + e.r_s)) + e.r_zp_out;
        q2 = q2 < e.r_qmin ? e.r_qmin : (q2 > e.r_qmax ? e.r_qmax : q2);
      } else {
        q2 = requant_exact_cold(v - e.r_zp_in, e.r_m, e.r_s, e.r_zp_out, e.r_qmin, e.r_qmax);
      }
      ml[j >> 2] |= (uint32_t)(q2 & 0xFF) << (8 * (j & 3));
      mh[j >> 2] |= (uint32_t)((q2 >> 8) & 0xFF) << (8 * (j & 3));
    }
    put(op2, e.out2_plane, ml, mh);
  }
}

}  // namespace qa
