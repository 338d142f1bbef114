// Tensor-core (tcgen05, kind::i8) implicit-GEMM contraction: declarations.
//
// One kernel template serves every integer GEMM / convolution that maps
// onto 8-bit tensor-core tiles:
//   * activations are NHWC byte planes (a GEMM's [M, K] matrix is the
//     1x1 image case), gathered per 128x128-byte K-block with cp.async into
//     the 128-byte swizzled shared-memory layout the MMA reads;
//   * weights are [Cout, K] K-major byte planes loaded by TMA;
//   * accumulators live in TMEM and are drained by an epilogue warpgroup.
// 8-bit operands use one plane each.  16-bit operands are split exactly
// into a signed high byte and an unsigned low byte (v = 256*hi + lo), and
// the four partial products land in three TMEM accumulators combined as
// ll + 256*(lh + hl) + 65536*hh.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "qa_direct.cuh"

namespace qa {

// Epilogue of the fused int8 path (device-resident executor).  Values are
// exactly the reference's layer sequence:
//   q   = clamp(mbqm(acc + bias[c], mult[c], shift[c]) + zp, qmin, qmax)
//         (ConvQuantize / GemmQuantize + requantize, quant_layers.py:320-341)
//   q   = lut[clamp(q - lut_offset, 0, lut_len - 1)]        (optional LUT)
//   q   = clamp(mbqm(res - za, ma, sa) + sign*mbqm(q - zb, mb, sb) + add_zo)
//         (optional residual AddQuantize, qa_kernels.cpp:319-331)
//   out[pixel, c]  = q                                      (optional)
//   out2[pixel, c] = clamp(mbqm(q - r_zp_in, r_m, r_s) + r_zp_out)
//         (optional rescaled copy into a Concat slice, quant_layers.py:549-560)
struct FusedEpilogue {
  const int64_t* bias;   // per output channel (length >= Cout), may be null
  const int64_t* mult;   // per output channel
  const int64_t* shift;  // per output channel
  int64_t zp, qmin, qmax;
  int32_t fast;          // host proved the 64-bit requantize path exact
  const int32_t* lut;    // optional activation table
  int64_t lut_offset, lut_len;
  const uint8_t* res;    // optional residual operand (NHWC bytes, channel 0)
  int64_t res_pix_stride;
  int32_t res_signed;
  int64_t za, ma, sa, zb, mb, sb, sign, add_zo, add_qmin, add_qmax;
  uint8_t* out;          // primary output (NHWC bytes, channel 0), may be null
  int64_t out_pix_stride;
  uint8_t* out2;         // optional rescaled copy (NHWC bytes, channel 0)
  int64_t out2_pix_stride;
  int32_t r_identity;    // copy (after clamping to r_qmin..r_qmax) instead of rescale
  int64_t r_zp_in, r_m, r_s, r_zp_out, r_qmin, r_qmax;
  // 16-bit layers: bytes from each low plane (res, out, out2) to its high
  // plane (v = lo + 256 * (int8)hi); unused by the 8-bit epilogue
  int64_t res_plane, out_plane, out2_plane;
  const int16_t* lut16;  // 16-bit layers: the table as int16 (shared-memory copy)
};

// ABI routes (host-pointer entry points, operands already on the device).
// Narrow int16 GEMM / conv with int32 results, bit-identical to the CPU
// library including its modulo-2^32 wrap; fall back to the CUDA-core
// kernels for shapes the tiles do not cover.
bool umma_gemm_i16_i32_abi(const int16_t* A, const int16_t* B, int32_t* C, int64_t M, int64_t N,
                           int64_t K, cudaStream_t st);
bool umma_conv_i16_i32_abi(const int32_t* x, const int16_t* w, int32_t* y, const ConvGeom& g,
                           cudaStream_t st);

}  // namespace qa
