// Device-resident Vision Transformer layers on 16-bit activations (int16
// graphs, the reference's accurate ViT route): the token embedding, the
// class-token Gather, LayerNorm, the attention core and the final
// dequantize, on int16 tensors held as two byte planes (low plane v & 0xFF,
// high plane v >> 8, `plane` bytes apart; every pointer names the low plane).
// The weighted layers run on the byte-split tensor-core kernel of the
// 16-bit executor.
//
// The float fallbacks follow the reference (quant_layers.py:195-205):
// dequantize to float32, the float op in float64 (float_ops.py LayerNorm,
// Softmax) or float32 (MatMul), quantize with the double-precision
// definition.  The attention products are exact integer sums here, so the
// only difference from the reference is the rounding of its float32 sums:
// within one output step.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/qa_kernels.h"
#include "qa_common.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_ptx.cuh"

namespace qa {
namespace {

__device__ __forceinline__ int32_t load16(const uint8_t* p, int64_t plane) {
  return (int32_t)p[0] | ((int32_t)(int8_t)p[plane] << 8);
}

__device__ __forceinline__ void store16(uint8_t* p, int64_t plane, int32_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[plane] = (uint8_t)((v >> 8) & 0xFF);
}

__device__ __forceinline__ float dequant16(int32_t q, int64_t zp, double scale) {
  return (float)((double)((int64_t)q - zp) * scale);
}

// clamp(rint((double)y / scale) + zp, qmin, qmax): the reference's quantize
__device__ __forceinline__ int32_t quantize16(double y, double scale, int64_t zp, int64_t qmin,
                                              int64_t qmax) {
  double v = rint(y / scale) + (double)zp;
  if (v < (double)qmin) v = (double)qmin;
  if ((double)qmax < v) v = (double)qmax;
  return (int32_t)v;
}

// ------------------------------------------------------ token embedding --
// out[n, 0, :] = cls_row; out[n, t, d] = clamp(ta[x[n, t-1, d] + 32768] +
// pos[t, d]) for t >= 1: the 8-bit embedding's exact integer tables over
// the 65536 int16 values.
__global__ void vit_embed16_kernel(const uint8_t* __restrict__ x, int64_t x_plane,
                                   int64_t x_stride, const int32_t* __restrict__ ta,
                                   const int32_t* __restrict__ pos,
                                   const int32_t* __restrict__ cls_row, int64_t qmin, int64_t qmax,
                                   uint8_t* __restrict__ out, int64_t out_plane,
                                   int64_t out_stride, int64_t B, int64_t T, int64_t D) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = B * T * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / D, d = i - row * D;
    const int64_t n = row / T, t = row - n * T;
    int32_t v;
    if (t == 0) {
      v = cls_row[d];
    } else {
      const int32_t a = load16(x + (n * (T - 1) + t - 1) * x_stride + d, x_plane);
      int64_t s = (int64_t)ta[a + 32768] + pos[t * D + d];
      v = (int32_t)(s < qmin ? qmin : (s > qmax ? qmax : s));
    }
    store16(out + row * out_stride + d, out_plane, v);
  }
}

// ------------------------------------------------------------ LayerNorm --
// One warp per row: float64 mean and variance of the dequantized row (the
// float64 sum of float32 values spanning fewer than 53 bits is exact in any
// order, so the mean is the reference's), (x - mean) / sqrt(var + eps) *
// gamma + beta in float64, rounded to float32, quantized.
__global__ void layernorm16_kernel(const uint8_t* __restrict__ x, int64_t x_plane,
                                   int64_t x_stride, int64_t zp_in, double s_in,
                                   const float* __restrict__ gamma, const float* __restrict__ beta,
                                   double eps, double s_out, int64_t zp_out, int64_t qmin,
                                   int64_t qmax, uint8_t* __restrict__ out, int64_t out_plane,
                                   int64_t out_stride, int64_t rows, int D) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const uint8_t* xr = x + r * x_stride;
    double sum = 0.0;
    for (int d = lane; d < D; d += 32) sum += (double)dequant16(load16(xr + d, x_plane), zp_in, s_in);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const double mean = sum / D;
    double sq = 0.0;
    for (int d = lane; d < D; d += 32) {
      const double c = (double)dequant16(load16(xr + d, x_plane), zp_in, s_in) - mean;
      sq += c * c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const double dev = sqrt(sq / D + eps);
    uint8_t* orow = out + r * out_stride;
    for (int d = lane; d < D; d += 32) {
      double y = ((double)dequant16(load16(xr + d, x_plane), zp_in, s_in) - mean) / dev;
      y = y * (double)gamma[d];
      if (beta) y = y + (double)beta[d];
      store16(orow + d, out_plane, quantize16((double)(float)y, s_out, zp_out, qmin, qmax));
    }
  }
}

// ------------------------------------------------------- attention core --
// One CTA per (image, head), one warp per query row at a time.  Scores
// S = q . k (exact int64 sum of the centred values) quantized on the scores
// grid, the scale Mul as the reference's integer op (exact mbqm of the
// centred product with the constant), Softmax over the dequantized row in
// float64, P quantized, O = P . v (exact int64) quantized on the output grid
// into the head-merged layout.
struct Attn16Params {
  const uint8_t* qkv;
  int64_t qkv_plane, qkv_stride, z_qkv;
  double s_qkv;
  int32_t T, H, hd;
  // scores, Mul output, softmax output, attention output grids
  double s_S, s_M, s_P, s_O;
  int64_t z_S, qmin_S, qmax_S;
  int64_t z_M, qmin_M, qmax_M;
  int64_t z_P, qmin_P, qmax_P;
  int64_t z_O, qmin_O, qmax_O;
  // the Mul: mbqm((S - zS_in) * (c - zc), mult, shift) + z_M
  int64_t mul_c, mul_zc, mul_zs, mul_mult, mul_shift;
  uint8_t* out;
  int64_t out_plane, out_stride;
};

constexpr int kA16Warps = 8;

__global__ void __launch_bounds__(kA16Warps * 32) attention16_kernel(const Attn16Params p) {
  extern __shared__ int32_t a16_smem[];
  const int T = p.T, hd = p.hd, D = p.H * hd;
  int16_t* s_k = reinterpret_cast<int16_t*>(a16_smem);  // [T][hd] raw values
  int16_t* s_v = s_k + T * hd;                          // [T][hd]
  double* s_row = reinterpret_cast<double*>(
      (reinterpret_cast<uintptr_t>(s_v + T * hd) + 7) & ~uintptr_t(7));  // [warps][T]
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int n = blockIdx.x / p.H, h = blockIdx.x - (blockIdx.x / p.H) * p.H;
  const uint8_t* base = p.qkv + (int64_t)n * T * p.qkv_stride;
  for (int i = threadIdx.x; i < T * hd; i += blockDim.x) {
    const int t = i / hd, d = i - t * hd;
    const uint8_t* row = base + (int64_t)t * p.qkv_stride;
    s_k[i] = (int16_t)load16(row + D + h * hd + d, p.qkv_plane);
    s_v[i] = (int16_t)load16(row + 2 * D + h * hd + d, p.qkv_plane);
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  double* srow = s_row + warp * T;
  const int64_t zq = p.z_qkv;
  for (int qi = warp; qi < T; qi += kA16Warps) {
    const uint8_t* qrow = base + (int64_t)qi * p.qkv_stride + h * hd;
    // (1) scores -> Mul -> dequantized softmax input, per key
    float xmax = -INFINITY;
    for (int t = lane; t < T; t += 32) {
      int64_t acc = 0;
      for (int d = 0; d < hd; ++d)
        acc += ((int64_t)load16(qrow + d, p.qkv_plane) - zq) * ((int64_t)s_k[t * hd + d] - zq);
      const int32_t sq = quantize16((double)(float)((double)acc * p.s_qkv * p.s_qkv), p.s_S,
                                    p.z_S, p.qmin_S, p.qmax_S);
      const int64_t mq = requant_exact(((int64_t)sq - p.mul_zs) * (p.mul_c - p.mul_zc),
                                       p.mul_mult, p.mul_shift, p.z_M, p.qmin_M, p.qmax_M);
      const float xv = dequant16((int32_t)mq, p.z_M, p.s_M);
      srow[t] = (double)xv;
      xmax = fmaxf(xmax, xv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) xmax = fmaxf(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
    // (2) softmax in float64
    double esum = 0.0;
    for (int t = lane; t < T; t += 32) {
      const double e = exp(srow[t] - (double)xmax);
      srow[t] = e;
      esum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) esum += __shfl_xor_sync(0xffffffffu, esum, o);
    for (int t = lane; t < T; t += 32) {
      const float pv = (float)(srow[t] / esum);
      srow[t] = (double)(quantize16((double)pv, p.s_P, p.z_P, p.qmin_P, p.qmax_P) - p.z_P);
    }
    __syncwarp();
    // (3) O = P . v, exact, quantized into the head-merged row
    uint8_t* orow = p.out + ((int64_t)n * T + qi) * p.out_stride + h * hd;
    for (int d = lane; d < hd; d += 32) {
      int64_t acc = 0;
      for (int t = 0; t < T; ++t) acc += (int64_t)srow[t] * ((int64_t)s_v[t * hd + d] - zq);
      const double y = (double)(float)((double)acc * p.s_P * p.s_qkv);
      store16(orow + d, p.out_plane, quantize16(y, p.s_O, p.z_O, p.qmin_O, p.qmax_O));
    }
    __syncwarp();
  }
}

// out[r, :] = table[x[r * every + first, :] + 32768]
__global__ void gather16_kernel(const uint8_t* __restrict__ x, int64_t x_plane, int64_t x_stride,
                                int64_t every, int64_t first, const int32_t* __restrict__ table,
                                uint8_t* __restrict__ out, int64_t out_plane, int64_t out_stride,
                                int64_t rows, int64_t D) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * D;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / D, d = i - r * D;
    const int32_t v = load16(x + (r * every + first) * x_stride + d, x_plane);
    store16(out + r * out_stride + d, out_plane, table[v + 32768]);
  }
}

__global__ void dequant_rows16_kernel(const uint8_t* __restrict__ x, int64_t x_plane,
                                      int64_t x_stride, int64_t zp, double scale,
                                      int32_t* __restrict__ q_out, float* __restrict__ f_out,
                                      int64_t rows, int64_t C) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * C;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / C, c = i - r * C;
    const int32_t v = load16(x + r * x_stride + c, x_plane);
    if (q_out) q_out[i] = v;
    if (f_out) f_out[i] = dequant16(v, zp, scale);
  }
}

}  // namespace
}  // namespace qa

using namespace qa;

QA_API int qa_vit_embed16_dev(const void* x, int64_t x_plane, int64_t x_stride,
                              const int32_t* ta, const int32_t* pos, const int32_t* cls_row,
                              int64_t qmin, int64_t qmax, void* out, int64_t out_plane,
                              int64_t out_stride, int64_t B, int64_t T, int64_t D, void* stream) {
  clear_error();
  if (!x || !ta || !pos || !cls_row || !out || B < 0 || T < 1 || D <= 0 || x_stride < D ||
      out_stride < D) {
    set_error(kBadArgument, "qa_vit_embed16_dev: bad arguments");
    return last_status();
  }
  if (B == 0) return 0;
  return launch_ex(vit_embed16_kernel, dim3(grid_for(B * T * D, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_plane, x_stride,
                   ta, pos, cls_row, qmin, qmax, static_cast<uint8_t*>(out), out_plane,
                   out_stride, B, T, D)
             ? 0
             : last_status();
}

QA_API int qa_layernorm16_dev(const void* x, int64_t x_plane, int64_t x_stride, int64_t zp_in,
                              double s_in, const float* gamma, const float* beta, double eps,
                              double s_out, int64_t zp_out, int64_t qmin, int64_t qmax, void* out,
                              int64_t out_plane, int64_t out_stride, int64_t rows, int64_t D,
                              void* stream) {
  clear_error();
  if (!x || !gamma || !out || rows < 0 || D <= 0 || D > (1 << 20) || x_stride < D ||
      out_stride < D || !(s_out > 0.0)) {
    set_error(kBadArgument, "qa_layernorm16_dev: bad arguments");
    return last_status();
  }
  if (rows == 0) return 0;
  return launch_ex(layernorm16_kernel, dim3(grid_for(rows * 32, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_plane, x_stride,
                   zp_in, s_in, gamma, beta, eps, s_out, zp_out, qmin, qmax,
                   static_cast<uint8_t*>(out), out_plane, out_stride, rows, (int)D)
             ? 0
             : last_status();
}

QA_API int qa_attention16_dev(const void* qkv, int64_t qkv_plane, int64_t qkv_stride,
                              int64_t z_qkv, double s_qkv, int64_t B, int64_t T, int64_t H,
                              int64_t hd, const double* s_params, const int64_t* z_params,
                              const int64_t* mul_params, void* out, int64_t out_plane,
                              int64_t out_stride, void* stream) {
  clear_error();
  if (!qkv || !s_params || !z_params || !mul_params || !out || B < 0 || T < 1 || H < 1 ||
      hd < 1 || qkv_stride < 3 * H * hd || out_stride < H * hd) {
    set_error(kBadArgument, "qa_attention16_dev: bad arguments");
    return last_status();
  }
  const size_t smem = (size_t)2 * T * hd * sizeof(int16_t) + 8 + (size_t)kA16Warps * T * 8;
  if (smem > 200 * 1024 || B * H > 0x7FFFFFFF) {
    set_error(kUnsupported, "qa_attention16_dev: sequence or head too large");
    return last_status();
  }
  if (B == 0) return 0;
  Attn16Params p;
  p.qkv = static_cast<const uint8_t*>(qkv);
  p.qkv_plane = qkv_plane;
  p.qkv_stride = qkv_stride;
  p.z_qkv = z_qkv;
  p.s_qkv = s_qkv;
  p.T = (int32_t)T;
  p.H = (int32_t)H;
  p.hd = (int32_t)hd;
  p.s_S = s_params[0];
  p.s_M = s_params[1];
  p.s_P = s_params[2];
  p.s_O = s_params[3];
  p.z_S = z_params[0];
  p.qmin_S = z_params[1];
  p.qmax_S = z_params[2];
  p.z_M = z_params[3];
  p.qmin_M = z_params[4];
  p.qmax_M = z_params[5];
  p.z_P = z_params[6];
  p.qmin_P = z_params[7];
  p.qmax_P = z_params[8];
  p.z_O = z_params[9];
  p.qmin_O = z_params[10];
  p.qmax_O = z_params[11];
  p.mul_c = mul_params[0];
  p.mul_zc = mul_params[1];
  p.mul_zs = mul_params[2];
  p.mul_mult = mul_params[3];
  p.mul_shift = mul_params[4];
  p.out = static_cast<uint8_t*>(out);
  p.out_plane = out_plane;
  p.out_stride = out_stride;
  if (smem > 48 * 1024 &&
      cuda_failed(cudaFuncSetAttribute(attention16_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                  "cudaFuncSetAttribute(attention16)"))
    return last_status();
  return launch_ex(attention16_kernel, dim3((unsigned)(B * H)), dim3(kA16Warps * 32), smem,
                   (cudaStream_t)stream, true, p)
             ? 0
             : last_status();
}

QA_API int qa_gather16_dev(const void* x, int64_t x_plane, int64_t x_stride, int64_t every,
                           int64_t first, const int32_t* table, void* out, int64_t out_plane,
                           int64_t out_stride, int64_t rows, int64_t D, void* stream) {
  clear_error();
  if (!x || !table || !out || rows < 0 || D <= 0 || every <= 0 || first < 0 || x_stride < D ||
      out_stride < D) {
    set_error(kBadArgument, "qa_gather16_dev: bad arguments");
    return last_status();
  }
  if (rows == 0) return 0;
  return launch_ex(gather16_kernel, dim3(grid_for(rows * D, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_plane, x_stride,
                   every, first, table, static_cast<uint8_t*>(out), out_plane, out_stride, rows, D)
             ? 0
             : last_status();
}

QA_API int qa_dequantize_rows16_dev(const void* x, int64_t x_plane, int64_t x_stride, int64_t zp,
                                    double scale, int32_t* q_out, float* f_out, int64_t rows,
                                    int64_t C, void* stream) {
  clear_error();
  if (!x || (!q_out && !f_out) || rows < 0 || C <= 0 || x_stride < C) {
    set_error(kBadArgument, "qa_dequantize_rows16_dev: bad arguments");
    return last_status();
  }
  if (rows == 0) return 0;
  return launch_ex(dequant_rows16_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_plane, x_stride,
                   zp, scale, q_out, f_out, rows, C)
             ? 0
             : last_status();
}
