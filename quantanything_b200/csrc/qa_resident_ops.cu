// Kernels of the device-resident executor other than the tensor-core
// contraction: graph-input quantization into NHWC bytes, grouped /
// depthwise convolution with the fused epilogue, GlobalAveragePool,
// the Softmax float fallback, and byte-tensor versions of the scale
// matching element-wise layers (LUT, Add, Concat rescale, MaxPool) for
// layers the fusion planner leaves standalone.
//
// Activations are NHWC byte tensors: pixel p (row of the [pixels, C] view)
// at base + p * pix_stride, channel c at + c; int8 or uint8 by a flag.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/qa_kernels.h"
#include "qa_common.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_fused_epilogue.cuh"
#include "qa_ptx.cuh"
#include "qa_umma.cuh"

namespace qa {

__device__ __forceinline__ int64_t bval(const uint8_t* p, int is_signed) {
  return is_signed ? (int64_t)(int8_t)*p : (int64_t)*p;
}

// ------------------------------------------------------- fused epilogue --
bool fill_fused_epilogue(FusedEpilogue& e, const qa_fused_conv_desc& d) {
  e.bias = d.bias;
  e.mult = d.mult;
  e.shift = d.shift;
  e.zp = d.zp;
  e.qmin = d.qmin;
  e.qmax = d.qmax;
  e.fast = d.fast ? 1 : 0;
  e.lut = d.lut;
  e.lut_offset = d.lut_offset;
  e.lut_len = d.lut_len;
  e.res = static_cast<const uint8_t*>(d.res);
  e.res_pix_stride = d.res_pix_stride;
  e.res_signed = d.res_signed ? 1 : 0;
  e.za = d.za;
  e.ma = d.ma;
  e.sa = d.sa;
  e.zb = d.zb;
  e.mb = d.mb;
  e.sb = d.sb;
  e.sign = d.sign;
  e.add_zo = d.add_zo;
  e.add_qmin = d.add_qmin;
  e.add_qmax = d.add_qmax;
  e.out = static_cast<uint8_t*>(d.out);
  e.out_pix_stride = d.out_pix_stride;
  e.out2 = static_cast<uint8_t*>(d.out2);
  e.out2_pix_stride = d.out2_pix_stride;
  e.r_identity = d.r_identity ? 1 : 0;
  e.r_zp_in = d.r_zp_in;
  e.r_m = d.r_m;
  e.r_s = d.r_s;
  e.r_zp_out = d.r_zp_out;
  e.r_qmin = d.r_qmin;
  e.r_qmax = d.r_qmax;
  return true;
}

// -------------------------------------------- grouped / depthwise conv ---
struct GroupedConvParams {
  const uint8_t* x;
  int64_t x_pix_stride;
  int32_t x_signed;
  int64_t x_zp;
  int64_t H, W, Cg, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW, Cout, Cog;
  const int8_t* w;
  int64_t w_kp;
  int64_t M;
  FusedEpilogue epi;
};

// One thread per (pixel, output channel); channel fastest so a warp reads
// shared input bytes and writes a contiguous output run.
__global__ void grouped_conv_kernel(const __grid_constant__ GroupedConvParams p) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = p.M * p.Cout;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t n = i % p.Cout, m = i / p.Cout;
    const int64_t ohw = p.OH * p.OW;
    const int64_t img = m / ohw, rem = m - img * ohw;
    const int64_t oy = rem / p.OW, ox = rem - oy * p.OW;
    const int64_t g = n / p.Cog;
    const uint8_t* xb = p.x + img * p.H * p.W * p.x_pix_stride + g * p.Cg;
    const int8_t* wb = p.w + n * p.w_kp;
    int64_t acc = 0;
    for (int64_t ky = 0; ky < p.KH; ++ky) {
      const int64_t iy = oy * p.SH - p.PH + ky * p.DH;
      for (int64_t kx = 0; kx < p.KW; ++kx) {
        const int64_t ix = ox * p.SW - p.PW + kx * p.DW;
        const int8_t* wt = wb + (ky * p.KW + kx) * p.Cg;
        if (iy < 0 || iy >= p.H || ix < 0 || ix >= p.W) {
          // outside the image: the raw zero point (centred value 0)
          int64_t ws = 0;
          for (int64_t c = 0; c < p.Cg; ++c) ws += wt[c];
          acc += ws * p.x_zp;
          continue;
        }
        const uint8_t* xp = xb + (iy * p.W + ix) * p.x_pix_stride;
        for (int64_t c = 0; c < p.Cg; ++c) acc += bval(xp + c, p.x_signed) * (int64_t)wt[c];
      }
    }
    fused_epilogue_store(p.epi, acc, m, (int)n);
  }
}

bool fused_conv_grouped(const qa_fused_conv_desc& d, cudaStream_t st) {
  if (d.Cout % d.groups) {
    set_error(kBadArgument, "qa_conv_fused_dev: Cout not divisible by groups");
    return false;
  }
  GroupedConvParams p;
  p.x = static_cast<const uint8_t*>(d.x);
  p.x_pix_stride = d.x_pix_stride;
  p.x_signed = d.x_signed ? 1 : 0;
  p.x_zp = d.x_zp;
  p.H = d.H;
  p.W = d.W;
  p.Cg = d.C;
  p.KH = d.KH;
  p.KW = d.KW;
  p.SH = d.SH;
  p.SW = d.SW;
  p.PH = d.PH;
  p.PW = d.PW;
  p.DH = d.DH;
  p.DW = d.DW;
  p.OH = d.OH;
  p.OW = d.OW;
  p.Cout = d.Cout;
  p.Cog = d.Cout / d.groups;
  p.w = static_cast<const int8_t*>(d.w);
  p.w_kp = d.w_kp;
  p.M = d.N * d.OH * d.OW;
  fill_fused_epilogue(p.epi, d);
  const int64_t total = p.M * p.Cout;
  if (total == 0) return true;
  return launch_ex(grouped_conv_kernel, dim3(grid_for(total, 256)), dim3(256), 0, st, true, p);
}

// -------------------------------------------- graph input quantization ---
// float NCHW -> bytes NHWC with pix_stride channels per pixel; channels
// C..pix_stride-1 (padding for the tensor-core K granularity) hold zp.
__global__ void quantize_to_nhwc_kernel(const float* __restrict__ x, uint8_t* __restrict__ y,
                                        int64_t N, int64_t C, int64_t HW, int64_t pix_stride,
                                        double scale, double zp, double qmin, double qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * HW;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t n = i / HW, p = i - n * HW;
    uint8_t* dst = y + i * pix_stride;
    for (int64_t c = 0; c < pix_stride; ++c) {
      double v;
      if (c < C) {
        v = rint((double)x[(n * C + c) * HW + p] / scale) + zp;
        if (v < qmin) v = qmin;
        if (qmax < v) v = qmax;
      } else {
        v = zp;
      }
      dst[c] = (uint8_t)(int64_t)v;
    }
  }
}

// Four consecutive pixels per thread for the common 3-channel image stored
// with a 4-byte pixel stride: one 16-byte load per channel plane, one
// 16-byte store of four packed pixels.
__device__ __forceinline__ uint32_t quantize_byte(float xv, double scale, double zp,
                                                  double qmin, double qmax) {
  double v = rint((double)xv / scale) + zp;
  if (v < qmin) v = qmin;
  if (qmax < v) v = qmax;
  return (uint32_t)(int32_t)v & 0xFFu;
}

__global__ void quantize_to_nhwc4_kernel(const float* __restrict__ x, uint8_t* __restrict__ y,
                                         int C, int quads_per_image, int quads, double scale,
                                         double zp, double qmin, double qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const uint32_t pad = (uint32_t)(int32_t)zp & 0xFFu;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += gridDim.x * blockDim.x) {
    const int n = i / quads_per_image, q = i - n * quads_per_image;
    uint32_t px[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c < C) {
        const float4 v = *reinterpret_cast<const float4*>(
            x + ((int64_t)n * C + c) * quads_per_image * 4 + (int64_t)q * 4);
        px[0] |= quantize_byte(v.x, scale, zp, qmin, qmax) << (8 * c);
        px[1] |= quantize_byte(v.y, scale, zp, qmin, qmax) << (8 * c);
        px[2] |= quantize_byte(v.z, scale, zp, qmin, qmax) << (8 * c);
        px[3] |= quantize_byte(v.w, scale, zp, qmin, qmax) << (8 * c);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) px[k] |= pad << (8 * c);
      }
    }
    *reinterpret_cast<uint4*>(y + (int64_t)i * 16) = make_uint4(px[0], px[1], px[2], px[3]);
  }
}

// ------------------------------------------------------------------ GAP --
// y[n, c] = clamp(mbqm(sum_p(x[n,p,c]) - HW*zp_in, m, s) + zp_out)
// (quant_layers.py:569-590: int64 sum of centred values, no bias).
__global__ void gap_kernel(const uint8_t* __restrict__ x, int64_t x_pix_stride, int x_signed,
                           int64_t N, int64_t HW, int64_t C, int64_t zp_in, int64_t m,
                           int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax,
                           uint8_t* __restrict__ y, int64_t y_pix_stride) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t n = i / C, c = i - n * C;
    const uint8_t* xb = x + n * HW * x_pix_stride + c;
    int64_t acc = 0;
    for (int64_t p = 0; p < HW; ++p) acc += bval(xb + p * x_pix_stride, x_signed);
    acc -= HW * zp_in;
    y[n * y_pix_stride + c] = (uint8_t)requant_exact(acc, m, s, zp_out, qmin, qmax);
  }
}

// -------------------------------------------------------------- Softmax --
// The reference's float fallback (quant_layers.py:195-205, float_ops.py
// :380-385): dequantize to float32, softmax in float64 with the row max
// subtracted, round to float32, quantize; optionally also the graph output's
// dequantized float32.
constexpr int kSoftmaxThreads = 256;

__device__ __forceinline__ double block_reduce(double v, bool is_max, double* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    const double u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmax(v, u) : v + u;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x / 32) ? sh[lane] : (is_max ? -INFINITY : 0.0);
    for (int o = 16; o > 0; o >>= 1) {
      const double u = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmax(v, u) : v + u;
    }
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  const double r = sh[0];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kSoftmaxThreads)
    softmax_kernel(const uint8_t* __restrict__ x, int64_t x_pix_stride, int x_signed, int64_t C,
                   double in_scale, int64_t in_zp, double out_scale, double out_zp, double qmin,
                   double qmax, int32_t* __restrict__ q_out, float* __restrict__ y_out,
                   double y_scale, int64_t y_zp) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  __shared__ double sh[32];
  const int64_t row = blockIdx.x;
  const uint8_t* xr = x + row * x_pix_stride;
  double mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float xf = (float)((double)(bval(xr + c, x_signed) - in_zp) * in_scale);
    mx = fmax(mx, (double)xf);
  }
  mx = block_reduce(mx, true, sh);
  double sum = 0.0;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float xf = (float)((double)(bval(xr + c, x_signed) - in_zp) * in_scale);
    sum += exp((double)xf - mx);
  }
  sum = block_reduce(sum, false, sh);
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float xf = (float)((double)(bval(xr + c, x_signed) - in_zp) * in_scale);
    const float pr = (float)(exp((double)xf - mx) / sum);
    double v = rint((double)pr / out_scale) + out_zp;
    if (v < qmin) v = qmin;
    if (qmax < v) v = qmax;
    const int32_t q = (int32_t)v;
    if (q_out) q_out[row * C + c] = q;
    if (y_out) y_out[row * C + c] = (float)((double)((int64_t)q - y_zp) * y_scale);
  }
}

// ---------------------------------------------------------- byte layers --
struct ByteView {
  const uint8_t* p;
  int64_t stride;
  int is_signed;
};

__global__ void lut_bytes_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride,
                                 int64_t rows, int64_t C, int64_t offset,
                                 const int32_t* __restrict__ lut, int64_t len) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    int64_t idx = bval(x.p + r * x.stride + c, x.is_signed) - offset;
    idx = idx < 0 ? 0 : (idx >= len ? len - 1 : idx);
    y[r * y_stride + c] = (uint8_t)__ldg(lut + idx);
  }
}

__global__ void add_bytes_kernel(ByteView a, ByteView b, uint8_t* __restrict__ y,
                                 int64_t y_stride, int64_t rows, int64_t C, int64_t za,
                                 int64_t ma, int64_t sa, int64_t zb, int64_t mb, int64_t sb,
                                 int64_t sign, int64_t zo, int64_t qmin, int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const I128 ta = mbqm(bval(a.p + r * a.stride + c, a.is_signed) - za, ma, sa);
    I128 tb = mbqm(bval(b.p + r * b.stride + c, b.is_signed) - zb, mb, sb);
    if (sign < 0) tb = neg_i128(tb);
    y[r * y_stride + c] = (uint8_t)clamp_i128(add_i128_i64(add_i128(ta, tb), zo), qmin, qmax);
  }
}

__global__ void rescale_bytes_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride,
                                     int64_t rows, int64_t C, int identity, int64_t zp_in,
                                     int64_t m, int64_t s, int64_t zp_out, int64_t qmin,
                                     int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const int64_t v = bval(x.p + r * x.stride + c, x.is_signed);
    int64_t q;
    if (identity) {
      q = v < qmin ? qmin : (v > qmax ? qmax : v);
    } else {
      q = requant_exact(v - zp_in, m, s, zp_out, qmin, qmax);
    }
    y[r * y_stride + c] = (uint8_t)q;
  }
}

__global__ void maxpool_bytes_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride,
                                     int64_t N, int64_t H, int64_t W, int64_t C, int64_t KH,
                                     int64_t KW, int64_t SH, int64_t SW, int64_t PH, int64_t PW,
                                     int64_t DH, int64_t DW, int64_t OH, int64_t OW,
                                     int64_t pad_value) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * OH * OW * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t c = i % C, pix = i / C;
    const int64_t ohw = OH * OW;
    const int64_t n = pix / ohw, rem = pix - n * ohw;
    const int64_t oy = rem / OW, ox = rem - oy * OW;
    int64_t best = INT64_MIN;
    for (int64_t ky = 0; ky < KH; ++ky) {
      const int64_t iy = oy * SH - PH + ky * DH;
      for (int64_t kx = 0; kx < KW; ++kx) {
        const int64_t ix = ox * SW - PW + kx * DW;
        const int64_t v = (iy < 0 || iy >= H || ix < 0 || ix >= W)
                              ? pad_value
                              : bval(x.p + ((n * H + iy) * W + ix) * x.stride + c, x.is_signed);
        best = v > best ? v : best;
      }
    }
    y[pix * y_stride + c] = (uint8_t)best;
  }
}

// NHWC bytes [N, HW, C] <-> NCHW int32.
__global__ void bytes_to_i32_kernel(ByteView x, int32_t* __restrict__ y, int64_t N, int64_t HW,
                                    int64_t C) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * C * HW;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t p = i % HW, t = i / HW;
    const int64_t c = t % C, n = t / C;
    y[i] = (int32_t)bval(x.p + (n * HW + p) * x.stride + c, x.is_signed);
  }
}

__global__ void i32_to_bytes_kernel(const int32_t* __restrict__ x, uint8_t* __restrict__ y,
                                    int64_t y_stride, int64_t N, int64_t HW, int64_t C) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * C * HW;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t p = i % HW, t = i / HW;
    const int64_t c = t % C, n = t / C;
    y[(n * HW + p) * y_stride + c] = (uint8_t)x[i];
  }
}


}  // namespace qa

using namespace qa;

QA_API int qa_quantize_to_nhwc_dev(const float* x, void* y, int64_t N, int64_t C, int64_t H,
                                   int64_t W, int64_t pix_stride, double scale, int64_t zp,
                                   int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (pix_stride < C || N < 0 || C <= 0 || scale == 0.0) {
    set_error(kBadArgument, "qa_quantize_to_nhwc_dev: bad arguments");
    return last_status();
  }
  const int64_t n = N * H * W;
  if (n == 0) return 0;
  const int64_t HW = H * W;
  if (pix_stride == 4 && C <= 4 && HW % 4 == 0 && HW * N / 4 < 0x7FFFFFFF &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const int64_t quads = N * HW / 4;
    return launch_ex(quantize_to_nhwc4_kernel, dim3(grid_for(quads, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), (int)C,
                     (int)(HW / 4), (int)quads, scale, (double)zp, (double)qmin, (double)qmax)
               ? 0
               : last_status();
  }
  return launch_ex(quantize_to_nhwc_kernel, dim3(grid_for(n, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), N, C, HW,
                   pix_stride, scale, (double)zp, (double)qmin, (double)qmax)
             ? 0
             : last_status();
}

QA_API int qa_gap_dev(const void* x, int64_t x_pix_stride, int64_t x_signed, int64_t N,
                      int64_t HW, int64_t C, int64_t zp_in, int64_t mult, int64_t shift,
                      int64_t zp_out, int64_t qmin, int64_t qmax, void* y, int64_t y_pix_stride,
                      void* stream) {
  clear_error();
  if (N * C == 0) return 0;
  return launch_ex(gap_kernel, dim3(grid_for(N * C, 256)), dim3(256), 0, (cudaStream_t)stream,
                   true, static_cast<const uint8_t*>(x), x_pix_stride, (int)x_signed, N, HW, C,
                   zp_in, mult, shift, zp_out, qmin, qmax, static_cast<uint8_t*>(y), y_pix_stride)
             ? 0
             : last_status();
}

QA_API int qa_softmax_dev(const void* x, int64_t x_pix_stride, int64_t x_signed, int64_t N,
                          int64_t C, double in_scale, int64_t in_zp, double out_scale,
                          int64_t out_zp, int64_t qmin, int64_t qmax, int32_t* q_out,
                          float* y_out, double y_scale, int64_t y_zp, void* stream) {
  clear_error();
  if (N == 0 || C == 0) return 0;
  if (N > 0x7FFFFFFF) {
    set_error(kBadArgument, "qa_softmax_dev: too many rows");
    return last_status();
  }
  return launch_ex(softmax_kernel, dim3((unsigned)N), dim3(kSoftmaxThreads), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_pix_stride,
                   (int)x_signed, C, in_scale, in_zp, out_scale, (double)out_zp, (double)qmin,
                   (double)qmax, q_out, y_out, y_scale, y_zp)
             ? 0
             : last_status();
}

QA_API int qa_lut_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                            int64_t y_stride, int64_t rows, int64_t C, int64_t offset,
                            const int32_t* lut, int64_t lut_len, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  return launch_ex(lut_bytes_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0, (cudaStream_t)stream, true,
      ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
      static_cast<uint8_t*>(y), y_stride, rows, C, offset, lut, lut_len)
             ? 0
             : last_status();
}

QA_API int qa_add_bytes_dev(const void* a, int64_t a_stride, int64_t a_signed, const void* b,
                            int64_t b_stride, int64_t b_signed, void* y, int64_t y_stride,
                            int64_t rows, int64_t C, int64_t za, int64_t ma, int64_t sa,
                            int64_t zb, int64_t mb, int64_t sb, int64_t sign, int64_t zo,
                            int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  return launch_ex(add_bytes_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0, (cudaStream_t)stream, true,
      ByteView{static_cast<const uint8_t*>(a), a_stride, (int)a_signed},
      ByteView{static_cast<const uint8_t*>(b), b_stride, (int)b_signed},
      static_cast<uint8_t*>(y), y_stride, rows, C, za, ma, sa, zb, mb, sb, sign, zo, qmin, qmax)
             ? 0
             : last_status();
}

QA_API int qa_rescale_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                                int64_t y_stride, int64_t rows, int64_t C, int64_t identity,
                                int64_t zp_in, int64_t m, int64_t s, int64_t zp_out,
                                int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  return launch_ex(rescale_bytes_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0, (cudaStream_t)stream, true,
      ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
      static_cast<uint8_t*>(y), y_stride, rows, C, (int)identity, zp_in, m, s, zp_out, qmin,
      qmax)
             ? 0
             : last_status();
}

QA_API int qa_maxpool_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                                int64_t y_stride, int64_t N, int64_t H, int64_t W, int64_t C,
                                int64_t KH, int64_t KW, int64_t SH, int64_t SW, int64_t PH,
                                int64_t PW, int64_t DH, int64_t DW, int64_t OH, int64_t OW,
                                int64_t pad_value, void* stream) {
  clear_error();
  const int64_t total = N * OH * OW * C;
  if (total == 0) return 0;
  return launch_ex(maxpool_bytes_kernel, dim3(grid_for(total, 256)), dim3(256), 0, (cudaStream_t)stream, true,
      ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
      static_cast<uint8_t*>(y), y_stride, N, H, W, C, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW,
      pad_value)
             ? 0
             : last_status();
}

QA_API int qa_bytes_to_i32_dev(const void* x, int64_t x_stride, int64_t x_signed, int32_t* y,
                               int64_t N, int64_t HW, int64_t C, void* stream) {
  clear_error();
  if (N * HW * C == 0) return 0;
  return launch_ex(bytes_to_i32_kernel, dim3(grid_for(N * HW * C, 256)), dim3(256), 0, (cudaStream_t)stream, true,
      ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed}, y, N, HW, C)
             ? 0
             : last_status();
}

QA_API int qa_i32_to_bytes_dev(const int32_t* x, void* y, int64_t y_stride, int64_t N,
                               int64_t HW, int64_t C, void* stream) {
  clear_error();
  if (N * HW * C == 0) return 0;
  return launch_ex(i32_to_bytes_kernel, dim3(grid_for(N * HW * C, 256)), dim3(256), 0, (cudaStream_t)stream, true,
      x, static_cast<uint8_t*>(y), y_stride, N, HW, C)
             ? 0
             : last_status();
}

QA_API int qa_device_status_dev(void* stream) {
  clear_error();
  return check_device_status((cudaStream_t)stream) ? 0 : last_status();
}

// ================================================ fused input convolution ==
// Graph input (float32 NCHW, at most 4 channels) -> quantize -> conv ->
// layer epilogue, in one CUDA-core kernel.  A block owns an 8 x 32 tile of
// output pixels and all output channels: it quantizes the input patch the
// tile reads (same rounding as qa_quantize_f32) into shared memory as one
// 4-channel word per pixel, then each thread accumulates its pixel's
// channels with dp4a over the KH x KW taps and runs the fused epilogue.
// Out-of-image taps hold the raw input zero point (the packed bias already
// carries -zp * sum(w)), exactly like the tensor-core path.
namespace qa {

constexpr int kInTileH = 8, kInTileW = 32, kInThreads = kInTileH * kInTileW;
constexpr int kInMaxCout = 64;

struct InputConvParams {
  const float* x;
  int32_t N, C, H, W, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW, Cout;
  int32_t patch_h, patch_w;  // input pixels a tile reads
  int32_t vec4;              // W % 4 == 0 and 16-byte aligned planes: float4 loads
  double scale, zp, qmin, qmax;
  const int8_t* w;  // [Cout][KH*KW*4] rows of w_kp bytes
  int64_t w_kp;
  int32_t fast;
  FusedEpilogue epi;
};

__global__ void __launch_bounds__(kInThreads)
    input_conv_kernel(const __grid_constant__ InputConvParams p) {
  extern __shared__ uint32_t in_smem[];
  uint32_t* s_patch = in_smem;                          // patch_h * patch_w words
  uint32_t* s_w = s_patch + p.patch_h * p.patch_w;      // Cout * KH * KW words
  const int tiles_x = (p.OW + kInTileW - 1) / kInTileW;
  const int tiles_y = (p.OH + kInTileH - 1) / kInTileH;
  const int img = blockIdx.x / (tiles_x * tiles_y);
  const int t = blockIdx.x - img * tiles_x * tiles_y;
  const int oy0 = (t / tiles_x) * kInTileH, ox0 = (t % tiles_x) * kInTileW;
  const int iy0 = oy0 * p.SH - p.PH, ix0 = ox0 * p.SW - p.PW;
  const int taps = p.KH * p.KW;
  // weights are static: stage them before waiting for the previous kernel
  for (int i = threadIdx.x; i < p.Cout * taps; i += kInThreads) {
    const int co = i / taps, tap = i - co * taps;
    s_w[i] = *reinterpret_cast<const uint32_t*>(p.w + co * p.w_kp + tap * 4);
  }
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const uint32_t zpb = (uint32_t)(int32_t)p.zp & 0xFFu;
  const uint32_t zp_word = zpb * 0x01010101u;
  const int plane = p.H * p.W;
  const float* img_base = p.x + (int64_t)img * p.C * plane;
  if (p.vec4) {
    // Groups of 4 image columns aligned to absolute x % 4 == 0: with W % 4 == 0
    // a group is wholly inside or wholly outside the image, and each channel
    // of a group is one aligned 16-byte load (all issued before any math).
    const int xa = ix0 & ~3;                    // first group's absolute x
    const int shift = ix0 - xa;                 // patch column 0 inside group 0
    const int groups = (shift + p.patch_w + 3) >> 2;
    for (int i = threadIdx.x; i < p.patch_h * groups; i += kInThreads) {
      const int py = i / groups, gx = i - py * groups;
      const int iy = iy0 + py, x0 = xa + 4 * gx;
      uint32_t w4[4] = {zp_word, zp_word, zp_word, zp_word};
      if (iy >= 0 && iy < p.H && x0 >= 0 && x0 < p.W) {
        float4 v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (c < p.C)
            v[c] = *reinterpret_cast<const float4*>(img_base + (int64_t)c * plane + iy * p.W + x0);
#pragma unroll
        for (int k = 0; k < 4; ++k) w4[k] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c < p.C) {
            w4[0] |= quantize_byte(v[c].x, p.scale, p.zp, p.qmin, p.qmax) << (8 * c);
            w4[1] |= quantize_byte(v[c].y, p.scale, p.zp, p.qmin, p.qmax) << (8 * c);
            w4[2] |= quantize_byte(v[c].z, p.scale, p.zp, p.qmin, p.qmax) << (8 * c);
            w4[3] |= quantize_byte(v[c].w, p.scale, p.zp, p.qmin, p.qmax) << (8 * c);
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) w4[k] |= zpb << (8 * c);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int px = 4 * gx + k - shift;  // patch column of this pixel
        if (px >= 0 && px < p.patch_w) s_patch[py * p.patch_w + px] = w4[k];
      }
    }
  } else {
    for (int i = threadIdx.x; i < p.patch_h * p.patch_w; i += kInThreads) {
      const int py = i / p.patch_w, px = i - py * p.patch_w;
      const int iy = iy0 + py, ix = ix0 + px;
      uint32_t word = zp_word;
      if (iy >= 0 && iy < p.H && ix >= 0 && ix < p.W) {
        word = 0;
        const float* src = img_base + iy * p.W + ix;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          word |= (c < p.C ? quantize_byte(src[(int64_t)c * plane], p.scale, p.zp, p.qmin,
                                           p.qmax)
                           : zpb) << (8 * c);
      }
      s_patch[i] = word;
    }
  }
  __syncthreads();
  const int oy = oy0 + threadIdx.x / kInTileW, ox = ox0 + threadIdx.x % kInTileW;
  if (oy >= p.OH || ox >= p.OW) return;
  const int64_t m = ((int64_t)img * p.OH + oy) * p.OW + ox;
  const int ly = (oy - oy0) * p.SH, lx = (ox - ox0) * p.SW;
  const FusedEpilogue& e = p.epi;
  for (int c0 = 0; c0 < p.Cout; c0 += 16) {
    int32_t acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0;
    for (int ky = 0; ky < p.KH; ++ky)
      for (int kx = 0; kx < p.KW; ++kx) {
        const int word = (int)s_patch[(ly + ky * p.DH) * p.patch_w + lx + kx * p.DW];
        const int tap = ky * p.KW + kx;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < p.Cout) acc[j] = __dp4a(word, (int)s_w[(c0 + j) * taps + tap], acc[j]);
      }
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = c0 + j;
      if (n >= p.Cout) continue;
      int64_t q;
      const int64_t x = (int64_t)acc[j] + (e.bias ? e.bias[n] : 0);
      if (p.fast) {
        const int ts = (int)(31 + e.shift[n]);
        q = ((x * e.mult[n] + ((int64_t)1 << (ts - 1))) >> ts) + e.zp;
        q = q < e.qmin ? e.qmin : (q > e.qmax ? e.qmax : q);
      } else {
        q = requant_exact(x, e.mult[n], e.shift[n], e.zp, e.qmin, e.qmax);
      }
      if (e.lut) {
        int64_t idx = q - e.lut_offset;
        idx = idx < 0 ? 0 : (idx >= e.lut_len ? e.lut_len - 1 : idx);
        q = __ldg(e.lut + idx);
      }
      o[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
    }
    uint8_t* op = e.out + m * e.out_pix_stride + c0;
    if (c0 + 16 <= p.Cout && (e.out_pix_stride % 16) == 0 &&
        (reinterpret_cast<uintptr_t>(e.out) & 15) == 0) {
      *reinterpret_cast<uint4*>(op) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c0 + j < p.Cout) op[j] = (uint8_t)(o[j >> 2] >> (8 * (j & 3)));
    }
  }
}

}  // namespace qa

QA_API int qa_conv_input_fused_dev(const qa_fused_conv_desc* d, const float* x, int64_t c_in,
                                   double scale, int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (!d || !x || d->C != 4 || c_in < 1 || c_in > 4 || d->groups != 1 || !d->x_signed ||
      d->Cout > kInMaxCout || d->w_kp < d->KH * d->KW * 4 || !d->out || d->res || d->out2 ||
      !d->mult || !d->shift || scale == 0.0) {
    set_error(kBadArgument, "qa_conv_input_fused_dev: unsupported layer");
    return last_status();
  }
  InputConvParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = x;
  p.N = (int32_t)d->N;
  p.C = (int32_t)c_in;  // channels of the float tensor (taps are packed 4 wide)
  p.H = (int32_t)d->H;
  p.W = (int32_t)d->W;
  p.KH = (int32_t)d->KH;
  p.KW = (int32_t)d->KW;
  p.SH = (int32_t)d->SH;
  p.SW = (int32_t)d->SW;
  p.PH = (int32_t)d->PH;
  p.PW = (int32_t)d->PW;
  p.DH = (int32_t)d->DH;
  p.DW = (int32_t)d->DW;
  p.OH = (int32_t)d->OH;
  p.OW = (int32_t)d->OW;
  p.Cout = (int32_t)d->Cout;
  p.patch_h = (kInTileH - 1) * p.SH + (p.KH - 1) * p.DH + 1;
  p.patch_w = (kInTileW - 1) * p.SW + (p.KW - 1) * p.DW + 1;
  p.vec4 = (p.W % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  p.scale = scale;
  p.zp = (double)d->x_zp;
  p.qmin = (double)qmin;
  p.qmax = (double)qmax;
  p.w = static_cast<const int8_t*>(d->w);
  p.w_kp = d->w_kp;
  p.fast = d->fast ? 1 : 0;
  fill_fused_epilogue(p.epi, *d);
  const int64_t tiles = d->N * ((d->OH + kInTileH - 1) / kInTileH) *
                        ((d->OW + kInTileW - 1) / kInTileW);
  const size_t smem = ((size_t)p.patch_h * p.patch_w + (size_t)p.Cout * p.KH * p.KW) * 4;
  if (tiles == 0) return 0;
  if (tiles > 0x7FFFFFFF || smem > 48 * 1024) {
    set_error(kUnsupported, "qa_conv_input_fused_dev: layer too large");
    return last_status();
  }
  return launch_ex(input_conv_kernel, dim3((unsigned)tiles), dim3(kInThreads), smem,
                   (cudaStream_t)stream, true, p)
             ? 0
             : last_status();
}
