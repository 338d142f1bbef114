// Kernels of the device-resident executor other than the tensor-core
// contraction: graph-input quantization into NHWC bytes, grouped /
// depthwise convolution with the fused epilogue, GlobalAveragePool,
// the Softmax float fallback, and byte-tensor versions of the scale
// matching element-wise layers (LUT, Add, Concat rescale, MaxPool) for
// layers the fusion planner leaves standalone.
//
// Activations are NHWC byte tensors: pixel p (row of the [pixels, C] view)
// at base + p * pix_stride, channel c at + c; int8 or uint8 by a flag.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/qa_kernels.h"
#include "qa_common.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_fused_epilogue.cuh"
#include "qa_ptx.cuh"
#include "qa_quant.cuh"
#include "qa_umma.cuh"

namespace qa {

bool encode_tiled_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides, const uint32_t* box);

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
  e.res_plane = e.out_plane = e.out2_plane = 0;
  e.lut16 = nullptr;
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
// Output layout: NHWC with 4 bytes per pixel (P == 0), or patch rows
// (P > 0): the P x P pixels of patch (py, px) of image n form row
// (n * H / P + py) * W / P + px of P * P * 4 bytes, pixel (ky, kx) at
// (ky * P + kx) * 4 -- the im2col rows of a P x P, stride-P convolution.
// kC3: the tensor has three channels (an RGB image), known at compile time.
template <bool kC3>
__global__ void __launch_bounds__(256, 4)
    quantize_to_nhwc4_kernel(const float* __restrict__ x, uint8_t* __restrict__ y, int C_,
                             int quads_per_image, int quads, int W, int P, const QuantK k) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int C = kC3 ? 3 : C_;
  const uint32_t pad = (uint32_t)(int32_t)k.zpd & 0xFFu;
  const QuantK kk = k;  // the fast path's constants in registers
  // each warp takes 32 * kQ consecutive quads; lane l the quads l, l + 32,
  // ..., all of their 16-byte loads in flight before any is used (one quad
  // per lane keeps the registers low enough for four blocks per SM)
  constexpr int kQ = 1;
  const int lane = threadIdx.x & 31;
  const int warp0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int w = warp0; w * 32 * kQ < quads; w += nwarps) {
    float4 v[kQ][4];
    int qi[kQ];
#pragma unroll
    for (int u = 0; u < kQ; ++u) {
      qi[u] = w * 32 * kQ + u * 32 + lane;
      const bool ok = qi[u] < quads;
      const int n = ok ? qi[u] / quads_per_image : 0, q = ok ? qi[u] - n * quads_per_image : 0;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        v[u][c] = (ok && c < C) ? *reinterpret_cast<const float4*>(
                                      x + ((int64_t)n * C + c) * quads_per_image * 4 + (int64_t)q * 4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kQ; ++u) {
      if (qi[u] >= quads) break;
      uint32_t bits[4][4];  // [channel][pixel]
      bool ok[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float fv[4] = {v[u][c].x, v[u][c].y, v[u][c].z, v[u][c].w};
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          ok[c][b] = true;
          bits[c][b] = c < C ? quantize_bits_fma(fv[b], kk, ok[c][b]) : pad;
        }
      }
      bool all_ok = true;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int b = 0; b < 4; ++b) all_ok = all_ok & (ok[c][b] || c >= C);
      if (!all_ok) {
        // rare (an element within 2^-13 of a rounding tie, NaN, or no float
        // scale): each such element is decided on its own
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float fv[4] = {v[u][c].x, v[u][c].y, v[u][c].z, v[u][c].w};
#pragma unroll
          for (int b = 0; b < 4; ++b)
            if (c < C && !ok[c][b]) bits[c][b] = quantize_byte_near_tie(fv[b], k);
        }
      }
      uint32_t px[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) px[b] = pack_bytes(bits[0][b], bits[1][b], bits[2][b], bits[3][b]);
      int64_t off = (int64_t)qi[u] * 16;
      if (P > 0) {
        const int n = qi[u] / quads_per_image, p0 = (qi[u] - n * quads_per_image) * 4;
        const int yy = p0 / W, xx = p0 - yy * W;
        const int pr = W / P, pc = quads_per_image * 4 / W / P;  // patches per row / column
        const int64_t row = ((int64_t)n * pc + yy / P) * pr + xx / P;
        off = row * (P * P * 4) + ((yy % P) * P + xx % P) * 4;
      }
      *reinterpret_cast<uint4*>(y + off) = make_uint4(px[0], px[1], px[2], px[3]);
    }
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

// Warp per (image, 16-channel group): lanes take pixels lane, lane + 32, ...
// and 16-byte loads of the group's channels; int32 partial sums (|sum| <=
// HW * 255 < 2^31 for HW < 2^23, host-checked) are reduced by shuffles and
// lane c (c < 16) requantizes channel c (same int64 sum as gap_kernel).
__global__ void gap16ch_kernel(const uint8_t* __restrict__ x, int64_t x_pix_stride, int x_signed,
                               int64_t N, int64_t HW, int64_t C, int64_t zp_in, int64_t m,
                               int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax,
                               uint8_t* __restrict__ y, int64_t y_pix_stride) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t groups = C / 16;
  const int64_t warps = N * groups;
  const int64_t wstride = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < warps;
       w += wstride) {
    const int64_t n = w / groups, g = w - n * groups;
    const uint8_t* base = x + n * HW * x_pix_stride + g * 16;
    int32_t acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0;
    for (int64_t p = lane; p < HW; p += 32) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + p * x_pix_stride));
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t b = (wv[j >> 2] >> (8 * (j & 3))) & 0xFFu;
        acc[j] += x_signed ? (int32_t)(int8_t)b : (int32_t)b;
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    int32_t mine = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) mine = lane == j ? acc[j] : mine;
    if (lane < 16) {
      const int64_t sum = (int64_t)mine - HW * zp_in;
      y[n * y_pix_stride + g * 16 + lane] = (uint8_t)requant_exact(sum, m, s, zp_out, qmin, qmax);
    }
  }
}

// Thread per (image, 16-channel group) for images of at most 256 pixels:
// every pixel's 16-byte load is independent (all in flight), the bytes are
// summed in 16-bit lanes (even and odd bytes of each word separately; a
// signed byte is biased by 128 first, so each lane sums at most 256 * 255),
// and the 64-bit rescale replaces the 128-bit one whenever the host proved
// it exact (`fast`).  Four loads in flight per thread and at most 40
// registers let twelve 128-thread blocks share an SM: DRAM latency is
// covered by resident warps rather than by a long unroll.
__global__ void __launch_bounds__(128, 12) gap16_thread_kernel(const uint8_t* __restrict__ x, int64_t x_pix_stride,
                                    int x_signed, int64_t N, int HW, int64_t groups,
                                    int64_t zp_in, int64_t m, int64_t s, int64_t zp_out,
                                    int64_t qmin, int64_t qmax, int fast, uint8_t* __restrict__ y,
                                    int64_t y_pix_stride) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * groups;
  const uint32_t flip = x_signed ? 0x80808080u : 0u;
  const int ts = (int)(31 + s);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / groups, g = i - n * groups;
    const uint8_t* base = x + n * HW * x_pix_stride + g * 16;
    uint32_t even[4] = {0, 0, 0, 0}, odd[4] = {0, 0, 0, 0};
#pragma unroll 4
    for (int p = 0; p < HW; ++p) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)p * x_pix_stride));
      const uint32_t w[4] = {v.x ^ flip, v.y ^ flip, v.z ^ flip, v.w ^ flip};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        even[k] += w[k] & 0x00FF00FFu;
        odd[k] += (w[k] >> 8) & 0x00FF00FFu;
      }
    }
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t word = (j & 1) ? odd[j >> 2] : even[j >> 2];
      int64_t sum = (int64_t)((word >> (16 * ((j >> 1) & 1))) & 0xFFFFu);
      if (x_signed) sum -= 128 * (int64_t)HW;
      sum -= (int64_t)HW * zp_in;
      int64_t q;
      if (fast) {
        q = ((sum * m + ((int64_t)1 << (ts - 1))) >> ts) + zp_out;
        q = q < qmin ? qmin : (q > qmax ? qmax : q);
      } else {
        q = requant_exact(sum, m, s, zp_out, qmin, qmax);
      }
      o[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
    }
    uint8_t* dst = y + n * y_pix_stride + g * 16;
    if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) dst[j] = (uint8_t)(o[j >> 2] >> (8 * (j & 3)));
    }
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

// ----------------------------------------- 16-channel vector forms ----
// One thread handles 16 channel bytes of one pixel with 16-byte loads and
// stores (C, the pixel strides and the base pointers multiples of 16).  An
// 8-bit operand takes only 256 values, so per-element maps are 256-entry
// tables built per block from the exact definitions.

// byte -> byte map of a standalone table layer or Concat rescale
struct ByteMap {
  int is_signed;
  int kind;                  // 0: activation table, 1: rescale / clip
  const int32_t* lut;
  int64_t offset, len;       // table: out = lut[clamp(v - offset, 0, len - 1)]
  int identity;              // rescale: clip to [qmin, qmax] instead
  int64_t zin, m, s, zout, qmin, qmax;
};

__device__ __forceinline__ uint8_t byte_map_entry(const ByteMap& mp, int b) {
  const int64_t v = mp.is_signed ? (int64_t)(int8_t)b : (int64_t)b;
  if (mp.kind == 0) {
    int64_t idx = v - mp.offset;
    idx = idx < 0 ? 0 : (idx >= mp.len ? mp.len - 1 : idx);
    return (uint8_t)mp.lut[idx];
  }
  if (mp.identity) return (uint8_t)(v < mp.qmin ? mp.qmin : (v > mp.qmax ? mp.qmax : v));
  return (uint8_t)requant_exact(v - mp.zin, mp.m, mp.s, mp.zout, mp.qmin, mp.qmax);
}

__device__ __forceinline__ uint4 map16(const uint8_t* tab, uint4 v) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w}, o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    o[k] = (uint32_t)tab[w[k] & 0xFF] | ((uint32_t)tab[(w[k] >> 8) & 0xFF] << 8) |
           ((uint32_t)tab[(w[k] >> 16) & 0xFF] << 16) | ((uint32_t)tab[w[k] >> 24] << 24);
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void map_bytes16_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride,
                                   int64_t rows, int64_t groups, ByteMap mp) {
  __shared__ uint8_t tab[256];
  ptx::pdl_launch_dependents();
  for (int b = threadIdx.x; b < 256; b += blockDim.x) tab[b] = byte_map_entry(mp, b);
  __syncthreads();
  ptx::pdl_wait();
  const int64_t total = rows * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // two vectors in flight per thread
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 2 * stride) {
    const int64_t i2 = i + stride;
    const int64_t r = i / groups, g = i - r * groups;
    const int64_t r2 = i2 / groups, g2 = i2 - r2 * groups;
    const uint4 v = *reinterpret_cast<const uint4*>(x.p + r * x.stride + g * 16);
    uint4 v2 = make_uint4(0, 0, 0, 0);
    if (i2 < total) v2 = *reinterpret_cast<const uint4*>(x.p + r2 * x.stride + g2 * 16);
    *reinterpret_cast<uint4*>(y + r * y_stride + g * 16) = map16(tab, v);
    if (i2 < total) *reinterpret_cast<uint4*>(y + r2 * y_stride + g2 * 16) = map16(tab, v2);
  }
}

// Sum of the two rescaled terms on 128 bits (the tables' range check failed).
__device__ __noinline__ int64_t add_bytes_exact(int64_t va, int64_t vb, int64_t za, int64_t ma,
                                                int64_t sa, int64_t zb, int64_t mb, int64_t sb,
                                                int64_t sign, int64_t zo, int64_t qmin,
                                                int64_t qmax) {
  const I128 x1 = mbqm(va - za, ma, sa);
  I128 x2 = mbqm(vb - zb, mb, sb);
  if (sign < 0) x2 = neg_i128(x2);
  return clamp_i128(add_i128_i64(add_i128(x1, x2), zo), qmin, qmax);
}

// Grid-stride walk over the 16-byte vectors of two byte views (rows x
// groups), two vectors per operand in flight per thread before `one`
// combines them; 32-bit row division when the vector count allows.
template <typename F>
__device__ __forceinline__ void two_in_flight(const ByteView& a, const ByteView& b,
                                              uint8_t* __restrict__ y, int64_t y_stride,
                                              int64_t total, int64_t groups, F&& one) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool narrow = total < (1ll << 31);
  auto row = [&](int64_t i) {
    return narrow ? (int64_t)((uint32_t)i / (uint32_t)groups) : i / groups;
  };
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 2 * stride) {
    const int64_t i2 = i + stride;
    const int64_t r = row(i), g = i - r * groups;
    const uint4 va = *reinterpret_cast<const uint4*>(a.p + r * a.stride + g * 16);
    const uint4 vb = *reinterpret_cast<const uint4*>(b.p + r * b.stride + g * 16);
    uint4 va2 = make_uint4(0, 0, 0, 0), vb2 = va2;
    int64_t r2 = 0, g2 = 0;
    if (i2 < total) {
      r2 = row(i2);
      g2 = i2 - r2 * groups;
      va2 = *reinterpret_cast<const uint4*>(a.p + r2 * a.stride + g2 * 16);
      vb2 = *reinterpret_cast<const uint4*>(b.p + r2 * b.stride + g2 * 16);
    }
    *reinterpret_cast<uint4*>(y + r * y_stride + g * 16) = one(va, vb);
    if (i2 < total) *reinterpret_cast<uint4*>(y + r2 * y_stride + g2 * 16) = one(va2, vb2);
  }
}

// Add with conflict-free table reads: the two rescaled terms (sign applied
// to the second) as int32 tables with one copy per lane (entry e of lane l
// at word e * 32 + l: a warp's 32 lookups always hit 32 different banks,
// where one shared copy serializes on the random banks of random bytes).
// Used when the host proves every term within 2^29 and the zero point
// within 2^30 (their sum is then exact in int32); 64 KB of shared memory
// per block, persistent grid.
constexpr int kAddRepThreads = 512;

// Four int32 values saturated to 8 bits (int8 or uint8) and packed
// little-endian (cvt.pack.sat: sat(b) | sat(a) << 8 | c << 16).
__device__ __forceinline__ uint32_t pack_sat4_bytes(int32_t a, int32_t b, int32_t c, int32_t d,
                                                    bool is_signed) {
  uint32_t hi, r;
  const uint32_t zero = 0;
  if (is_signed) {
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(d), "r"(c), "r"(zero));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(b), "r"(a), "r"(hi));
  } else {
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(d), "r"(c), "r"(zero));
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(b), "r"(a), "r"(hi));
  }
  return r;
}

__global__ void __launch_bounds__(kAddRepThreads) add_bytes16_rep_kernel(
    ByteView a, ByteView b, uint8_t* __restrict__ y, int64_t y_stride, int64_t rows,
    int64_t groups, int64_t za, int64_t ma, int64_t sa, int64_t zb, int64_t mb, int64_t sb,
    int64_t sign, int64_t zo, int64_t qmin, int64_t qmax) {
  extern __shared__ int32_t add_rep[];  // [2][256][32]
  ptx::pdl_launch_dependents();
  for (int e = threadIdx.x; e < 256; e += blockDim.x) {
    const int64_t va = a.is_signed ? (int64_t)(int8_t)e : (int64_t)e;
    const int64_t vb = b.is_signed ? (int64_t)(int8_t)e : (int64_t)e;
    const I128 x1 = mbqm(va - za, ma, sa);
    I128 x2 = mbqm(vb - zb, mb, sb);
    if (sign < 0) x2 = neg_i128(x2);
    const int32_t t1 = (int32_t)(int64_t)x1.lo, t2 = (int32_t)(int64_t)x2.lo;
#pragma unroll 8
    for (int l = 0; l < 32; ++l) {
      add_rep[e * 32 + l] = t1;
      add_rep[(256 + e) * 32 + l] = t2;
    }
  }
  __syncthreads();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int32_t* ta = add_rep + lane;
  const int32_t* tb = add_rep + 256 * 32 + lane;
  const int32_t zo32 = (int32_t)zo, lo32 = (int32_t)qmin, hi32 = (int32_t)qmax;
  // a full 8-bit output range lets the saturating pack do the clamp
  const bool sat_s8 = qmin == -128 && qmax == 127, sat_u8 = qmin == 0 && qmax == 255;
  if (sat_s8 || sat_u8) {
    auto one = [&](const uint4 va4, const uint4 vb4) {
      const uint32_t wa[4] = {va4.x, va4.y, va4.z, va4.w}, wb[4] = {vb4.x, vb4.y, vb4.z, vb4.w};
      uint32_t o[4];
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        int32_t q[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t ea = (wa[k4] >> (8 * b)) & 0xFFu, eb = (wb[k4] >> (8 * b)) & 0xFFu;
          q[b] = ta[ea * 32] + tb[eb * 32] + zo32;
        }
        o[k4] = pack_sat4_bytes(q[0], q[1], q[2], q[3], sat_s8);
      }
      return make_uint4(o[0], o[1], o[2], o[3]);
    };
    two_in_flight(a, b, y, y_stride, rows * groups, groups, one);
    return;
  }
  auto one = [&](const uint4 va4, const uint4 vb4) {
    const uint32_t wa[4] = {va4.x, va4.y, va4.z, va4.w}, wb[4] = {vb4.x, vb4.y, vb4.z, vb4.w};
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t ea = (wa[j >> 2] >> (8 * (j & 3))) & 0xFFu;
      const uint32_t eb = (wb[j >> 2] >> (8 * (j & 3))) & 0xFFu;
      const int32_t q = min(max(ta[ea * 32] + tb[eb * 32] + zo32, lo32), hi32);
      o[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  };
  two_in_flight(a, b, y, y_stride, rows * groups, groups, one);
}

// Add: the two rescaled terms (sign applied to the second) as int64 tables;
// exact when every entry's 128-bit value lies within +-2^61 (checked while
// building: the sum of two terms and the zero point then cannot overflow),
// else every element takes the 128-bit path.
__global__ void __launch_bounds__(256, 3) add_bytes16_kernel(ByteView a, ByteView b, uint8_t* __restrict__ y,
                                   int64_t y_stride, int64_t rows, int64_t groups, int64_t za,
                                   int64_t ma, int64_t sa, int64_t zb, int64_t mb, int64_t sb,
                                   int64_t sign, int64_t zo, int64_t qmin, int64_t qmax) {
  __shared__ int64_t ta[256], tb[256];
  __shared__ int32_t ta32[256], tb32[256];
  ptx::pdl_launch_dependents();
  int ok = 1, ok32 = 1;
  for (int e = threadIdx.x; e < 256; e += blockDim.x) {
    const int64_t va = a.is_signed ? (int64_t)(int8_t)e : (int64_t)e;
    const int64_t vb = b.is_signed ? (int64_t)(int8_t)e : (int64_t)e;
    const I128 x1 = mbqm(va - za, ma, sa);
    I128 x2 = mbqm(vb - zb, mb, sb);
    if (sign < 0) x2 = neg_i128(x2);
    const int64_t lim = (int64_t)1 << 61;
    ok &= x1.hi == ((int64_t)x1.lo >> 63) && (int64_t)x1.lo > -lim && (int64_t)x1.lo < lim;
    ok &= x2.hi == ((int64_t)x2.lo >> 63) && (int64_t)x2.lo > -lim && (int64_t)x2.lo < lim;
    ta[e] = (int64_t)x1.lo;
    tb[e] = (int64_t)x2.lo;
    const int64_t l29 = (int64_t)1 << 29;
    ok32 &= ta[e] > -l29 && ta[e] < l29 && tb[e] > -l29 && tb[e] < l29;
    ta32[e] = (int32_t)ta[e];
    tb32[e] = (int32_t)tb[e];
  }
  const bool tables = __syncthreads_and(ok);
  // both terms within 2^29 and the zero point within 2^30: the sum is
  // exact in int32
  const bool tables32 = __syncthreads_and(ok32) && zo > -(1 << 30) && zo < (1 << 30) &&
                        qmin > -(1ll << 31) && qmax < (1ll << 31);
  ptx::pdl_wait();
  auto one = [&](const uint4 va4, const uint4 vb4) {
    const uint32_t wa[4] = {va4.x, va4.y, va4.z, va4.w}, wb[4] = {vb4.x, vb4.y, vb4.z, vb4.w};
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int ea = (wa[j >> 2] >> (8 * (j & 3))) & 0xFF;
      const int eb = (wb[j >> 2] >> (8 * (j & 3))) & 0xFF;
      int64_t q;
      if (tables32) {
        int32_t q32 = ta32[ea] + tb32[eb] + (int32_t)zo;
        q32 = q32 < (int32_t)qmin ? (int32_t)qmin : (q32 > (int32_t)qmax ? (int32_t)qmax : q32);
        q = q32;
      } else if (tables) {
        q = ta[ea] + tb[eb] + zo;
        q = q < qmin ? qmin : (q > qmax ? qmax : q);
      } else {
        q = add_bytes_exact(a.is_signed ? (int64_t)(int8_t)ea : ea,
                            b.is_signed ? (int64_t)(int8_t)eb : eb, za, ma, sa, zb, mb, sb, sign,
                            zo, qmin, qmax);
      }
      o[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  };
  two_in_flight(a, b, y, y_stride, rows * groups, groups, one);
}

__global__ void mul_bytes16_kernel(ByteView a, ByteView b, uint8_t* __restrict__ y,
                                   int64_t y_stride, int64_t rows, int64_t groups, int64_t za,
                                   int64_t zb, int64_t m, int64_t s, int64_t zo, int64_t qmin,
                                   int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const bool small = small_applies(m, s);
  // with |za|, |zb| < 2^12 the centred operands lie within +-(2^12 + 255),
  // so |p| < 2^26 fits int32
  const bool small32 = small && za > -(1 << 12) && za < (1 << 12) && zb > -(1 << 12) &&
                       zb < (1 << 12);
  const int ts = (int)(31 + s);
  const int64_t rnd = small ? ((int64_t)1 << (ts - 1)) : 0;
  // 32-bit form: (hi32(p * m) + 2^(ts - 33)) >> (ts - 32) equals the
  // rounded shift for ts in [33, 62] (the low word cannot carry into the
  // rounding bit), with 0 <= m < 2^31 and |p| < 2^31
  const bool hi32 = small32 && ts >= 33 && ts <= 62 && m >= 0 && m < (int64_t(1) << 31) &&
                    zo > -(1 << 20) && zo < (1 << 20);
  if (hi32) {
    const int32_t za32 = (int32_t)za, zb32 = (int32_t)zb, m32 = (int32_t)m;
    const int32_t r32 = 1 << (ts - 33), sh = ts - 32;
    const int32_t zo32 = (int32_t)zo, lo32 = (int32_t)qmin, hi32v = (int32_t)qmax;
    const uint32_t fa = a.is_signed ? 0x80u : 0u, fb = b.is_signed ? 0x80u : 0u;
    auto one32 = [&](const uint4 va4, const uint4 vb4) {
      const uint32_t wa[4] = {va4.x, va4.y, va4.z, va4.w}, wb[4] = {vb4.x, vb4.y, vb4.z, vb4.w};
      uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // a signed byte: (b ^ 0x80) - 0x80
        const int32_t ea = (int32_t)(((wa[j >> 2] >> (8 * (j & 3))) & 0xFFu) ^ fa) - (int32_t)fa;
        const int32_t eb = (int32_t)(((wb[j >> 2] >> (8 * (j & 3))) & 0xFFu) ^ fb) - (int32_t)fb;
        const int32_t p = (ea - za32) * (eb - zb32);
        const int32_t q = min(max(((__mulhi(p, m32) + r32) >> sh) + zo32, lo32), hi32v);
        o[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
      }
      return make_uint4(o[0], o[1], o[2], o[3]);
    };
    two_in_flight(a, b, y, y_stride, rows * groups, groups, one32);
    return;
  }
  auto one = [&](const uint4 va4, const uint4 vb4) {
    const uint32_t wa[4] = {va4.x, va4.y, va4.z, va4.w}, wb[4] = {vb4.x, vb4.y, vb4.z, vb4.w};
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int ea = (wa[j >> 2] >> (8 * (j & 3))) & 0xFF;
      const int eb = (wb[j >> 2] >> (8 * (j & 3))) & 0xFF;
      const int64_t p = ((a.is_signed ? (int64_t)(int8_t)ea : ea) - za) *
                        ((b.is_signed ? (int64_t)(int8_t)eb : eb) - zb);
      int64_t q;
      if (small32) {
        // |p| < 2^31 and |m| < 2^31: one 32 x 32 -> 64-bit product
        const int64_t t = ((int64_t)(int32_t)p * (int64_t)(int32_t)m + rnd) >> ts;
        q = t + zo;
        q = q < qmin ? qmin : (q > qmax ? qmax : q);
      } else if (small) {
        q = mbqm_small(p, m, (int)(31 + s)) + zo;
        q = q < qmin ? qmin : (q > qmax ? qmax : q);
      } else {
        q = requant_exact_cold(p, m, s, zo, qmin, qmax);
      }
      o[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  };
  two_in_flight(a, b, y, y_stride, rows * groups, groups, one);
}

// MaxPool: per-byte SIMD max over the window, out-of-image taps read the
// pad value (qmin) in every byte.
__global__ void maxpool_bytes16_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride,
                                       int64_t N, int64_t H, int64_t W, int64_t groups,
                                       int64_t KH, int64_t KW, int64_t SH, int64_t SW,
                                       int64_t PH, int64_t PW, int64_t DH, int64_t DW,
                                       int64_t OH, int64_t OW, uint32_t pad_word) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * OH * OW * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t g = i % groups, pix = i / groups;
    const int64_t ohw = OH * OW;
    const int64_t n = pix / ohw, rem = pix - n * ohw;
    const int64_t oy = rem / OW, ox = rem - oy * OW;
    uint32_t best[4] = {pad_word, pad_word, pad_word, pad_word};
    bool first = true;
    for (int64_t ky = 0; ky < KH; ++ky) {
      const int64_t iy = oy * SH - PH + ky * DH;
      for (int64_t kx = 0; kx < KW; ++kx) {
        const int64_t ix = ox * SW - PW + kx * DW;
        uint4 v = make_uint4(pad_word, pad_word, pad_word, pad_word);
        if (iy >= 0 && iy < H && ix >= 0 && ix < W)
          v = *reinterpret_cast<const uint4*>(x.p + ((n * H + iy) * W + ix) * x.stride + g * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
          best[k] = first ? w[k] : (x.is_signed ? __vmaxs4(best[k], w[k]) : __vmaxu4(best[k], w[k]));
        first = false;
      }
    }
    *reinterpret_cast<uint4*>(y + pix * y_stride + g * 16) =
        make_uint4(best[0], best[1], best[2], best[3]);
  }
}

// Stride-1 MaxPool (SPPF's k5 s1 p2) tiled and separable: a block stages
// the input rows and columns of an 8 x 32 output tile (plus the window's
// halo, out-of-image taps = the pad value) for one 16-channel group in
// shared memory, takes the maxima along each row, then along each column.
constexpr int kMpTH = 8, kMpTW = 32, kMpMaxK = 7;

__global__ void __launch_bounds__(256)
    maxpool_bytes16_s1_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride, int64_t H,
                              int64_t W, int64_t groups, int KH, int KW, int64_t PH, int64_t PW,
                              int64_t OH, int64_t OW, int64_t tiles_x, int64_t tiles_y,
                              uint32_t pad_word) {
  __shared__ uint4 s_in[kMpTH + kMpMaxK - 1][kMpTW + kMpMaxK - 1];
  __shared__ uint4 s_row[kMpTH + kMpMaxK - 1][kMpTW];
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t t = blockIdx.x;
  const int64_t tx = t % tiles_x, ty = (t / tiles_x) % tiles_y, ng = t / (tiles_x * tiles_y);
  const int64_t n = ng / groups, g = ng - n * groups;
  const int64_t oy0 = ty * kMpTH, ox0 = tx * kMpTW;
  const int rows = kMpTH + KH - 1, cols = kMpTW + KW - 1;
  auto vmax = [&](uint4 a, uint4 b) {
    return x.is_signed ? make_uint4(__vmaxs4(a.x, b.x), __vmaxs4(a.y, b.y), __vmaxs4(a.z, b.z),
                                    __vmaxs4(a.w, b.w))
                       : make_uint4(__vmaxu4(a.x, b.x), __vmaxu4(a.y, b.y), __vmaxu4(a.z, b.z),
                                    __vmaxu4(a.w, b.w));
  };
  for (int i = threadIdx.x; i < rows * cols; i += blockDim.x) {
    const int r = i / cols, c = i - r * cols;
    const int64_t iy = oy0 - PH + r, ix = ox0 - PW + c;
    uint4 v = make_uint4(pad_word, pad_word, pad_word, pad_word);
    if (iy >= 0 && iy < H && ix >= 0 && ix < W)
      v = __ldg(reinterpret_cast<const uint4*>(x.p + ((n * H + iy) * W + ix) * x.stride +
                                               g * 16));
    s_in[r][c] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * kMpTW; i += blockDim.x) {
    const int r = i / kMpTW, c = i - r * kMpTW;
    uint4 m = s_in[r][c];
    for (int k = 1; k < KW; ++k) m = vmax(m, s_in[r][c + k]);
    s_row[r][c] = m;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kMpTH * kMpTW; i += blockDim.x) {
    const int r = i / kMpTW, c = i - r * kMpTW;
    const int64_t oy = oy0 + r, ox = ox0 + c;
    if (oy >= OH || ox >= OW) continue;
    uint4 m = s_row[r][c];
    for (int k = 1; k < KH; ++k) m = vmax(m, s_row[r + k][c]);
    *reinterpret_cast<uint4*>(y + ((n * OH + oy) * OW + ox) * y_stride + g * 16) = m;
  }
}

// Column walker for stride-1 max pools with a KH x KW window known at compile
// time: a thread owns two neighbouring output columns of one image and one
// 16-channel group (lanes walk the groups of consecutive pixel pairs, so a
// warp reads and writes contiguous bytes), walks down a chunk of output
// rows, takes each input row's maxima over the horizontal taps (neighbouring
// lanes' loads hit L1) and keeps the last KH row maxima in registers: every
// input byte comes from DRAM once, every output byte is written once.
// The maxima run on 16-bit lanes with one native `max.{s,u}16x2` per two
// bytes.  A 16-bit lane compares its high byte first (signed for signed
// bytes, as `max.s16x2` reads it), so the high byte of a lane maximum is the
// maximum of the high bytes whatever the low bytes hold: a 16-byte vector
// is kept as eight words, each input word w as is (its odd bytes 1 and 3
// are lane high bytes) and w << 8 (its even bytes 0 and 2 become lane high
// bytes); the result's high bytes are gathered back with one `prmt` a word.
struct Wide16 {
  uint32_t e[4], o[4];  // word i << 8 (even bytes high) / word i (odd bytes high)
};

template <bool kSigned>
__device__ __forceinline__ Wide16 widen16(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  Wide16 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r.e[i] = w[i] << 8;
    r.o[i] = w[i];
  }
  return r;
}

template <bool kSigned>
__device__ __forceinline__ uint32_t max16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (kSigned)
    asm("max.s16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <bool kSigned>
__device__ __forceinline__ Wide16 wmax16(const Wide16& a, const Wide16& b) {
  Wide16 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r.e[i] = max16x2<kSigned>(a.e[i], b.e[i]);
    r.o[i] = max16x2<kSigned>(a.o[i], b.o[i]);
  }
  return r;
}

__device__ __forceinline__ uint4 narrow16(const Wide16& a) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)  // high bytes: even lane 0, odd lane 0, even lane 1, odd lane 1
    asm("prmt.b32 %0, %1, %2, 0x7351;" : "=r"(w[i]) : "r"(a.e[i]), "r"(a.o[i]));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Two output columns per thread: the windows of columns ox and ox + 1 share
// K - 1 of their K + 1 taps, so a row costs K + 1 loads and one maximum of
// the middle K - 1 taps for both columns, and a thread keeps two fresh
// 16-byte DRAM loads in flight.  The row maxima of the K input rows under
// output row oy live in one ring per column, packed (16 bytes each):
// input row oy - PH + k sits in slot (oy - oy0 + k) % K; the row loop is
// unrolled K times so that every ring index is a constant.
template <int K, bool kSigned>
__global__ void __launch_bounds__(256)
    maxpool_s1_pairs_kernel(const uint8_t* __restrict__ x, int64_t x_stride,
                            uint8_t* __restrict__ y, int64_t y_stride, int H, int W, int groups,
                            int PH, int PW, int OH, int OW, int rows_per, int chunks,
                            int64_t total, uint32_t pad_word) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  const int pairs = (OW + 1) / 2;
  const int g = (int)(t % groups);
  int64_t rest = t / groups;
  const int ox = 2 * (int)(rest % pairs);
  rest /= pairs;
  const int chunk = (int)(rest % chunks);
  const int64_t n = rest / chunks;
  const int oy0 = chunk * rows_per;
  const int oy1 = min(OH, oy0 + rows_per);
  const bool two = ox + 1 < OW;
  const uint4 padv = make_uint4(pad_word, pad_word, pad_word, pad_word);
  // taps j = 0 .. K: input column ox - PW + j (column ox reads 0 .. K - 1,
  // column ox + 1 reads 1 .. K)
  uint32_t inside = 0;
#pragma unroll
  for (int j = 0; j <= K; ++j) {
    const int ix = ox - PW + j;
    inside |= (ix >= 0 && ix < W ? 1u : 0u) << j;
  }
  const int64_t row_bytes = (int64_t)W * x_stride;
  const uint8_t* const col = x + n * H * row_bytes + (int64_t)(ox - PW) * x_stride + g * 16;
  const bool full = inside == (1u << (K + 1)) - 1;
  auto hmax = [&](int iy, uint4& m0, uint4& m1) {
    if (iy < 0 || iy >= H) {  // a padded row holds the pad value
      m0 = padv;
      m1 = padv;
      return;
    }
    const uint8_t* p = col + (int64_t)iy * row_bytes;
    uint4 v[K + 1];
    if (full) {
#pragma unroll
      for (int j = 0; j <= K; ++j) v[j] = __ldg(reinterpret_cast<const uint4*>(p + j * x_stride));
    } else {
#pragma unroll
      for (int j = 0; j <= K; ++j)
        v[j] = (inside & (1u << j)) ? __ldg(reinterpret_cast<const uint4*>(p + j * x_stride))
                                    : padv;
    }
    Wide16 mid = widen16<kSigned>(v[1]);
#pragma unroll
    for (int j = 2; j < K; ++j) mid = wmax16<kSigned>(mid, widen16<kSigned>(v[j]));
    m0 = narrow16(wmax16<kSigned>(mid, widen16<kSigned>(v[0])));
    m1 = narrow16(wmax16<kSigned>(mid, widen16<kSigned>(v[K])));
  };
  uint4 w0[K], w1[K];
#pragma unroll
  for (int k = 0; k < K - 1; ++k) hmax(oy0 - PH + k, w0[k], w1[k]);
  uint8_t* out = y + ((n * OH + oy0) * OW + ox) * y_stride + g * 16;
  const int64_t out_row = (int64_t)OW * y_stride;
  for (int oy = oy0; oy < oy1; oy += K) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (oy + j < oy1) {
        hmax(oy + j - PH + K - 1, w0[(j + K - 1) % K], w1[(j + K - 1) % K]);
        Wide16 a = widen16<kSigned>(w0[0]), b = widen16<kSigned>(w1[0]);
#pragma unroll
        for (int k = 1; k < K; ++k) {
          a = wmax16<kSigned>(a, widen16<kSigned>(w0[k]));
          b = wmax16<kSigned>(b, widen16<kSigned>(w1[k]));
        }
        *reinterpret_cast<uint4*>(out) = narrow16(a);
        if (two) *reinterpret_cast<uint4*>(out + y_stride) = narrow16(b);
        out += out_row;
      }
    }
  }
}

__host__ __device__ inline bool vec16_ok(const void* p, int64_t stride) {
  return ((reinterpret_cast<uintptr_t>(p) | (uint64_t)stride) & 15) == 0;
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

// out = clamp(mbqm((a - za)(b - zb), m, s) + zo): the integer Mul of two
// activations (qa_kernels.cpp:334-345, quant_layers.py:516-540).
__global__ void mul_bytes_kernel(ByteView a, ByteView b, uint8_t* __restrict__ y,
                                 int64_t y_stride, int64_t rows, int64_t C, int64_t za,
                                 int64_t zb, int64_t m, int64_t s, int64_t zo, int64_t qmin,
                                 int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const int64_t va = bval(a.p + r * a.stride + c, a.is_signed) - za;
    const int64_t vb = bval(b.p + r * b.stride + c, b.is_signed) - zb;
    y[r * y_stride + c] = (uint8_t)requant_exact(va * vb, m, s, zo, qmin, qmax);
  }
}

// Inference BatchNorm (quant_layers.py:405-441): per channel
// clamp(mbqm(x - zp_in, mult[c], shift[c]) + post[c] + zp_out).
__global__ void bn_bytes_kernel(ByteView x, uint8_t* __restrict__ y, int64_t y_stride,
                                int64_t rows, int64_t C, int64_t zp_in,
                                const int64_t* __restrict__ mult,
                                const int64_t* __restrict__ shift,
                                const int64_t* __restrict__ post, int64_t zp_out, int64_t qmin,
                                int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const int64_t v = bval(x.p + r * x.stride + c, x.is_signed) - zp_in;
    y[r * y_stride + c] = (uint8_t)requant_exact(v, __ldg(mult + c), __ldg(shift + c),
                                                 __ldg(post + c) + zp_out, qmin, qmax);
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
    return launch_ex(C == 3 ? quantize_to_nhwc4_kernel<true> : quantize_to_nhwc4_kernel<false>,
                     dim3(grid_for(quads, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), (int)C,
                     (int)(HW / 4), (int)quads, (int)W, 0, make_quant_k(scale, zp, qmin, qmax))
               ? 0
               : last_status();
  }
  return launch_ex(quantize_to_nhwc_kernel, dim3(grid_for(n, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), N, C, HW,
                   pix_stride, scale, (double)zp, (double)qmin, (double)qmax)
             ? 0
             : last_status();
}

QA_API int qa_quantize_to_patch_rows_dev(const float* x, void* y, int64_t N, int64_t C, int64_t H,
                                         int64_t W, int64_t P, double scale, int64_t zp,
                                         int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (N < 0 || C <= 0 || C > 4 || P <= 0 || P % 4 || H % P || W % P || W % 4 || scale == 0.0 ||
      N * H * W / 4 >= 0x7FFFFFFF || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 15)) {
    set_error(kBadArgument, "qa_quantize_to_patch_rows_dev: bad arguments");
    return last_status();
  }
  const int64_t quads = N * H * W / 4;
  if (quads == 0) return 0;
  return launch_ex(C == 3 ? quantize_to_nhwc4_kernel<true> : quantize_to_nhwc4_kernel<false>,
                   dim3(grid_for(quads, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), (int)C,
                   (int)(H * W / 4), (int)quads, (int)W, (int)P,
                   make_quant_k(scale, zp, qmin, qmax))
             ? 0
             : last_status();
}

QA_API int qa_gap_dev(const void* x, int64_t x_pix_stride, int64_t x_signed, int64_t N,
                      int64_t HW, int64_t C, int64_t zp_in, int64_t mult, int64_t shift,
                      int64_t zp_out, int64_t qmin, int64_t qmax, void* y, int64_t y_pix_stride,
                      void* stream) {
  clear_error();
  if (N * C == 0) return 0;
  if (C % 16 == 0 && x_pix_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      HW >= 1 && HW <= 256 && N * HW * x_pix_stride < (int64_t(1) << 62)) {
    // 64-bit rescale exact: |sum| <= HW * 383 + HW * |zp_in|, the rounded
    // product below 2^62
    const int64_t ts = 31 + shift;
    const double bound = (double)HW * (383.0 + std::fabs((double)zp_in)) *
                             std::fabs((double)mult) + std::ldexp(1.0, (int)std::min<int64_t>(ts, 62));
    const int fast = ts >= 1 && ts <= 62 && bound < std::ldexp(1.0, 62) ? 1 : 0;
    const int64_t total = N * (C / 16);
    // one (image, group) per thread in a single pass: a capped grid would
    // leave a partly filled second round
    const int64_t gblocks = std::max<int64_t>(1, (total + 127) / 128);
    return launch_ex(gap16_thread_kernel,
                     dim3((unsigned)std::min<int64_t>(gblocks, 0x7FFFFFFF)), dim3(128), 0,
                     (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_pix_stride,
                     (int)x_signed, N, (int)HW, C / 16, zp_in, mult, shift, zp_out, qmin, qmax,
                     fast, static_cast<uint8_t*>(y), y_pix_stride)
               ? 0
               : last_status();
  }
  if (C % 16 == 0 && x_pix_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      HW < (int64_t(1) << 23)) {
    const int64_t warps = N * (C / 16);
    return launch_ex(gap16ch_kernel, dim3(grid_for(warps * 32, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_pix_stride,
                     (int)x_signed, N, HW, C, zp_in, mult, shift, zp_out, qmin, qmax,
                     static_cast<uint8_t*>(y), y_pix_stride)
               ? 0
               : last_status();
  }
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
  if (C % 16 == 0 && vec16_ok(x, x_stride) && vec16_ok(y, y_stride)) {
    ByteMap mp{};
    mp.is_signed = (int)x_signed;
    mp.kind = 0;
    mp.lut = lut;
    mp.offset = offset;
    mp.len = lut_len;
    return launch_ex(map_bytes16_kernel, dim3(grid_for(rows * C / 16, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true,
                     ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
                     static_cast<uint8_t*>(y), y_stride, rows, C / 16, mp)
               ? 0
               : last_status();
  }
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
  // |mbqm(v - z, m, s)| <= (384 + |z|) * |m| * 2^-(31 + s) + 1 for every byte v
  auto term_small = [](int64_t z, int64_t m, int64_t s) {
    if (s < -64 || s > 64) return false;
    const double t = (384.0 + std::fabs((double)z)) * std::fabs((double)m) *
                         std::ldexp(1.0, -(int)(31 + s)) + 2.0;
    return t < std::ldexp(1.0, 29) * 0.999;
  };
  const bool vec = C % 16 == 0 && vec16_ok(a, a_stride) && vec16_ok(b, b_stride) &&
                   vec16_ok(y, y_stride);
  if (vec && term_small(za, ma, sa) && term_small(zb, mb, sb) && (sign == 1 || sign == -1) &&
      zo > -(1 << 30) && zo < (1 << 30) && qmin >= -128 && qmax <= 255) {
    const size_t smem = 2 * 256 * 32 * sizeof(int32_t);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      if (cuda_failed(cudaFuncSetAttribute(add_bytes16_rep_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem),
                      "cudaFuncSetAttribute(add_rep)"))
        return last_status();
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int64_t vectors = rows * C / 16;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((vectors + kAddRepThreads - 1) /
                                                                     kAddRepThreads,
                                                                 (int64_t)sm_count() * 3));
    return launch_ex(add_bytes16_rep_kernel, dim3((unsigned)grid), dim3(kAddRepThreads), smem,
                     (cudaStream_t)stream, true,
                     ByteView{static_cast<const uint8_t*>(a), a_stride, (int)a_signed},
                     ByteView{static_cast<const uint8_t*>(b), b_stride, (int)b_signed},
                     static_cast<uint8_t*>(y), y_stride, rows, C / 16, za, ma, sa, zb, mb, sb,
                     sign, zo, qmin, qmax)
               ? 0
               : last_status();
  }
  if (vec)
    return launch_ex(add_bytes16_kernel, dim3(grid_for(rows * C / 16, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true,
                     ByteView{static_cast<const uint8_t*>(a), a_stride, (int)a_signed},
                     ByteView{static_cast<const uint8_t*>(b), b_stride, (int)b_signed},
                     static_cast<uint8_t*>(y), y_stride, rows, C / 16, za, ma, sa, zb, mb, sb,
                     sign, zo, qmin, qmax)
               ? 0
               : last_status();
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
  if (C % 16 == 0 && vec16_ok(x, x_stride) && vec16_ok(y, y_stride)) {
    ByteMap mp{};
    mp.is_signed = (int)x_signed;
    mp.kind = 1;
    mp.identity = identity != 0;
    mp.zin = zp_in;
    mp.m = m;
    mp.s = s;
    mp.zout = zp_out;
    mp.qmin = qmin;
    mp.qmax = qmax;
    return launch_ex(map_bytes16_kernel, dim3(grid_for(rows * C / 16, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true,
                     ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
                     static_cast<uint8_t*>(y), y_stride, rows, C / 16, mp)
               ? 0
               : last_status();
  }
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
  const bool s1_vec = C % 16 == 0 && vec16_ok(x, x_stride) && vec16_ok(y, y_stride) &&
                      SH == 1 && SW == 1 && DH == 1 && DW == 1;
  if (s1_vec && KH == KW && (KH == 3 || KH == 5) && OH == H + 2 * PH - KH + 1 &&
      OW == W + 2 * PW - KW + 1 && H * W * x_stride < (int64_t(1) << 31) && OW < (1 << 20)) {
    // column walker: output rows in chunks of at most 16, enough threads to
    // fill the GPU
    const uint32_t pw = ((uint32_t)pad_value & 0xFFu) * 0x01010101u;
    const int rows_per = (int)std::min<int64_t>(OH, 16);
    const int chunks = (int)((OH + rows_per - 1) / rows_per);
    const int64_t threads = N * chunks * ((OW + 1) / 2) * (C / 16);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    auto kern = KH == 3 ? (x_signed ? maxpool_s1_pairs_kernel<3, true>
                                    : maxpool_s1_pairs_kernel<3, false>)
                        : (x_signed ? maxpool_s1_pairs_kernel<5, true>
                                    : maxpool_s1_pairs_kernel<5, false>);
    return launch_ex(kern, dim3(blocks), dim3(256), 0, (cudaStream_t)stream, true,
                     static_cast<const uint8_t*>(x), x_stride, static_cast<uint8_t*>(y), y_stride,
                     (int)H, (int)W, (int)(C / 16), (int)PH, (int)PW, (int)OH, (int)OW, rows_per,
                     chunks, threads, pw)
               ? 0
               : last_status();
  }
  if (s1_vec && KH <= kMpMaxK && KW <= kMpMaxK && KH >= 1 && KW >= 1) {
    const uint32_t pw = ((uint32_t)pad_value & 0xFFu) * 0x01010101u;
    const int64_t tiles_x = (OW + kMpTW - 1) / kMpTW, tiles_y = (OH + kMpTH - 1) / kMpTH;
    const int64_t blocks = tiles_x * tiles_y * N * (C / 16);
    if (blocks < 0x7FFFFFFF)
      return launch_ex(maxpool_bytes16_s1_kernel, dim3((unsigned)blocks), dim3(256), 0,
                       (cudaStream_t)stream, true,
                       ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
                       static_cast<uint8_t*>(y), y_stride, H, W, C / 16, (int)KH, (int)KW, PH,
                       PW, OH, OW, tiles_x, tiles_y, pw)
                 ? 0
                 : last_status();
  }
  if (C % 16 == 0 && vec16_ok(x, x_stride) && vec16_ok(y, y_stride)) {
    const uint32_t pw = ((uint32_t)pad_value & 0xFFu) * 0x01010101u;
    return launch_ex(maxpool_bytes16_kernel, dim3(grid_for(N * OH * OW * (C / 16), 256)),
                     dim3(256), 0, (cudaStream_t)stream, true,
                     ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
                     static_cast<uint8_t*>(y), y_stride, N, H, W, C / 16, KH, KW, SH, SW, PH, PW,
                     DH, DW, OH, OW, pw)
               ? 0
               : last_status();
  }
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

// ======================================================== window copy ==
// The resident form of the scale-preserving layout operators Pad, Slice and
// Transpose (quant_layers.py:593-650; float_ops.py Pad / Slice / Transpose):
// an NHWC byte tensor is copied into a new one, output element (n, c, y, x)
// (NCHW order) reading source element
//     base + sum_a (start[a] + i[a] * step[a]) * stride[a]
// (i = (n, c, y, x); stride[a] in bytes of the source axis that output axis
// a reads, so a Transpose permutes the strides), or `fill` -- the Pad's zero
// point -- when a source coordinate lies outside [0, dim[a]).  A thread
// writes one 16-channel chunk of one output pixel.
namespace qa {
namespace {
struct WindowGeom {
  int64_t start[4], step[4], dim[4], stride[4];
};

__global__ void window_copy_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                   int64_t y_stride, int64_t ON, int64_t OC, int64_t OH,
                                   int64_t OW, WindowGeom g, uint32_t fill, int vec) {
  ptx::pdl_wait();
  const int64_t chunks = (OC + 15) / 16;
  const int64_t total = ON * OH * OW * chunks;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t cg = t % chunks;
    const int64_t pix = t / chunks;
    const int64_t ox = pix % OW, oy = (pix / OW) % OH, n = pix / (OW * OH);
    const int64_t sn = g.start[0] + n * g.step[0], sy = g.start[2] + oy * g.step[2],
                  sx = g.start[3] + ox * g.step[3];
    const bool pix_in = (uint64_t)sn < (uint64_t)g.dim[0] && (uint64_t)sy < (uint64_t)g.dim[2] &&
                        (uint64_t)sx < (uint64_t)g.dim[3];
    const int64_t base = sn * g.stride[0] + sy * g.stride[2] + sx * g.stride[3];
    uint32_t w[4] = {0, 0, 0, 0};
    const int64_t c0 = cg * 16;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t sc = g.start[1] + (c0 + j) * g.step[1];
      const bool in = pix_in && (uint64_t)sc < (uint64_t)g.dim[1];
      const uint32_t b = in ? (uint32_t)x[base + sc * g.stride[1]] : fill;
      w[j >> 2] |= (b & 0xFFu) << (8 * (j & 3));
    }
    uint8_t* dst = y + pix * y_stride + c0;
    if (vec && c0 + 16 <= OC) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int j = 0; j < 16 && c0 + j < OC; ++j) dst[j] = (uint8_t)(w[j >> 2] >> (8 * (j & 3)));
    }
  }
}
}  // namespace
}  // namespace qa

QA_API int qa_window_copy_bytes_dev(const void* x, void* y, int64_t y_pix_stride, int64_t ON,
                                    int64_t OC, int64_t OH, int64_t OW, const int64_t* start,
                                    const int64_t* step, const int64_t* dim,
                                    const int64_t* stride, int64_t fill, void* stream) {
  clear_error();
  QA_REQUIRE(x && y && start && step && dim && stride && ON >= 0 && OC >= 0 && OH >= 0 &&
                 OW >= 0 && y_pix_stride >= OC,
             "qa_window_copy_bytes_dev: bad arguments", last_status());
  QA_REQUIRE(fill >= -128 && fill <= 255, "qa_window_copy_bytes_dev: fill must be a byte value",
             last_status());
  const int64_t total = ON * OH * OW * ((OC + 15) / 16);
  if (total == 0) return 0;
  WindowGeom g;
  for (int a = 0; a < 4; ++a) {
    g.start[a] = start[a];
    g.step[a] = step[a];
    g.dim[a] = dim[a];
    g.stride[a] = stride[a];
  }
  const int vec = (reinterpret_cast<uintptr_t>(y) % 16 == 0) && (y_pix_stride % 16 == 0);
  return launch_ex(window_copy_kernel, dim3(grid_for(total, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x),
                   static_cast<uint8_t*>(y), y_pix_stride, ON, OC, OH, OW, g,
                   (uint32_t)(fill & 0xFF), vec)
             ? 0
             : last_status();
}

// Self-test of the bounded-wait error channel every tensor-core kernel uses:
// one thread initialises an mbarrier expecting one arrival, arrives on it
// only when `arrive` is set, and waits with the same bounded wait as the
// kernels.  A wait that runs out records its code in the device status word
// (read by qa_device_status_dev) and the thread returns; no copy is in
// flight, so the context stays usable.
namespace qa {
namespace {
constexpr int kWaitProbeTimeoutCode = 0x7100;

__global__ void wait_probe_kernel(int* status, unsigned long long budget_cycles, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = ptx::smem_addr(&bar);
  ptx::mbar_init(b, 1);
  ptx::fence_mbar_init();
  if (arrive) ptx::mbar_arrive(b);
  if (!ptx::mbar_wait(b, 0, budget_cycles)) atomicExch(status, kWaitProbeTimeoutCode);
}
}  // namespace
}  // namespace qa

QA_API int qa_wait_probe_dev(int64_t budget_cycles, int arrive, void* stream) {
  clear_error();
  QA_REQUIRE(budget_cycles >= 0 && budget_cycles <= (int64_t(1) << 32),
             "qa_wait_probe_dev: budget must lie in [0, 2^32] SM cycles", last_status());
  int* status = device_status_word();
  if (!status) return last_status();
  return launch_ex(wait_probe_kernel, dim3(1), dim3(1), 0, (cudaStream_t)stream, false, status,
                   (unsigned long long)budget_cycles, arrive)
             ? 0
             : last_status();
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

// 16 x 28 output pixels per tile (448 rows of four 128-row MMA blocks, the
// last one half used): 28 divides the 112-pixel rows of a 224 x 224 image
// after a stride-2 stem, and a multiple of 4 keeps every tile's first input
// column on one residue mod 4
constexpr int kInTileH = 16, kInTileW = 28, kInThreads = 256;
constexpr int kInPix = kInTileH * kInTileW;
constexpr int kInMaxCout = 64;
constexpr int kInMaxTaps = 16;  // K = taps * 4 bytes <= 64: four 16-byte K chunks
constexpr int kInTab = 384;     // byte-domain activation table, index v + 128
constexpr int kInStages = 2;    // float patches in flight per CTA
constexpr int kInABlock = 128 * 64;  // one 128-row A block: 4 K chunks x 16 row groups x 128 B
constexpr uint64_t kInBudget = 4000000000ull;  // bounded waits (~2 s)

struct InputConvParams {
  int32_t N, C, H, W, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW, Cout, CoutP;
  int32_t patch_h, patch_w;  // input pixels a tile reads
  int32_t box_w, shift;      // TMA box width (floats, multiple of 4); patch column 0 in the box
  int32_t stage_bytes;       // one float patch (C x patch_h x box_w), 1024-aligned
  int32_t tiles_x, tiles_y, tiles;
  int32_t tmem_cols;
  uint32_t pw_magic;         // ceil(2^32 / patch_w): i / patch_w == umulhi(i, pw_magic)
  int32_t patch_words;       // quantized patch words in shared memory (stem form: patch_h x box_w)
  QuantK qk;
  const int8_t* w;  // [Cout][KH*KW*4] rows of w_kp bytes
  int64_t w_kp;
  int32_t fast;
  int32_t vec_out;  // output base and pixel stride 16-byte aligned
  int32_t* status;
  FusedEpilogue epi;
};

// Bytes of 16 channel values of one pixel (16-byte store when aligned).
__device__ __forceinline__ void store_pixel16(const int32_t (&q)[16], uint8_t* op, bool vec,
                                              int nval) {
  uint32_t o[4];
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4)
    o[k4] = __byte_perm(__byte_perm((uint32_t)q[4 * k4], (uint32_t)q[4 * k4 + 1], 0x0040),
                        __byte_perm((uint32_t)q[4 * k4 + 2], (uint32_t)q[4 * k4 + 3], 0x0040),
                        0x5410);
  if (vec) {
    *reinterpret_cast<uint4*>(op) = make_uint4(o[0], o[1], o[2], o[3]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nval) op[j] = (uint8_t)(o[j >> 2] >> (8 * (j & 3)));
  }
}

// Graph input quantization fused with the first convolution, on the tensor
// cores.  Persistent: each CTA walks 16 x 28 tiles of output pixels.
//   * thread 0 keeps kInStages float input patches in flight by TMA (4-D
//     tiled loads of C x patch_h x box_w; outside the image they read 0.0,
//     which quantizes to the input zero point exactly as the reference pads);
//   * the block quantizes the patch (quantize_bits_try) into one 4-channel
//     word per input pixel, then writes the 448 implicit-GEMM rows (one
//     4-byte tap per word, K <= 64) as four 128-row A blocks in the plain
//     K-major layout (8-row x 16-byte core matrices);
//   * thread 0 issues tcgen05.mma (M = 128, N = Cout rounded to 16) for the
//     four blocks into four TMEM accumulators and commits;
//   * all eight warps drain TMEM (warp w: lanes 32 * (w % 4), blocks
//     2 * (w / 4) and 2 * (w / 4) + 1) through the fused epilogue
//     (high-word requantize, byte-domain activation table).
__global__ void __launch_bounds__(kInThreads, 2)
    input_conv_kernel(const __grid_constant__ InputConvParams p,
                      const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ uint8_t in_smem_raw[];
  const uint32_t raw = ptx::smem_addr(in_smem_raw);
  uint8_t* sm = in_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int CoutP = p.CoutP, taps = p.KH * p.KW;
  const float* s_x = reinterpret_cast<const float*>(sm);
  uint8_t* s_a = sm + kInStages * p.stage_bytes;        // 4 A blocks
  uint8_t* s_b = s_a + 4 * kInABlock;                   // CoutP rows x 64 B, same layout
  int4* s_ch = reinterpret_cast<int4*>(s_b + CoutP * 64);
  int64_t* s_bias = reinterpret_cast<int64_t*>(s_ch + CoutP);
  int64_t* s_mult = s_bias + CoutP;
  int64_t* s_shift = s_mult + CoutP;
  int32_t* s_tab = reinterpret_cast<int32_t*>(s_shift + CoutP);
  int32_t* s_tapoff = s_tab + kInTab;  // patch word offset of each tap
  uint32_t* s_patch = reinterpret_cast<uint32_t*>(s_tapoff + kInMaxTaps);  // patch_h * patch_w words
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(s_patch + p.patch_h * p.patch_w) + 7) & ~uintptr_t(7));
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + kInStages + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  const uint32_t bar0 = ptx::smem_addr(bars);
  const uint32_t mma_bar = bar0 + 8u * kInStages;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const FusedEpilogue& e = p.epi;
  // B: row co, K chunk j at j * (CoutP / 8) * 128 + (co / 8) * 128 + (co % 8) * 16
  const uint32_t b_lbo = (uint32_t)(CoutP / 8) * 128u;

  // static operands, loaded while the previous kernel may still run
  int hi_ok = 1;
  for (int i = tid; i < CoutP * 4; i += kInThreads) {
    const int co = i / 4, j = i % 4;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (co < p.Cout) {
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int tap = 4 * j + q;
        wv[q] = tap < taps ? *reinterpret_cast<const uint32_t*>(p.w + co * p.w_kp + tap * 4) : 0u;
      }
      v = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    *reinterpret_cast<uint4*>(s_b + j * b_lbo + (co / 8) * 128 + (co % 8) * 16) = v;
  }
  for (int c = tid; c < CoutP; c += kInThreads) {
    const bool v = c < p.Cout;
    s_bias[c] = (v && e.bias) ? e.bias[c] : 0;
    s_mult[c] = v ? e.mult[c] : 0;
    s_shift[c] = v ? e.shift[c] : 0;
    const int ts = (int)(31 + s_shift[c]);
    const bool hi = ts >= 33 && ts <= 62;
    if (v && !hi) hi_ok = 0;
    const int sh = hi ? ts - 32 : 1;
    s_ch[c] = make_int4((int32_t)s_bias[c], (int32_t)s_mult[c], 1 << (sh - 1), sh);
  }
  if (e.lut)
    for (int i = tid; i < kInTab; i += kInThreads) {
      const int64_t idx = min(max((int64_t)(i - 128) - e.lut_offset, (int64_t)0), e.lut_len - 1);
      s_tab[i] = (int32_t)min(max((int64_t)e.lut[idx], (int64_t)-128), (int64_t)255);
    }
  if (tid < kInMaxTaps) {
    const int ky = tid / p.KW, kx = tid - (tid / p.KW) * p.KW;
    s_tapoff[tid] = tid < taps ? ky * p.DH * p.patch_w + kx * p.DW : 0;
  }
  ptx::fence_proxy_async_smem();  // B, written here, is read by the tensor cores
  if (tid == 0) {
    for (int s = 0; s <= kInStages; ++s) ptx::mbar_init(bar0 + 8u * s, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&xmap);
  }
  if (warp == 0) {
    ptx::tmem_alloc(ptx::smem_addr(s_tmem), (uint32_t)p.tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  const int hi_all = __syncthreads_and(hi_ok);
  ptx::tc_fence_after();
  const uint32_t tmem = *s_tmem;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();

  // tile k of this CTA is blockIdx.x + k * gridDim.x
  auto issue = [&](int k) {
    const int t = blockIdx.x + k * gridDim.x;
    const int img = t / (p.tiles_x * p.tiles_y), r = t - img * p.tiles_x * p.tiles_y;
    const int oy0 = (r / p.tiles_x) * kInTileH, ox0 = (r % p.tiles_x) * kInTileW;
    const int s = k % kInStages;
    ptx::mbar_arrive_expect_tx(bar0 + 8u * s, (uint32_t)(p.C * p.patch_h * p.box_w * 4));
    ptx::tma_load_4d(ptx::smem_addr(sm) + s * p.stage_bytes, &xmap, bar0 + 8u * s,
                     ox0 * p.SW - p.PW - p.shift, oy0 * p.SH - p.PH, 0, img);
  };
  const int my_tiles = p.tiles > (int)blockIdx.x
                           ? (p.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                           : 0;
  int issued = 0;  // tiles whose patch load thread 0 has issued
  int mmas = 0;    // tiles whose MMAs thread 0 has committed
  if (tid == 0)
    for (; issued < kInStages && issued < my_tiles; ++issued) issue(issued);

  const bool hi_rq = p.fast && hi_all && e.zp > -(1 << 20) && e.zp < (1 << 20);
  const int32_t zp32 = (int32_t)e.zp, qmin32 = (int32_t)e.qmin, qmax32 = (int32_t)e.qmax;
  const int32_t* t_lut = s_tab + 128;
  const bool has_lut = e.lut != nullptr;
  uint8_t* const out_p = e.out;
  const int64_t out_stride = e.out_pix_stride;
  const QuantK qk = p.qk;  // in registers: no generic parameter loads in the loops
  const uint32_t in_zp = (uint32_t)qk.zp_i & 0xFFu;
  const int plane = p.patch_h * p.box_w;  // floats per channel in a staged patch
  const int npatch = p.patch_h * p.patch_w;
  const uint32_t idesc = ptx::idesc_i8(128, CoutP, 1, 1);
  const int ksteps = (taps * 4 + 31) / 32;
  const uint32_t a_base = ptx::smem_addr(s_a), b_base = ptx::smem_addr(s_b);
  const int quarter = warp & 3, half = warp >> 2;

  int k = 0;
  for (; k < my_tiles; ++k) {
    const int t = blockIdx.x + k * gridDim.x;
    const int img = t / (p.tiles_x * p.tiles_y), r = t - img * p.tiles_x * p.tiles_y;
    const int oy0 = (r / p.tiles_x) * kInTileH, ox0 = (r % p.tiles_x) * kInTileW;
    const int s = k % kInStages;
    if (!ptx::mbar_wait_sleep(bar0 + 8u * s, (k / kInStages) & 1, kInBudget)) {
      *s_abort = 1;
      if (p.status) atomicExch(p.status, 0x7003);
    }
    // (1) quantize the staged float patch into 4-channel words
    const float* xs = s_x + s * (p.stage_bytes / 4) + p.shift;
#pragma unroll 2
    for (int i = tid; i < npatch; i += kInThreads) {
      const int py = (int)__umulhi((uint32_t)i, p.pw_magic), px = i - py * p.patch_w;
      const float* src = xs + py * p.box_w + px;
      float f[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) f[c] = c < p.C ? src[c * plane] : 0.f;
      bool ok = true;
      uint32_t b[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) b[c] = c < p.C ? quantize_bits_try(f[c], qk, ok) : in_zp;
      uint32_t word = pack_bytes(b[0], b[1], b[2], b[3]);
      if (!ok) word = quantize_word_exact(src, plane, p.C, in_zp, p.qk);
      s_patch[i] = word;
    }
    __syncthreads();
    if (*s_abort) break;
    // stage s is free again: thread 0 refills it
    if (tid == 0 && issued < my_tiles) {
      ptx::fence_proxy_async_smem();
      issue(issued++);
    }
    // (2) the implicit-GEMM rows: pixel P of the tile is row P % 128 of
    // block P / 128; chunk j holds taps 4j .. 4j + 3
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int P = tid + u * kInThreads;
      if (P >= kInPix) continue;  // rows past the tile: their results are discarded
      const int py = P / kInTileW, px = P % kInTileW;
      const int base = py * p.SH * p.patch_w + px * p.SW;
      uint8_t* row = s_a + (P / 128) * kInABlock + ((P % 128) / 8) * 128 + (P % 8) * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t wv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int tap = 4 * j + q;
          // taps past the filter read word 0 (in bounds) and contribute 0
          const int idx = tap < taps ? base + s_tapoff[tap] : 0;
          const uint32_t wd = s_patch[idx];
          wv[q] = tap < taps ? wd : 0u;
        }
        if (4 * j < taps || j < 2 * ksteps)
          *reinterpret_cast<uint4*>(row + j * 2048) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();
    // (3) the tensor cores: four 128-row blocks into four accumulators
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll 1
      for (int b = 0; b < 4; ++b)
        for (int kk = 0; kk < ksteps; ++kk)
          ptx::mma_i8(tmem + (uint32_t)(b * CoutP),
                      ptx::smem_desc_kmajor_plain(a_base + b * kInABlock + kk * 4096, 2048, 128),
                      ptx::smem_desc_kmajor_plain(b_base + kk * 2 * b_lbo, b_lbo, 128), idesc,
                      kk > 0 ? 1u : 0u);
      ptx::mma_commit(mma_bar);
      ++mmas;
    }
    if (!ptx::mbar_wait_sleep(mma_bar, k & 1, kInBudget)) {
      *s_abort = 1;
      if (p.status) atomicExch(p.status, 0x7003);
    }
    __syncwarp();
    ptx::tc_fence_after();
    // (4) epilogue: this warp's 32 rows of blocks 2 * half and 2 * half + 1
#pragma unroll 1
    for (int bb = 0; bb < 2; ++bb) {
      const int b = 2 * half + bb;
      const int P = b * 128 + quarter * 32 + lane;
      const int oy = oy0 + P / kInTileW, ox = ox0 + P % kInTileW;
      const bool valid = P < kInPix && oy < p.OH && ox < p.OW && !*s_abort;
      const int64_t m = ((int64_t)img * p.OH + oy) * p.OW + ox;
#pragma unroll 1
      for (int c0 = 0; c0 < CoutP; c0 += 16) {
        uint32_t v[16];
        ptx::tmem_ld16(tmem + (((uint32_t)quarter * 32u) << 16) + (uint32_t)(b * CoutP + c0), v);
        ptx::tmem_ld_wait(v);
        const int nval = min(16, p.Cout - c0);
        if (!valid || nval <= 0) continue;
        int32_t q[16];
        if (hi_rq) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int4 ch = s_ch[c0 + j];
            const int32_t rq = (__mulhi((int32_t)v[j] + ch.x, ch.y) + ch.z) >> ch.w;
            q[j] = min(max(rq + zp32, qmin32), qmax32);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int c = c0 + j;
            const int64_t xv = (int64_t)(int32_t)v[j] + s_bias[c];
            q[j] = p.fast ? (int32_t)requant_fast(xv, s_mult[c], (int)(31 + s_shift[c]), e.zp,
                                                  e.qmin, e.qmax)
                          : (int32_t)requant_exact(xv, s_mult[c], s_shift[c], e.zp, e.qmin,
                                                   e.qmax);
          }
        }
        if (has_lut) {
#pragma unroll
          for (int j = 0; j < 16; ++j) q[j] = t_lut[q[j]];
        }
        store_pixel16(q, out_p + m * out_stride + c0, p.vec_out && nval == 16, nval);
      }
    }
    ptx::tc_fence_before();
    __syncthreads();  // TMEM and the A blocks are rewritten by the next tile
    if (*s_abort) break;
  }
  // after an abort, wait (bounded) for the patch loads and the MMAs still in
  // flight before the CTA's shared memory and TMEM are released
  if (tid == 0 && *s_abort) {
    for (int kk = k; kk < issued; ++kk)
      ptx::mbar_wait(bar0 + 8u * (kk % kInStages), (kk / kInStages) & 1, kInBudget);
    if (mmas > k) ptx::mbar_wait(mma_bar, k & 1, kInBudget);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

}  // namespace qa

// ============================================ warp-specialized stem layer ==
// The 3 x 3, stride-2, undilated input layer over three float channels (the
// YOLO stem), same arithmetic as input_conv_kernel, with the four steps of a
// tile run by separate warps that hand work to each other through mbarriers,
// so the quantization of one tile, the MMAs of the previous one and the
// epilogue of the one before overlap.  Two CTAs of 10 warps share an SM
// (two float patch stages and one A buffer each): the roles are latency-
// bound, and two independent pipelines per SM cover each other's waits
// (one CTA of 20 warps, three stages and two A buffers ran 12% slower):
//   warp 0     lane 0 keeps kStemStages float patches in flight by TMA;
//   warp 1     allocates TMEM; lane 0 issues the tile's MMAs (four 128-row
//              blocks, two K-steps) into one of two accumulator sets;
//   warps 2-5  quantize the patch four box columns at a time (16-byte reads
//              of each channel row) into 4-channel words, then write the
//              tile's 448 implicit-GEMM rows (nine words at fixed offsets)
//              into the A buffer;
//   warps 6-9  drain the finished accumulator set through the epilogue, one
//              per TMEM lane quarter.
namespace qa {
namespace {
constexpr int kStemC = 3;           // float channels of the stem form
constexpr int kStemStages = 2;      // float patches in flight
constexpr int kStemASets = 1;       // A buffers
constexpr int kStemCtas = 2;        // CTAs per SM
constexpr int kStemBuildWarp0 = 2, kStemBuildThreads = 128;
constexpr int kStemEpiWarp0 = 6, kStemEpiWarps = 4;  // one per TMEM lane quarter
constexpr int kStemThreads = (kStemEpiWarp0 + kStemEpiWarps) * 32;
constexpr int kStemBarBuild = 1;    // named barrier of the builder warps
constexpr int kStemTimeout = 0x7004;

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Named barrier whose result (OR of every participant's `pred`) is the same
// for all participants.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
}  // namespace

__global__ void __launch_bounds__(kStemThreads, kStemCtas)
    stem_conv_kernel(const __grid_constant__ InputConvParams p,
                     const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ uint8_t in_smem_raw[];
  const uint32_t raw = ptx::smem_addr(in_smem_raw);
  uint8_t* sm = in_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int CoutP = p.CoutP, taps = p.KH * p.KW;
  const float* s_x = reinterpret_cast<const float*>(sm);
  uint8_t* s_a = sm + kStemStages * p.stage_bytes;      // kStemASets x 4 A blocks
  uint8_t* s_b = s_a + kStemASets * 4 * kInABlock;      // CoutP rows x 64 B
  int4* s_ch = reinterpret_cast<int4*>(s_b + CoutP * 64);
  int64_t* s_bias = reinterpret_cast<int64_t*>(s_ch + CoutP);
  int64_t* s_mult = s_bias + CoutP;
  int64_t* s_shift = s_mult + CoutP;
  int32_t* s_tab = reinterpret_cast<int32_t*>(s_shift + CoutP);
  uint32_t* s_patch = reinterpret_cast<uint32_t*>(s_tab + kInTab);  // patch_h x box_w words
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(s_patch + p.patch_words) + 7) & ~uintptr_t(7));
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2 * kStemStages + 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  const uint32_t bar0 = ptx::smem_addr(bars);
  auto patch_full = [&](int s) { return bar0 + 8u * s; };
  auto patch_empty = [&](int s) { return bar0 + 8u * (kStemStages + s); };
  auto a_full = [&](int b) { return bar0 + 8u * (2 * kStemStages + b); };
  auto a_empty = [&](int b) { return bar0 + 8u * (2 * kStemStages + 2 + b); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * kStemStages + 4 + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * kStemStages + 6 + b); };
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const FusedEpilogue& e = p.epi;
  const uint32_t b_lbo = (uint32_t)(CoutP / 8) * 128u;
  const bool has_zp_fold = e.zp > -(1 << 20) && e.zp < (1 << 20);

  // ---- prologue (static operands; overlaps the previous kernel)
  int hi_ok = 1, fold_ok = 1;
  for (int i = tid; i < CoutP * 4; i += kStemThreads) {
    const int co = i / 4, j = i % 4;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (co < p.Cout) {
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int tap = 4 * j + q;
        wv[q] = tap < taps ? *reinterpret_cast<const uint32_t*>(p.w + co * p.w_kp + tap * 4) : 0u;
      }
      v = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    *reinterpret_cast<uint4*>(s_b + j * b_lbo + (co / 8) * 128 + (co % 8) * 16) = v;
  }
  for (int c = tid; c < CoutP; c += kStemThreads) {
    const bool v = c < p.Cout;
    s_bias[c] = (v && e.bias) ? e.bias[c] : 0;
    s_mult[c] = v ? e.mult[c] : 0;
    s_shift[c] = v ? e.shift[c] : 0;
    const int ts = (int)(31 + s_shift[c]);
    const bool hi = ts >= 33 && ts <= 62;
    if (v && !hi) hi_ok = 0;
    const int sh = hi ? ts - 32 : 1;
    // the zero point joins the rounding term while the sum stays in int32
    // (|hi32((acc + b) * M0)| < 2^30)
    const int64_t z = (int64_t)1 << (sh - 1);
    const int64_t zz = has_zp_fold ? e.zp * ((int64_t)1 << sh) : 0;
    if (zz + z >= ((int64_t)1 << 30) || zz + z < -((int64_t)1 << 30)) fold_ok = 0;
    s_ch[c] = make_int4((int32_t)s_bias[c], (int32_t)s_mult[c], (int32_t)(uint32_t)(z + zz), sh);
  }
  if (e.lut)
    for (int i = tid; i < kInTab; i += kStemThreads) {
      const int64_t idx = min(max((int64_t)(i - 128) - e.lut_offset, (int64_t)0), e.lut_len - 1);
      s_tab[i] = (int32_t)min(max((int64_t)e.lut[idx], (int64_t)-128), (int64_t)255);
    }
  // K bytes 36 .. 63 of every A row stay zero: written once
  for (int P = tid; P < kStemASets * 512; P += kStemThreads) {
    uint8_t* row = s_a + (P / 128) * kInABlock + ((P % 128) / 8) * 128 + (P % 8) * 16;
    *reinterpret_cast<uint4*>(row + 2 * 2048) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(row + 3 * 2048) = make_uint4(0, 0, 0, 0);
  }
  ptx::fence_proxy_async_smem();  // B and the zero K bytes are read by the tensor cores
  if (tid == 0) {
    for (int s = 0; s < kStemStages; ++s) {
      ptx::mbar_init(patch_full(s), 1);
      ptx::mbar_init(patch_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(a_full(b), 1);
      ptx::mbar_init(a_empty(b), 1);
      ptx::mbar_init(acc_full(b), 1);
      ptx::mbar_init(acc_empty(b), kStemEpiWarps);  // one arrival per epilogue warp
    }
    *s_abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&xmap);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(s_tmem), (uint32_t)p.tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  const int hi_all = __syncthreads_and(hi_ok);
  const int fold_all = __syncthreads_and(fold_ok);
  ptx::tc_fence_after();
  const uint32_t tmem = *s_tmem;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();

  const int my_tiles = p.tiles > (int)blockIdx.x
                           ? (p.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                           : 0;
  const uint32_t set_cols = (uint32_t)(4 * CoutP);
  // bounded wait; false (and the abort flag set) on expiry or after an abort
  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (ptx::mbar_wait(bar, parity, kInBudget)) return true;
    *s_abort = 1;
    if (p.status) atomicExch(p.status, kStemTimeout);
    return false;
  };
  auto tile_origin = [&](int k, int& img, int& oy0, int& ox0) {
    const int t = blockIdx.x + k * gridDim.x;
    img = t / (p.tiles_x * p.tiles_y);
    const int r = t - img * p.tiles_x * p.tiles_y;
    oy0 = (r / p.tiles_x) * kInTileH;
    ox0 = (r % p.tiles_x) * kInTileW;
  };

  int issued = 0;     // producer: tiles whose patch load was issued
  int committed = 0;  // MMA issuer: tiles whose MMAs were committed
  if (warp == 0) {
    // ---------------------------------------------------- patch producer --
    if (lane == 0) {
      for (int k = 0; k < my_tiles; ++k) {
        const int s = k % kStemStages;
        if (k >= kStemStages && !wait(patch_empty(s), ((k / kStemStages) - 1) & 1)) break;
        int img, oy0, ox0;
        tile_origin(k, img, oy0, ox0);
        ptx::mbar_arrive_expect_tx(patch_full(s), (uint32_t)(kStemC * p.patch_h * p.box_w * 4));
        ptx::tma_load_4d(ptx::smem_addr(sm) + s * p.stage_bytes, &xmap, patch_full(s),
                         ox0 * p.SW - p.PW - p.shift, oy0 * p.SH - p.PH, 0, img);
        issued = k + 1;
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_i8(128, CoutP, 1, 1);
      const uint32_t b_base = ptx::smem_addr(s_b);
      for (int k = 0; k < my_tiles; ++k) {
        const int set = k & 1, aset = k % kStemASets;
        if (!wait(a_full(aset), (k / kStemASets) & 1)) break;
        if (k >= 2 && !wait(acc_empty(set), ((k >> 1) - 1) & 1)) break;
        ptx::tc_fence_after();
        const uint32_t a_base = ptx::smem_addr(s_a) + aset * 4 * kInABlock;
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            ptx::mma_i8(tmem + set * set_cols + (uint32_t)(b * CoutP),
                        ptx::smem_desc_kmajor_plain(a_base + b * kInABlock + kk * 4096, 2048, 128),
                        ptx::smem_desc_kmajor_plain(b_base + kk * 2 * b_lbo, b_lbo, 128), idesc,
                        kk > 0 ? 1u : 0u);
        ptx::mma_commit(a_empty(aset));
        ptx::mma_commit(acc_full(set));
        committed = k + 1;
      }
    }
  } else if (warp < kStemEpiWarp0) {
    // ------------------------------------------ quantizer / row builders --
    const int bt = tid - kStemBuildWarp0 * 32;
    // the quantizer constants in registers (through a reference to the
    // parameter block every read would be a long-latency generic load)
    const QuantK qk = p.qk;
    const uint32_t in_zp = (uint32_t)qk.zp_i & 0xFFu;
    const int plane = p.patch_h * p.box_w;
    const int groups = p.patch_h * (p.box_w / 4);
    const int bw = p.box_w;
    for (int k = 0; k < my_tiles; ++k) {
      const int s = k % kStemStages, set = k % kStemASets;
      const bool got = wait(patch_full(s), (k / kStemStages) & 1);
      if (named_bar_or(kStemBarBuild, kStemBuildThreads, !got)) break;
      // (1) quantize the box: four columns of the three channel rows per step
      const float* xs = s_x + s * (p.stage_bytes / 4);
      for (int g = bt; g < groups; g += kStemBuildThreads) {
        const int off = 4 * g;  // box rows hold box_w floats: groups never straddle them
        float4 f[kStemC];
#pragma unroll
        for (int c = 0; c < kStemC; ++c)
          f[c] = *reinterpret_cast<const float4*>(xs + c * plane + off);
        // per-element exactness flags: an element within 2^-13 of a
        // rounding tie (about one in 4096) is decided on its own
        // (quantize_byte_near_tie)
        bool ok[kStemC][4];
        uint32_t t[kStemC][4];
#pragma unroll
        for (int c = 0; c < kStemC; ++c) {
          const float fv[4] = {f[c].x, f[c].y, f[c].z, f[c].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            ok[c][u] = true;
            t[c][u] = quantize_bits_fma(fv[u], qk, ok[c][u]);
          }
        }
        bool all_ok = true;
#pragma unroll
        for (int c = 0; c < kStemC; ++c)
#pragma unroll
          for (int u = 0; u < 4; ++u) all_ok = all_ok & ok[c][u];
        if (!all_ok) {
#pragma unroll
          for (int c = 0; c < kStemC; ++c) {
            const float fv[4] = {f[c].x, f[c].y, f[c].z, f[c].w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (!ok[c][u]) t[c][u] = quantize_byte_near_tie(fv[u], p.qk);
          }
        }
        uint4 w;
        w.x = pack_bytes(t[0][0], t[1][0], t[2][0], in_zp);
        w.y = pack_bytes(t[0][1], t[1][1], t[2][1], in_zp);
        w.z = pack_bytes(t[0][2], t[1][2], t[2][2], in_zp);
        w.w = pack_bytes(t[0][3], t[1][3], t[2][3], in_zp);
        *reinterpret_cast<uint4*>(s_patch + off) = w;
      }
      named_bar_sync(kStemBarBuild, kStemBuildThreads);
      if (bt == 0) ptx::mbar_arrive(patch_empty(s));  // the stage may be refilled
      const bool freed = k < kStemASets || wait(a_empty(set), ((k / kStemASets) - 1) & 1);
      if (named_bar_or(kStemBarBuild, kStemBuildThreads, !freed)) break;
      // (2) the implicit-GEMM rows of the tile: pixel P is row P % 128 of
      // block P / 128; K chunk j holds taps 4j .. 4j + 3
      uint8_t* a_set = s_a + set * 4 * kInABlock;
      for (int P = bt; P < kInPix; P += kStemBuildThreads) {
        const int py = P / kInTileW, px = P - (P / kInTileW) * kInTileW;
        uint8_t* row = a_set + (P / 128) * kInABlock + ((P % 128) / 8) * 128 + (P % 8) * 16;
        // box word of tap (ky, kx): (2 py + ky) * box_w + 2 px + kx + shift
        const uint32_t* pw = s_patch + 2 * py * bw + 2 * px + p.shift;
        uint32_t tw[9];
#pragma unroll
        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) tw[3 * ky + kx] = pw[ky * bw + kx];
        *reinterpret_cast<uint4*>(row) = make_uint4(tw[0], tw[1], tw[2], tw[3]);
        *reinterpret_cast<uint4*>(row + 2048) = make_uint4(tw[4], tw[5], tw[6], tw[7]);
        *reinterpret_cast<uint32_t*>(row + 2 * 2048) = tw[8];
      }
      ptx::fence_proxy_async_smem();
      named_bar_sync(kStemBarBuild, kStemBuildThreads);
      if (bt == 0) ptx::mbar_arrive(a_full(set));
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int ew = warp - kStemEpiWarp0;
    const int quarter = warp & 3;  // TMEM lane quarter of this warp
    const bool hi_rq = p.fast && hi_all && has_zp_fold;
    const bool zfold = hi_rq && fold_all;
    const int32_t zp32 = (int32_t)e.zp, qmin32 = (int32_t)e.qmin, qmax32 = (int32_t)e.qmax;
    const int32_t* t_lut = s_tab + 128;
    const bool has_lut = e.lut != nullptr;
    uint8_t* const out_p = e.out;
    const int64_t out_stride = e.out_pix_stride;
    for (int k = 0; k < my_tiles; ++k) {
      const int set = k & 1;
      const bool got = wait(acc_full(set), (k >> 1) & 1);
      if (!__all_sync(0xffffffffu, got)) break;
      ptx::tc_fence_after();
      int img, oy0, ox0;
      tile_origin(k, img, oy0, ox0);
      // 128-row blocks ew / 4, ew / 4 + kStemEpiWarps / 4, ...
#pragma unroll 1
      for (int b = ew >> 2; b < 4; b += kStemEpiWarps / 4) {
        const int P = b * 128 + quarter * 32 + lane;
        const int oy = oy0 + P / kInTileW, ox = ox0 + P % kInTileW;
        const bool valid = P < kInPix && oy < p.OH && ox < p.OW;
        const int64_t m = ((int64_t)img * p.OH + oy) * p.OW + ox;
        // (warp-uniform: a quarter of block 3 past the 448 rows has no live row)
        const bool live = __any_sync(0xffffffffu, valid);
#pragma unroll 1
        for (int c0 = 0; live && c0 < CoutP; c0 += 16) {
          uint32_t v[16];
          ptx::tmem_ld16(tmem + (((uint32_t)quarter * 32u) << 16) + set * set_cols +
                             (uint32_t)(b * CoutP + c0),
                         v);
          ptx::tmem_ld_wait(v);
          const int nval = min(16, p.Cout - c0);
          if (!valid || nval <= 0) continue;
          int32_t q[16];
          if (zfold) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int4 ch = s_ch[c0 + j];
              const int32_t rq = (__mulhi((int32_t)v[j] + ch.x, ch.y) + ch.z) >> ch.w;
              q[j] = min(max(rq, qmin32), qmax32);
            }
          } else if (hi_rq) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int4 ch = s_ch[c0 + j];
              // the plain rounding term (modulo 2^32: it fits int32)
              const int32_t z = (int32_t)((uint32_t)ch.z - (uint32_t)zp32 * (1u << ch.w));
              const int32_t rq = (__mulhi((int32_t)v[j] + ch.x, ch.y) + z) >> ch.w;
              q[j] = min(max(rq + zp32, qmin32), qmax32);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int c = c0 + j;
              const int64_t xv = (int64_t)(int32_t)v[j] + s_bias[c];
              q[j] = p.fast ? (int32_t)requant_fast(xv, s_mult[c], (int)(31 + s_shift[c]), e.zp,
                                                    e.qmin, e.qmax)
                            : (int32_t)requant_exact(xv, s_mult[c], s_shift[c], e.zp, e.qmin,
                                                     e.qmax);
            }
          }
          if (has_lut) {
#pragma unroll
            for (int j = 0; j < 16; ++j) q[j] = t_lut[q[j]];
          }
          store_pixel16(q, out_p + m * out_stride + c0, p.vec_out && nval == 16, nval);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(acc_empty(set));
    }
  }
  // every role has left its loop; after an abort, the last patch load of
  // every stage and the last committed MMAs complete before the CTA releases
  // its shared memory and TMEM
  __syncthreads();
  if (tid == 0 && *s_abort)
    for (int k = max(0, issued - kStemStages); k < issued; ++k)
      ptx::mbar_wait(patch_full(k % kStemStages), (k / kStemStages) & 1, kInBudget);
  if (tid == 32 && *s_abort && committed > 0)
    ptx::mbar_wait(acc_full((committed - 1) & 1), ((committed - 1) >> 1) & 1, kInBudget);
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

}  // namespace qa

QA_API int qa_conv_input_fused_dev(const qa_fused_conv_desc* d, const float* x, int64_t c_in,
                                   double scale, int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (!d || !x || d->C != 4 || c_in < 1 || c_in > 4 || d->groups != 1 || !d->x_signed ||
      d->Cout > kInMaxCout || d->KH * d->KW > kInMaxTaps || d->w_kp < d->KH * d->KW * 4 ||
      !d->out || d->res || d->out2 || d->gap_sum ||
      !d->mult || !d->shift || scale == 0.0) {
    set_error(kBadArgument, "qa_conv_input_fused_dev: unsupported layer");
    return last_status();
  }
  if (!byte_range_host(d->qmin, d->qmax)) {
    set_error(kUnsupported, "qa_conv_input_fused_dev: output range must be 8-bit");
    return last_status();
  }
  InputConvParams p;
  std::memset(&p, 0, sizeof(p));
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
  p.CoutP = (p.Cout + 15) / 16 * 16;
  p.patch_h = (kInTileH - 1) * p.SH + (p.KH - 1) * p.DH + 1;
  p.patch_w = (kInTileW - 1) * p.SW + (p.KW - 1) * p.DW + 1;
  // exact for i * patch_w < 2^32 (i < patch_h * patch_w < 2^16 here)
  p.pw_magic = (uint32_t)(((uint64_t)1 << 32) / (uint64_t)p.patch_w + 1);
  // every tile's first input column is ox0 * SW - PW with ox0 a multiple of
  // 28 (so of 4): the same residue mod 4, so one shift aligns every box start
  // to 16 B
  p.shift = (int32_t)(((-(d->PW)) % 4 + 4) % 4);
  p.box_w = (p.patch_w + p.shift + 3) / 4 * 4;
  p.stage_bytes = (p.C * p.patch_h * p.box_w * 4 + 1023) / 1024 * 1024;
  p.tiles_x = (p.OW + kInTileW - 1) / kInTileW;
  p.tiles_y = (p.OH + kInTileH - 1) / kInTileH;
  const int64_t tiles = d->N * (int64_t)p.tiles_x * p.tiles_y;
  p.tiles = (int32_t)tiles;
  p.qk = make_quant_k(scale, d->x_zp, qmin, qmax);
  {
    int cols = 32;
    while (cols < 4 * p.CoutP) cols *= 2;
    p.tmem_cols = cols;
  }
  p.w = static_cast<const int8_t*>(d->w);
  p.w_kp = d->w_kp;
  p.fast = d->fast ? 1 : 0;
  p.vec_out = (reinterpret_cast<uintptr_t>(d->out) & 15) == 0 && d->out_pix_stride % 16 == 0;
  p.status = device_status_word();
  fill_fused_epilogue(p.epi, *d);
  if (tiles == 0) return 0;
  const size_t smem = 1024 + (size_t)kInStages * p.stage_bytes + 4 * kInABlock +
                      (size_t)p.CoutP * 64 + (size_t)p.CoutP * (16 + 3 * 8) + kInTab * 4 +
                      (size_t)kInMaxTaps * 4 + (size_t)p.patch_h * p.patch_w * 4 + 8 +
                      (kInStages + 1) * 8 + 16;
  // zero padding in float must quantize to the zero point, and the box must
  // fit the TMA limits
  if (tiles > 0x7FFFFFFF || smem > 110 * 1024 || p.box_w > 256 || p.patch_h > 256 ||
      (int64_t)p.patch_h * p.patch_w >= 65536 ||
      d->W % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15)) {
    set_error(kUnsupported, "qa_conv_input_fused_dev: layer geometry outside the kernel's limits");
    return last_status();
  }
  CUtensorMap xmap;
  const uint64_t dims[4] = {(uint64_t)d->W, (uint64_t)d->H, (uint64_t)c_in, (uint64_t)d->N};
  const uint64_t strides[3] = {(uint64_t)d->W * 4, (uint64_t)(d->W * d->H) * 4,
                               (uint64_t)(d->W * d->H * c_in) * 4};
  const uint32_t box[4] = {(uint32_t)p.box_w, (uint32_t)p.patch_h, (uint32_t)c_in, 1u};
  int dev = 0;
  cudaGetDevice(&dev);
  // the stem form (3 x 3, stride 2, undilated, three float channels) runs
  // on the warp-specialized kernel: two CTAs per SM, each with two patch
  // stages, one A buffer and two accumulator sets
  const bool stem = p.KH == 3 && p.KW == 3 && p.SH == 2 && p.SW == 2 && p.DH == 1 &&
                    p.DW == 1 && c_in == kStemC;
  if (stem) {
    p.patch_words = p.patch_h * p.box_w;
    int cols = 32;
    while (cols < 8 * p.CoutP) cols *= 2;
    p.tmem_cols = cols;
    const size_t ssmem = 1024 + (size_t)kStemStages * p.stage_bytes + kStemASets * 4 * kInABlock +
                         (size_t)p.CoutP * (64 + 16 + 3 * 8) + kInTab * 4 +
                         (size_t)p.patch_words * 4 + 8 + (2 * kStemStages + 8) * 8 + 16;
    if (ssmem > 220 * 1024 / kStemCtas || p.tmem_cols * kStemCtas > 512) {
      set_error(kUnsupported, "qa_conv_input_fused_dev: stem layer outside the kernel's limits");
      return last_status();
    }
    if (!encode_tiled_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, dims, strides, box))
      return last_status();
    static size_t stem_attr[64] = {};
    if (dev < 0 || dev >= 64 || stem_attr[dev] < ssmem) {
      if (cuda_failed(cudaFuncSetAttribute(stem_conv_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)ssmem),
                      "cudaFuncSetAttribute(stem_conv)"))
        return last_status();
      if (dev >= 0 && dev < 64) stem_attr[dev] = ssmem;
    }
    const int64_t grid = std::min<int64_t>(tiles, (int64_t)kStemCtas * sm_count());
    return launch_ex(stem_conv_kernel, dim3((unsigned)grid), dim3(kStemThreads), ssmem,
                     (cudaStream_t)stream, true, p, xmap)
               ? 0
               : last_status();
  }
  p.patch_words = p.patch_h * p.patch_w;
  if (!encode_tiled_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, dims, strides, box))
    return last_status();
  static size_t attr_bytes[64] = {};
  if (dev < 0 || dev >= 64 || attr_bytes[dev] < smem) {
    if (cuda_failed(cudaFuncSetAttribute(input_conv_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "cudaFuncSetAttribute(input_conv)"))
      return last_status();
    if (dev >= 0 && dev < 64) attr_bytes[dev] = smem;
  }
  const int64_t grid = std::min<int64_t>(tiles, (int64_t)sm_count() * 2);
  return launch_ex(input_conv_kernel, dim3((unsigned)grid), dim3(kInThreads), smem,
                   (cudaStream_t)stream, true, p, xmap)
             ? 0
             : last_status();
}

QA_API int qa_mul_bytes_dev(const void* a, int64_t a_stride, int64_t a_signed, const void* b,
                            int64_t b_stride, int64_t b_signed, void* y, int64_t y_stride,
                            int64_t rows, int64_t C, int64_t za, int64_t zb, int64_t m,
                            int64_t s, int64_t zo, int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  if (C % 16 == 0 && vec16_ok(a, a_stride) && vec16_ok(b, b_stride) && vec16_ok(y, y_stride))
    return launch_ex(mul_bytes16_kernel, dim3(grid_for(rows * C / 16, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true,
                     ByteView{static_cast<const uint8_t*>(a), a_stride, (int)a_signed},
                     ByteView{static_cast<const uint8_t*>(b), b_stride, (int)b_signed},
                     static_cast<uint8_t*>(y), y_stride, rows, C / 16, za, zb, m, s, zo, qmin,
                     qmax)
               ? 0
               : last_status();
  return launch_ex(mul_bytes_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   ByteView{static_cast<const uint8_t*>(a), a_stride, (int)a_signed},
                   ByteView{static_cast<const uint8_t*>(b), b_stride, (int)b_signed},
                   static_cast<uint8_t*>(y), y_stride, rows, C, za, zb, m, s, zo, qmin, qmax)
             ? 0
             : last_status();
}

QA_API int qa_bn_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                           int64_t y_stride, int64_t rows, int64_t C, int64_t zp_in,
                           const int64_t* mult, const int64_t* shift, const int64_t* post,
                           int64_t zp_out, int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  if (!mult || !shift || !post) {
    set_error(kBadArgument, "qa_bn_bytes_dev: null parameter array");
    return last_status();
  }
  return launch_ex(bn_bytes_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   ByteView{static_cast<const uint8_t*>(x), x_stride, (int)x_signed},
                   static_cast<uint8_t*>(y), y_stride, rows, C, zp_in, mult, shift, post, zp_out,
                   qmin, qmax)
             ? 0
             : last_status();
}
