// Device-resident layers of 16-bit (int16) graphs other than the dense
// tensor-core contraction (qa_umma.cu, umma_conv16_fused): graph-input
// quantization into int16 planes, grouped / depthwise convolution with the
// 16-bit fused epilogue, GlobalAveragePool, the Softmax float fallback and
// the standalone scale-matching layers (LUT, Add, Concat rescale).
//
// An int16 tensor is two NHWC byte planes of one geometry: pixel p,
// channel c at base + p * pix_stride + c in the low plane (v & 0xFF) and
// `plane` bytes further in the high plane (v >> 8).  The arithmetic of each
// layer is the reference's (quant_layers.py, qa_kernels.cpp) on int64 /
// exact 128-bit values, as in the 8-bit kernels of qa_resident_ops.cu.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/qa_kernels.h"
#include "qa_common.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_fused_epilogue.cuh"
#include "qa_ptx.cuh"
#include "qa_quant.cuh"
#include "qa_umma.cuh"

namespace qa {

bool fill_fused_epilogue(FusedEpilogue& e, const qa_fused_conv_desc& d);  // qa_resident_ops.cu
bool umma_conv16_fused(const qa_fused_conv16_desc& d, cudaStream_t st);  // qa_umma.cu

namespace {

struct Planes16 {
  const uint8_t* p;  // low plane, channel 0
  int64_t plane;     // bytes to the high plane
  int64_t stride;    // bytes between pixels
};

__device__ __forceinline__ int64_t at(const Planes16& v, int64_t pix, int64_t c) {
  return plane16_value(v.p + pix * v.stride + c, v.plane);
}

// -------------------------------------------- grouped / depthwise conv ---
struct GroupedConv16Params {
  Planes16 x;
  int64_t x_zp;
  int64_t H, W, Cg, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW, Cout, Cog;
  const uint8_t* w;  // planes [w_planes][w_rows][w_kp]
  int64_t w_plane, w_kp;
  int32_t w_planes;  // 2: int16 weights; 3: 17-bit (bytes 0, 1 and a sign byte)
  int64_t M;
  FusedEpilogue epi;
};

// One thread per (pixel, output channel), channel fastest.  Exact int64
// accumulation of the raw values; out-of-image taps contribute the raw
// zero point, whose centred value is 0 (qa_kernels.cpp:124-133).
__global__ void grouped_conv16_kernel(const __grid_constant__ GroupedConv16Params p) {
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
    const int64_t img_pix = img * p.H * p.W;
    const uint8_t* wb = p.w + n * p.w_kp;
    int64_t acc = 0;
    for (int64_t ky = 0; ky < p.KH; ++ky) {
      const int64_t iy = oy * p.SH - p.PH + ky * p.DH;
      for (int64_t kx = 0; kx < p.KW; ++kx) {
        const int64_t ix = ox * p.SW - p.PW + kx * p.DW;
        const uint8_t* wt = wb + (ky * p.KW + kx) * p.Cg;
        const bool inside = iy >= 0 && iy < p.H && ix >= 0 && ix < p.W;
        const int64_t pix = img_pix + iy * p.W + ix;
        for (int64_t c = 0; c < p.Cg; ++c) {
          const int64_t wv =
              p.w_planes == 3
                  ? (int64_t)wt[c] + 256 * (int64_t)wt[c + p.w_plane] +
                        65536 * (int64_t)(int8_t)wt[c + 2 * p.w_plane]
                  : plane16_value(wt + c, p.w_plane);
          acc += wv * (inside ? at(p.x, pix, g * p.Cg + c) : p.x_zp);
        }
      }
    }
    fused_epilogue_store16(p.epi, acc, m, (int)n);
  }
}

bool grouped_conv16(const qa_fused_conv16_desc& d16, cudaStream_t st) {
  const qa_fused_conv_desc& d = d16.base;
  if (d.groups <= 0 || d.Cout % d.groups || d.x_signed != 1 || !d.mult || !d.shift ||
      d.w_kp < d.KH * d.KW * d.C || d.w_rows < d.Cout || (d.res && d.res_signed != 1)) {
    set_error(kBadArgument, "qa_conv16_fused_dev: bad grouped layer");
    return false;
  }
  GroupedConv16Params p;
  p.x = Planes16{static_cast<const uint8_t*>(d.x), d16.x_plane, d.x_pix_stride};
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
  p.w = static_cast<const uint8_t*>(d.w);
  p.w_plane = d.w_rows * d.w_kp;
  p.w_kp = d.w_kp;
  p.w_planes = d16.w_planes == 3 ? 3 : 2;
  p.M = d.N * d.OH * d.OW;
  fill_fused_epilogue(p.epi, d);
  p.epi.res_plane = d16.res_plane;
  p.epi.out_plane = d16.out_plane;
  p.epi.out2_plane = d16.out2_plane;
  const int64_t total = p.M * p.Cout;
  if (total == 0) return true;
  return launch_ex(grouped_conv16_kernel, dim3(grid_for(total, 256)), dim3(256), 0, st, true, p);
}

// -------------------------------------------- graph input quantization ---
// float NCHW -> int16 planes NHWC; channels C..pix_stride-1 hold zp.  The
// reference's qa_quantize_f32 (qa_kernels.cpp:363-376):
// clamp(rint((double)x / scale) + zp, qmin, qmax).
__global__ void quantize_to_planes16_kernel(const float* __restrict__ x, uint8_t* __restrict__ y,
                                            int64_t plane, int64_t N, int64_t C, int64_t HW,
                                            int64_t pix_stride, double scale, double zp,
                                            double qmin, double qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * HW * pix_stride;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t c = i % pix_stride, t = i / pix_stride;
    const int64_t n = t / HW, pix = t - n * HW;
    double v = zp;
    if (c < C) {
      v = rint((double)x[(n * C + c) * HW + pix] / scale) + zp;
      if (v < qmin) v = qmin;
      if (qmax < v) v = qmax;
    }
    plane16_store(y + i, plane, (int64_t)(int32_t)v);
  }
}

// Four consecutive pixels per thread (pix_stride 4, C <= 4, H*W % 4 == 0):
// 16-byte reads of each channel plane, 16-byte stores of both output planes.
// Each value is rounded inside one FMA (quantize_bits16_fma); an element in
// the tie band, NaN or +-inf is decided on its own (quantize_value16_near_tie).
// kC3: three channels (an RGB image), known at compile time.
template <bool kC3>
__global__ void __launch_bounds__(256, 4)
    quantize_to_planes16_x4_kernel(const float* __restrict__ x, uint8_t* __restrict__ y,
                                   int64_t plane, int C_, int64_t HW, int64_t quads,
                                   const QuantK k) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int C = kC3 ? 3 : C_;
  const QuantK kk = k;  // the fast path's constants in registers
  const uint32_t pad = (uint32_t)kk.zp_i;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < quads; q += stride) {
    const int64_t p0 = q * 4;
    const int64_t n = p0 / HW, pix = p0 - n * HW;
    float4 v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      v[c] = c < C ? __ldg(reinterpret_cast<const float4*>(x + (n * C + c) * HW + pix))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t bits[4][4];  // [channel][pixel]: the value in the low 16 bits
    bool ok[4][4];
    bool all_ok = true;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float e[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ok[c][j] = true;
        bits[c][j] = c < C ? quantize_bits16_fma(e[j], kk, ok[c][j]) : pad;
        all_ok = all_ok & (ok[c][j] || c >= C);
      }
    }
    if (!all_ok) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float e[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c < C && !ok[c][j]) bits[c][j] = (uint32_t)quantize_value16_near_tie(e[j], k);
      }
    }
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // byte 0 (low plane) and byte 1 (high plane) of each channel's value
      lo[j] = __byte_perm(__byte_perm(bits[0][j], bits[1][j], 0x0040),
                          __byte_perm(bits[2][j], bits[3][j], 0x0040), 0x5410);
      hi[j] = __byte_perm(__byte_perm(bits[0][j], bits[1][j], 0x0051),
                          __byte_perm(bits[2][j], bits[3][j], 0x0051), 0x5410);
    }
    *reinterpret_cast<uint4*>(y + p0 * 4) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(y + plane + p0 * 4) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  }
}

// ------------------------------------------------------------------ GAP --
// y[n, c] = clamp(mbqm(sum_p(x[n,p,c]) - HW*zp_in, m, s) + zp_out)
// (quant_layers.py:569-590).  One warp per (n, c) run of 32 channels:
// lanes read consecutive channels of each pixel.
__global__ void gap16_kernel(Planes16 x, int64_t N, int64_t HW, int64_t C, int64_t zp_in,
                             int64_t m, int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax,
                             uint8_t* __restrict__ y, int64_t y_plane, int64_t y_pix_stride) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = N * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t n = i / C, c = i - n * C;
    int64_t acc = 0;
    for (int64_t p = 0; p < HW; ++p) acc += at(x, n * HW + p, c);
    acc -= HW * zp_in;
    plane16_store(y + n * y_pix_stride + c, y_plane,
                  requant_exact(acc, m, s, zp_out, qmin, qmax));
  }
}

// Warp per (image, 16-channel group), as gap16ch_kernel of the 8-bit
// kernels: lanes take pixels, 16-byte loads of both planes, int64 partial
// sums reduced by shuffles, lane c (c < 16) requantizes channel c.
__global__ void gap16_planes_kernel(Planes16 x, int64_t N, int64_t HW, int64_t C, int64_t zp_in,
                                    int64_t m, int64_t s, int64_t zp_out, int64_t qmin,
                                    int64_t qmax, uint8_t* __restrict__ y, int64_t y_plane,
                                    int64_t y_pix_stride) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t groups = C / 16;
  const int64_t warps = N * groups;
  const int64_t wstride = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < warps;
       w += wstride) {
    const int64_t n = w / groups, g = w - n * groups;
    const uint8_t* base = x.p + n * HW * x.stride + g * 16;
    int64_t acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0;
    for (int64_t p = lane; p < HW; p += 32) {
      const uint4 l = __ldg(reinterpret_cast<const uint4*>(base + p * x.stride));
      const uint4 h = __ldg(reinterpret_cast<const uint4*>(base + x.plane + p * x.stride));
      const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t lb = (lw[j >> 2] >> (8 * (j & 3))) & 0xFFu;
        const uint32_t hb = (hw[j >> 2] >> (8 * (j & 3))) & 0xFFu;
        acc[j] += (int64_t)(int16_t)(uint16_t)(lb | (hb << 8));
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    int64_t mine = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) mine = lane == j ? acc[j] : mine;
    if (lane < 16)
      plane16_store(y + n * y_pix_stride + g * 16 + lane, y_plane,
                    requant_exact(mine - HW * zp_in, m, s, zp_out, qmin, qmax));
  }
}

// Thread per (image, 16-channel group) for images of at most 256 pixels:
// every pixel's two 16-byte plane loads are independent (several pixels in
// flight per thread), the two bytes of each value become one sign-extended
// int32 in one `prmt` (selector nibbles with bit 3 set replicate the sign of
// the high byte), and the int32 sums (at most 256 * 2^15 in magnitude) are
// requantized once per channel.
__device__ __forceinline__ int32_t plane_value(uint32_t lo, uint32_t hi, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(lo), "r"(hi), "r"(sel));
  return (int32_t)r;
}

__global__ void __launch_bounds__(256)
    gap16_thread_planes_kernel(Planes16 x, int64_t N, int HW, int64_t groups, int64_t zp_in,
                               int64_t m, int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax,
                               uint8_t* __restrict__ y, int64_t y_plane, int64_t y_pix_stride,
                               int vec_out) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  // value k of a word pair: bytes (lo.k, hi.k, sign(hi.k), sign(hi.k))
  constexpr uint32_t kSel[4] = {0xCC40u, 0xDD51u, 0xEE62u, 0xFF73u};
  const int64_t total = N * groups;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / groups, g = i - n * groups;
    const uint8_t* base = x.p + n * HW * x.stride + g * 16;
    int32_t acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0;
#pragma unroll 4
    for (int p = 0; p < HW; ++p) {
      const uint4 l = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)p * x.stride));
      const uint4 h =
          __ldg(reinterpret_cast<const uint4*>(base + x.plane + (int64_t)p * x.stride));
      const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] += plane_value(lw[j >> 2], hw[j >> 2], kSel[j & 3]);
    }
    uint8_t* dst = y + n * y_pix_stride + g * 16;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t q =
          requant_exact((int64_t)acc[j] - (int64_t)HW * zp_in, m, s, zp_out, qmin, qmax);
      lo[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
      hi[j >> 2] |= (((uint32_t)q >> 8) & 0xFFu) << (8 * (j & 3));
    }
    if (vec_out) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      *reinterpret_cast<uint4*>(dst + y_plane) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        dst[j] = (uint8_t)(lo[j >> 2] >> (8 * (j & 3)));
        dst[y_plane + j] = (uint8_t)(hi[j >> 2] >> (8 * (j & 3)));
      }
    }
  }
}

// Integer Mul of two activations (qa_kernels.cpp:334-345): the product of
// two centred int16 values fits int64; the 128-bit mbqm requantizes it.
__global__ void mul16_kernel(Planes16 a, Planes16 b, uint8_t* __restrict__ y, int64_t y_plane,
                             int64_t y_stride, int64_t rows, int64_t C, int64_t za, int64_t zb,
                             int64_t m, int64_t s, int64_t zo, int64_t qmin, int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const int64_t p = (at(a, r, c) - za) * (at(b, r, c) - zb);
    plane16_store(y + r * y_stride + c, y_plane, requant_exact(p, m, s, zo, qmin, qmax));
  }
}

// Inference BatchNorm on int16 planes (quant_layers.py:405-441).
__global__ void bn16_kernel(Planes16 x, uint8_t* __restrict__ y, int64_t y_plane,
                            int64_t y_stride, int64_t rows, int64_t C, int64_t zp_in,
                            const int64_t* __restrict__ mult, const int64_t* __restrict__ shift,
                            const int64_t* __restrict__ post, int64_t zp_out, int64_t qmin,
                            int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    plane16_store(y + r * y_stride + c, y_plane,
                  requant_exact(at(x, r, c) - zp_in, __ldg(mult + c), __ldg(shift + c),
                                __ldg(post + c) + zp_out, qmin, qmax));
  }
}

// ------------------------------------------------------------- MaxPool --
// Integer MaxPool as the reference runs it through float_ops on int32
// tensors, out-of-image taps padded with qmin (quant_layers.py:647-648).
__global__ void maxpool16_kernel(Planes16 x, uint8_t* __restrict__ y, int64_t y_plane,
                                 int64_t y_stride, int64_t N, int64_t H, int64_t W, int64_t C,
                                 int64_t KH, int64_t KW, int64_t SH, int64_t SW, int64_t PH,
                                 int64_t PW, int64_t DH, int64_t DW, int64_t OH, int64_t OW,
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
                              : at(x, (n * H + iy) * W + ix, c);
        best = v > best ? v : best;
      }
    }
    plane16_store(y + pix * y_stride + c, y_plane, best);
  }
}

// -------------------------------------------------------------- Softmax --
// quant_layers.py:195-205 / float_ops.py:380-385 over int16 rows, as
// softmax_kernel of qa_resident_ops.cu.
constexpr int kSoftmaxThreads = 256;

__device__ __forceinline__ double block_reduce16(double v, bool is_max, double* sh) {
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
    softmax16_kernel(Planes16 x, int64_t C, double in_scale, int64_t in_zp, double out_scale,
                     double out_zp, double qmin, double qmax, int32_t* __restrict__ q_out,
                     float* __restrict__ y_out, double y_scale, int64_t y_zp) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  __shared__ double sh[32];
  const int64_t row = blockIdx.x;
  double mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float xf = (float)((double)(at(x, row, c) - in_zp) * in_scale);
    mx = fmax(mx, (double)xf);
  }
  mx = block_reduce16(mx, true, sh);
  double sum = 0.0;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float xf = (float)((double)(at(x, row, c) - in_zp) * in_scale);
    sum += exp((double)xf - mx);
  }
  sum = block_reduce16(sum, false, sh);
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float xf = (float)((double)(at(x, row, c) - in_zp) * in_scale);
    const float pr = (float)(exp((double)xf - mx) / sum);
    double v = rint((double)pr / out_scale) + out_zp;
    if (v < qmin) v = qmin;
    if (qmax < v) v = qmax;
    const int32_t q = (int32_t)v;
    if (q_out) q_out[row * C + c] = q;
    if (y_out) y_out[row * C + c] = (float)((double)((int64_t)q - y_zp) * y_scale);
  }
}

// ----------------------------------------------------- element-wise ----
__global__ void lut16_kernel(Planes16 x, uint8_t* __restrict__ y, int64_t y_plane,
                             int64_t y_stride, int64_t rows, int64_t C, int64_t offset,
                             const int32_t* __restrict__ lut, int64_t lut_len) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    int64_t idx = at(x, r, c) - offset;  // qa_kernels.cpp:348-358
    idx = idx < 0 ? 0 : (idx >= lut_len ? lut_len - 1 : idx);
    plane16_store(y + r * y_stride + c, y_plane, __ldg(lut + idx));
  }
}

__global__ void add16_kernel(Planes16 a, Planes16 b, uint8_t* __restrict__ y, int64_t y_plane,
                             int64_t y_stride, int64_t rows, int64_t C, int64_t za, int64_t ma,
                             int64_t sa, int64_t zb, int64_t mb, int64_t sb, int64_t sign,
                             int64_t zo, int64_t qmin, int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const I128 ta = mbqm(at(a, r, c) - za, ma, sa);  // qa_kernels.cpp:319-331
    I128 tb = mbqm(at(b, r, c) - zb, mb, sb);
    if (sign < 0) tb = neg_i128(tb);
    plane16_store(y + r * y_stride + c, y_plane,
                  clamp_i128(add_i128_i64(add_i128(ta, tb), zo), qmin, qmax));
  }
}

__global__ void rescale16_kernel(Planes16 x, uint8_t* __restrict__ y, int64_t y_plane,
                                 int64_t y_stride, int64_t rows, int64_t C, int identity,
                                 int64_t zp_in, int64_t m, int64_t s, int64_t zp_out,
                                 int64_t qmin, int64_t qmax) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const int64_t v = at(x, r, c);
    // quant_layers.py:553-559: clip on the same grid, else qa_rescale
    const int64_t q = identity ? (v < qmin ? qmin : (v > qmax ? qmax : v))
                               : requant_exact(v - zp_in, m, s, zp_out, qmin, qmax);
    plane16_store(y + r * y_stride + c, y_plane, q);
  }
}

}  // namespace
}  // namespace qa

using namespace qa;

QA_API int qa_conv16_fused_dev(const qa_fused_conv16_desc* desc, void* stream) {
  clear_error();
  if (!desc) {
    set_error(kBadArgument, "qa_conv16_fused_dev: null descriptor");
    return last_status();
  }
  const bool ok = desc->base.groups == 1 ? umma_conv16_fused(*desc, (cudaStream_t)stream)
                                         : grouped_conv16(*desc, (cudaStream_t)stream);
  return ok ? 0 : last_status();
}

QA_API int qa_quantize_to_planes16_dev(const float* x, void* y, int64_t y_plane, int64_t N,
                                       int64_t C, int64_t H, int64_t W, int64_t pix_stride,
                                       double scale, int64_t zp, int64_t qmin, int64_t qmax,
                                       void* stream) {
  clear_error();
  if (pix_stride < C || N < 0 || C <= 0 || scale == 0.0 || qmin < -32768 || qmax > 32767) {
    set_error(kBadArgument, "qa_quantize_to_planes16_dev: bad arguments");
    return last_status();
  }
  const int64_t total = N * H * W * pix_stride;
  if (total == 0) return 0;
  const int64_t HW = H * W;
  if (pix_stride == 4 && C <= 4 && HW % 4 == 0 && (y_plane & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const int64_t quads = N * HW / 4;
    return launch_ex(C == 3 ? quantize_to_planes16_x4_kernel<true>
                            : quantize_to_planes16_x4_kernel<false>,
                     dim3(grid_for(quads, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), y_plane, (int)C,
                     HW, quads, make_quant_k16(scale, zp, qmin, qmax))
               ? 0
               : last_status();
  }
  return launch_ex(quantize_to_planes16_kernel, dim3(grid_for(total, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, x, static_cast<uint8_t*>(y), y_plane, N, C,
                   H * W, pix_stride, scale, (double)zp, (double)qmin, (double)qmax)
             ? 0
             : last_status();
}

QA_API int qa_gap16_dev(const void* x, int64_t x_plane, int64_t x_pix_stride, int64_t N,
                        int64_t HW, int64_t C, int64_t zp_in, int64_t mult, int64_t shift,
                        int64_t zp_out, int64_t qmin, int64_t qmax, void* y, int64_t y_plane,
                        int64_t y_pix_stride, void* stream) {
  clear_error();
  if (N * C == 0) return 0;
  if (C % 16 == 0 && x_pix_stride % 16 == 0 && (x_plane & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && HW >= 1 && HW <= 256) {
    // one thread per (image, 16-channel group), every group in one pass
    const int64_t total = N * (C / 16);
    const int vec_out = ((reinterpret_cast<uintptr_t>(y) | (uint64_t)y_plane |
                          (uint64_t)y_pix_stride) & 15) == 0;
    return launch_ex(gap16_thread_planes_kernel,
                     dim3((unsigned)std::min<int64_t>((total + 255) / 256, 0x7FFFFFFF)),
                     dim3(256), 0, (cudaStream_t)stream, true,
                     Planes16{static_cast<const uint8_t*>(x), x_plane, x_pix_stride}, N,
                     (int)HW, C / 16, zp_in, mult, shift, zp_out, qmin, qmax,
                     static_cast<uint8_t*>(y), y_plane, y_pix_stride, vec_out)
               ? 0
               : last_status();
  }
  if (C % 16 == 0 && x_pix_stride % 16 == 0 && (x_plane & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const int64_t warps = N * (C / 16);
    return launch_ex(gap16_planes_kernel, dim3(grid_for(warps * 32, 256)), dim3(256), 0,
                     (cudaStream_t)stream, true,
                     Planes16{static_cast<const uint8_t*>(x), x_plane, x_pix_stride}, N, HW, C,
                     zp_in, mult, shift, zp_out, qmin, qmax, static_cast<uint8_t*>(y), y_plane,
                     y_pix_stride)
               ? 0
               : last_status();
  }
  return launch_ex(gap16_kernel, dim3(grid_for(N * C, 256)), dim3(256), 0, (cudaStream_t)stream,
                   true, Planes16{static_cast<const uint8_t*>(x), x_plane, x_pix_stride}, N, HW,
                   C, zp_in, mult, shift, zp_out, qmin, qmax, static_cast<uint8_t*>(y), y_plane,
                   y_pix_stride)
             ? 0
             : last_status();
}

QA_API int qa_softmax16_dev(const void* x, int64_t x_plane, int64_t x_pix_stride, int64_t N,
                            int64_t C, double in_scale, int64_t in_zp, double out_scale,
                            int64_t out_zp, int64_t qmin, int64_t qmax, int32_t* q_out,
                            float* y_out, double y_scale, int64_t y_zp, void* stream) {
  clear_error();
  if (N == 0 || C == 0) return 0;
  if (N > 0x7FFFFFFF) {
    set_error(kBadArgument, "qa_softmax16_dev: too many rows");
    return last_status();
  }
  return launch_ex(softmax16_kernel, dim3((unsigned)N), dim3(kSoftmaxThreads), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(x), x_plane, x_pix_stride}, C, in_scale,
                   in_zp, out_scale, (double)out_zp, (double)qmin, (double)qmax, q_out, y_out,
                   y_scale, y_zp)
             ? 0
             : last_status();
}

QA_API int qa_lut16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y,
                        int64_t y_plane, int64_t y_stride, int64_t rows, int64_t C,
                        int64_t offset, const int32_t* lut, int64_t lut_len, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  if (!lut || lut_len <= 0) {
    set_error(kBadArgument, "qa_lut16_dev: empty table");
    return last_status();
  }
  return launch_ex(lut16_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(x), x_plane, x_stride},
                   static_cast<uint8_t*>(y), y_plane, y_stride, rows, C, offset, lut, lut_len)
             ? 0
             : last_status();
}

QA_API int qa_add16_dev(const void* a, int64_t a_plane, int64_t a_stride, const void* b,
                        int64_t b_plane, int64_t b_stride, void* y, int64_t y_plane,
                        int64_t y_stride, int64_t rows, int64_t C, int64_t za, int64_t ma,
                        int64_t sa, int64_t zb, int64_t mb, int64_t sb, int64_t sign, int64_t zo,
                        int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  return launch_ex(add16_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(a), a_plane, a_stride},
                   Planes16{static_cast<const uint8_t*>(b), b_plane, b_stride},
                   static_cast<uint8_t*>(y), y_plane, y_stride, rows, C, za, ma, sa, zb, mb, sb,
                   sign, zo, qmin, qmax)
             ? 0
             : last_status();
}

QA_API int qa_rescale16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y,
                            int64_t y_plane, int64_t y_stride, int64_t rows, int64_t C,
                            int64_t identity, int64_t zp_in, int64_t m, int64_t s, int64_t zp_out,
                            int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  return launch_ex(rescale16_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(x), x_plane, x_stride},
                   static_cast<uint8_t*>(y), y_plane, y_stride, rows, C, (int)(identity != 0),
                   zp_in, m, s, zp_out, qmin, qmax)
             ? 0
             : last_status();
}

QA_API int qa_maxpool16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y,
                            int64_t y_plane, int64_t y_stride, int64_t N, int64_t H, int64_t W,
                            int64_t C, int64_t KH, int64_t KW, int64_t SH, int64_t SW,
                            int64_t PH, int64_t PW, int64_t DH, int64_t DW, int64_t OH,
                            int64_t OW, int64_t pad_value, void* stream) {
  clear_error();
  const int64_t total = N * OH * OW * C;
  if (total == 0) return 0;
  return launch_ex(maxpool16_kernel, dim3(grid_for(total, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(x), x_plane, x_stride},
                   static_cast<uint8_t*>(y), y_plane, y_stride, N, H, W, C, KH, KW, SH, SW, PH,
                   PW, DH, DW, OH, OW, pad_value)
             ? 0
             : last_status();
}

QA_API int qa_mul16_dev(const void* a, int64_t a_plane, int64_t a_stride, const void* b,
                        int64_t b_plane, int64_t b_stride, void* y, int64_t y_plane,
                        int64_t y_stride, int64_t rows, int64_t C, int64_t za, int64_t zb,
                        int64_t m, int64_t s, int64_t zo, int64_t qmin, int64_t qmax,
                        void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  return launch_ex(mul16_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(a), a_plane, a_stride},
                   Planes16{static_cast<const uint8_t*>(b), b_plane, b_stride},
                   static_cast<uint8_t*>(y), y_plane, y_stride, rows, C, za, zb, m, s, zo, qmin,
                   qmax)
             ? 0
             : last_status();
}

QA_API int qa_bn16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y,
                       int64_t y_plane, int64_t y_stride, int64_t rows, int64_t C,
                       int64_t zp_in, const int64_t* mult, const int64_t* shift,
                       const int64_t* post, int64_t zp_out, int64_t qmin, int64_t qmax,
                       void* stream) {
  clear_error();
  if (rows * C == 0) return 0;
  if (!mult || !shift || !post) {
    set_error(kBadArgument, "qa_bn16_dev: null parameter array");
    return last_status();
  }
  return launch_ex(bn16_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true,
                   Planes16{static_cast<const uint8_t*>(x), x_plane, x_stride},
                   static_cast<uint8_t*>(y), y_plane, y_stride, rows, C, zp_in, mult, shift,
                   post, zp_out, qmin, qmax)
             ? 0
             : last_status();
}
