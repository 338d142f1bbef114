// Device-resident kernels of the transformer (ViT) graphs: the float
// fallbacks the reference runs as dequantize -> float op -> quantize
// (LayerNormalization, activation x activation MatMul, Softmax), fused
// where one feeds the next, and the exact integer tables of the token
// embedding.  Activations are byte rows [rows, features] (row stride in
// bytes); every kernel enqueues on the caller's stream and returns a status.
//
// Float semantics follow the reference (quant_layers.py:195-205,
// float_ops.py:336-347 / 380-385, qa_kernels.cpp:363-386):
//   dequantize: x = (float)((double)(q - zp) * scale)
//   quantize:   q = clamp(rint((double)x / scale) + zp, qmin, qmax)
// and the float ops in float64 where the reference computes in float64.
// Sums run in a different order than NumPy's, so a result can differ from
// the reference's by one output step when it lies on a rounding boundary.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/qa_kernels.h"
#include "qa_common.cuh"
#include "qa_ptx.cuh"
#include "qa_quant.cuh"

namespace qa {
namespace {

__device__ __forceinline__ int32_t load_q(const uint8_t* p, int is_signed) {
  return is_signed ? (int32_t)(int8_t)*p : (int32_t)*p;
}

__device__ __forceinline__ float dequant(int32_t q, int64_t zp, double scale) {
  return (float)((double)((int64_t)q - zp) * scale);
}


// Four-byte dot product with each operand's bytes signed or unsigned.
__device__ __forceinline__ int32_t dp4a_any(uint32_t a, uint32_t b, int32_t c, int a_signed,
                                            int b_signed) {
  int32_t d;
  if (a_signed && b_signed)
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else if (a_signed)
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else if (b_signed)
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ------------------------------------------------------ token embedding --
// out[n, 0, :] = cls_row; out[n, t, d] = clamp(ta[x[n, t-1, d]] + pos[t, d])
// for t >= 1 (x's byte value indexes `ta` as value + 128).  `ta` is the
// concat rescale of x composed with the Add's first term, `pos` the Add's
// second term plus the output zero point: exact integer tables built on
// the host with the reference's own integer functions.
__global__ void vit_embed_kernel(const uint8_t* __restrict__ x, int64_t x_stride, int x_signed,
                                 const int32_t* __restrict__ ta, const int32_t* __restrict__ pos,
                                 const uint8_t* __restrict__ cls_row, int64_t qmin, int64_t qmax,
                                 uint8_t* __restrict__ out, int64_t out_stride, int64_t B,
                                 int64_t T, int64_t D) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = B * T * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / D, d = i - row * D;
    const int64_t n = row / T, t = row - n * T;
    uint8_t v;
    if (t == 0) {
      v = cls_row[d];
    } else {
      const int32_t a = load_q(x + (n * (T - 1) + t - 1) * x_stride + d, x_signed);
      int64_t s = (int64_t)ta[a + 128] + pos[t * D + d];
      s = s < qmin ? qmin : (s > qmax ? qmax : s);
      v = (uint8_t)s;
    }
    out[row * out_stride + d] = v;
  }
}

// ------------------------------------------------------------ LayerNorm --
// One warp per row: float64 mean and variance of the dequantized row,
// (x - mean) / sqrt(var + eps) * gamma + beta in float64, rounded to float32,
// then quantized.  Rows of up to 32 * kLnCache features stay in registers.
constexpr int kLnCache = 32;

__global__ void layernorm_kernel(const uint8_t* __restrict__ x, int64_t x_stride, int x_signed,
                                 int64_t zp_in, double s_in, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, double eps, QuantK o,
                                 uint8_t* __restrict__ out, int64_t out_stride, int64_t rows,
                                 int D) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool cached = D <= 32 * kLnCache;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const uint8_t* xr = x + r * x_stride;
    float v[kLnCache];
    double sum = 0.0;
    if (cached) {
#pragma unroll
      for (int j = 0; j < kLnCache; ++j) {
        const int d = lane + 32 * j;
        v[j] = d < D ? dequant(load_q(xr + d, x_signed), zp_in, s_in) : 0.f;
        sum += (double)v[j];
      }
    } else {
      for (int d = lane; d < D; d += 32) sum += (double)dequant(load_q(xr + d, x_signed), zp_in, s_in);
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o_);
    const double mean = sum / D;
    double sq = 0.0;
    if (cached) {
#pragma unroll
      for (int j = 0; j < kLnCache; ++j) {
        const double c = (double)v[j] - mean;
        if (lane + 32 * j < D) sq += c * c;
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        const double c = (double)dequant(load_q(xr + d, x_signed), zp_in, s_in) - mean;
        sq += c * c;
      }
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o_);
    // the reference divides by the deviation; one reciprocal and a product
    // differ from that quotient by at most one float64 ulp, which reaches
    // the float32 result only on a float32 rounding boundary
    const double inv = 1.0 / sqrt(sq / D + eps);
    uint8_t* orow = out + r * out_stride;
    if (cached) {
#pragma unroll
      for (int j = 0; j < kLnCache; ++j) {
        const int d = lane + 32 * j;
        if (d >= D) break;
        double y = ((double)v[j] - mean) * inv * (double)gamma[d];
        if (beta) y = y + (double)beta[d];
        orow[d] = (uint8_t)quantize_value((float)y, o);
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        double y = ((double)dequant(load_q(xr + d, x_signed), zp_in, s_in) - mean) * inv;
        y = y * (double)gamma[d];
        if (beta) y = y + (double)beta[d];
        orow[d] = (uint8_t)quantize_value((float)y, o);
      }
    }
  }
}

// ------------------------------------------------------------ attention --
// One CTA per (image, head).  q, k, v are the head's columns of the QKV
// rows (k and v at +D and +2D); all three share the QKV quantization.
//   S = quant_S(deq(q) . deq(k)^T)          (activation x activation MatMul)
//   M = mul_table[S]                          (Mul by the 1/sqrt(hd) constant)
//   P = quant_P(softmax(deq_M(M)))            (float64, along the keys)
//   O = quant_O(deq_P(P) . deq(v))            (second MatMul)
// written to out[(n * T + t) * out_stride + h * hd + d] (the head merge
// Transpose + Reshape).  The dot products are exact integer sums of the
// centred bytes; each is scaled in double and rounded to float32 like the
// reference's float32 MatMul result.
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxT = 256, kAttnMaxHd = 128;
constexpr int kAttnKeys = kAttnMaxT / 32;  // keys per lane of a score row

struct AttnParams {
  const uint8_t* qkv;
  int64_t qkv_stride;
  int qkv_signed;
  int64_t z_qkv;
  double s_qkv;
  int T, H, hd, D;
  QuantK S;                 // scores quantization
  const int32_t* mul_table; // [384]: Mul output for S byte value v at v + 128
  int64_t z_m;              // Mul output (softmax input) quantization
  double s_m;
  QuantK P;                 // softmax output quantization
  int p_signed;
  QuantK O;                 // second MatMul output quantization
  uint8_t* out;
  int64_t out_stride;
};

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnParams a) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  const int T = a.T, hd = a.hd;
  const int kw = hd / 4 + 1;      // words per padded k row (bank spread)
  const int tp = (T + 3) & ~3;    // keys padded to whole words for P . V
  int32_t* s_q = reinterpret_cast<int32_t*>(attn_smem);  // [T][hd/4] words
  int32_t* s_k = s_q + T * (hd / 4);                        // [T][kw] words
  uint8_t* s_vt = reinterpret_cast<uint8_t*>(s_k + T * kw); // [hd][tp] bytes (v transposed)
  int32_t* s_qsum = reinterpret_cast<int32_t*>(s_vt + hd * tp);  // [T]
  int32_t* s_ksum = s_qsum + T;                                   // [T]
  int32_t* s_vsum = s_ksum + T;                                   // [hd]
  uint8_t* s_p = reinterpret_cast<uint8_t*>(s_vsum + hd);         // [warps][tp] P rows
  int32_t* s_mul = reinterpret_cast<int32_t*>(s_p + (kAttnThreads / 32) * tp);  // [384]

  const int n = blockIdx.x / a.H, h = blockIdx.x - n * a.H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();

  // stage q, k, v (bytes of the head's columns) and their sums
  const uint8_t* base = a.qkv + (int64_t)n * T * a.qkv_stride + (int64_t)h * hd;
  const int wpr = hd / 4;
  for (int i = tid; i < T * wpr; i += kAttnThreads) {
    const int t = i / wpr, w = i - t * wpr;
    const uint8_t* row = base + (int64_t)t * a.qkv_stride;
    s_q[t * wpr + w] = *reinterpret_cast<const int32_t*>(row + 4 * w);
    s_k[t * kw + w] = *reinterpret_cast<const int32_t*>(row + a.D + 4 * w);
  }
  for (int i = tid; i < hd * tp; i += kAttnThreads) {
    const int d = i / tp, t = i - d * tp;
    s_vt[i] = t < T ? base[(int64_t)t * a.qkv_stride + 2 * a.D + d]
                    : (uint8_t)(int8_t)a.z_qkv;  // padding keys contribute (z - z) = 0
  }
  __syncthreads();
  for (int t = tid; t < T; t += kAttnThreads) {
    int32_t sq = 0, sk = 0;
    for (int d = 0; d < hd; ++d) {
      sq += load_q(reinterpret_cast<const uint8_t*>(s_q + t * wpr) + d, a.qkv_signed);
      sk += load_q(reinterpret_cast<const uint8_t*>(s_k + t * kw) + d, a.qkv_signed);
    }
    s_qsum[t] = sq;
    s_ksum[t] = sk;
  }
  for (int d = tid; d < hd; d += kAttnThreads) {
    int32_t sv = 0;
    for (int t = 0; t < T; ++t) sv += load_q(s_vt + d * tp + t, a.qkv_signed);
    s_vsum[d] = sv;
  }
  for (int i = tid; i < 384; i += kAttnThreads) s_mul[i] = a.mul_table[i];
  __syncthreads();

  const int64_t z = a.z_qkv;
  const double ss = a.s_qkv * a.s_qkv;
  uint8_t* prow = s_p + warp * tp;
  for (int t1 = warp; t1 < T; t1 += kAttnThreads / 32) {
    // scores of this query row, lane l taking keys l, l + 32, ...: eight
    // independent dot products per lane -> S -> Mul table -> dequantized M
    const int32_t* qr = s_q + t1 * wpr;
    int32_t acc[kAttnKeys];
#pragma unroll
    for (int j = 0; j < kAttnKeys; ++j) acc[j] = 0;
    for (int w = 0; w < wpr; ++w) {
      const uint32_t qv = (uint32_t)qr[w];
#pragma unroll
      for (int j = 0; j < kAttnKeys; ++j) {
        const int t2 = min(lane + 32 * j, T - 1);  // clamped rows are discarded below
        acc[j] = dp4a_any(qv, (uint32_t)s_k[t2 * kw + w], acc[j], a.qkv_signed, a.qkv_signed);
      }
    }
    float xm[kAttnKeys];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kAttnKeys; ++j) {
      const int t2 = lane + 32 * j;
      xm[j] = -INFINITY;
      if (t2 < T) {
        // sum (q - z)(k - z) over the head dimension
        const int64_t dot =
            (int64_t)acc[j] - z * s_ksum[t2] - z * s_qsum[t1] + (int64_t)hd * z * z;
        const int32_t sq8 = quantize_value((float)((double)dot * ss), a.S);
        xm[j] = dequant(s_mul[sq8 + 128], a.z_m, a.s_m);
        mx = fmaxf(mx, xm[j]);
      }
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o_));
    double e[kAttnKeys];
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < kAttnKeys; ++j) {
      e[j] = lane + 32 * j < T ? exp((double)xm[j] - (double)mx) : 0.0;
      sum += e[j];
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o_);
    int32_t psum = 0;
    const double rsum = 1.0 / sum;  // (e * rsum differs from e / sum by <= 1 ulp)
#pragma unroll
    for (int j = 0; j < kAttnKeys; ++j) {
      const int t2 = lane + 32 * j;
      if (t2 < T) {
        const int32_t pq = quantize_value((float)(e[j] * rsum), a.P);
        psum += pq;
        prow[t2] = (uint8_t)pq;
      } else if (t2 < tp) {
        prow[t2] = (uint8_t)a.P.zp_i;  // padding keys: P byte = its zero point
      }
    }
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o_);
    __syncwarp();
    // P . V for this row: lane handles head dimensions d = lane, lane + 32, ...
    const int32_t* pw = reinterpret_cast<const int32_t*>(prow);
    const double sp = a.P.scale * a.s_qkv;
    const int64_t zP = a.P.zp_i;
    for (int d = lane; d < hd; d += 32) {
      const int32_t* vw = reinterpret_cast<const int32_t*>(s_vt + d * tp);
      int32_t acc2 = 0;
      for (int w = 0; w < tp / 4; ++w)
        acc2 = dp4a_any((uint32_t)pw[w], (uint32_t)vw[w], acc2, a.p_signed, a.qkv_signed);
      // sum over real keys of (p - zP)(v - z): the padded keys add
      // zP * z (their v is z) to acc2, removed with the padded count
      const int64_t pad = tp - T;
      const int64_t dot = (int64_t)acc2 - pad * zP * z - z * psum - zP * s_vsum[d] +
                          (int64_t)T * zP * z;
      a.out[((int64_t)n * T + t1) * a.out_stride + (int64_t)h * hd + d] =
          (uint8_t)quantize_value((float)((double)dot * sp), a.O);
    }
    __syncwarp();
  }
}

// ------------------------------------------------- row gather + table --
// out[r, d] = table[x[(r * every + first) row, d] + 128]: a Gather of one
// token per image through the requantization it carries.
__global__ void gather_table_kernel(const uint8_t* __restrict__ x, int64_t x_stride, int x_signed,
                                    int64_t every, int64_t first, const int32_t* __restrict__ table,
                                    uint8_t* __restrict__ out, int64_t out_stride, int64_t rows,
                                    int64_t D) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / D, d = i - r * D;
    const int32_t v = load_q(x + (r * every + first) * x_stride + d, x_signed);
    out[r * out_stride + d] = (uint8_t)table[v + 128];
  }
}

// --------------------------------------------------------- dequantize --
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ x, int64_t x_stride, int x_signed,
                                    int64_t zp, double scale, int32_t* __restrict__ q_out,
                                    float* __restrict__ f_out, int64_t rows, int64_t C) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int64_t total = rows * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / C, c = i - r * C;
    const int32_t q = load_q(x + r * x_stride + c, x_signed);
    if (q_out) q_out[i] = q;
    if (f_out) f_out[i] = dequant(q, zp, scale);
  }
}

}  // namespace
}  // namespace qa

using namespace qa;

QA_API int qa_vit_embed_dev(const void* x, int64_t x_stride, int32_t x_signed,
                            const int32_t* ta, const int32_t* pos, const void* cls_row,
                            int64_t qmin, int64_t qmax, void* out, int64_t out_stride, int64_t B,
                            int64_t T, int64_t D, void* stream) {
  clear_error();
  if (!x || !ta || !pos || !cls_row || !out || B < 0 || T < 2 || D <= 0 || x_stride < D ||
      out_stride < D) {
    set_error(kBadArgument, "qa_vit_embed_dev: bad arguments");
    return last_status();
  }
  if (B == 0) return 0;
  return launch_ex(vit_embed_kernel, dim3(grid_for(B * T * D, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_stride,
                   (int)x_signed, ta, pos, static_cast<const uint8_t*>(cls_row), qmin, qmax,
                   static_cast<uint8_t*>(out), out_stride, B, T, D)
             ? 0
             : last_status();
}

QA_API int qa_layernorm_bytes_dev(const void* x, int64_t x_stride, int32_t x_signed,
                                  int64_t zp_in, double scale_in, const float* gamma,
                                  const float* beta, double eps, double scale_out, int64_t zp_out,
                                  int64_t qmin, int64_t qmax, void* out, int64_t out_stride,
                                  int64_t rows, int64_t D, void* stream) {
  clear_error();
  if (!x || !out || !gamma || rows < 0 || D <= 0 || D > (1 << 20) || x_stride < D ||
      out_stride < D || scale_out == 0.0) {
    set_error(kBadArgument, "qa_layernorm_bytes_dev: bad arguments");
    return last_status();
  }
  if (rows == 0) return 0;
  const QuantK o = make_quant_k(scale_out, zp_out, qmin, qmax);
  return launch_ex(layernorm_kernel, dim3(grid_for(rows * 32, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_stride,
                   (int)x_signed, zp_in, scale_in, gamma, beta, eps, o,
                   static_cast<uint8_t*>(out), out_stride, rows, (int)D)
             ? 0
             : last_status();
}

QA_API int qa_attention_bytes_dev(const void* qkv, int64_t qkv_stride, int32_t qkv_signed,
                                  int64_t z_qkv, double s_qkv, int64_t B, int64_t T, int64_t H,
                                  int64_t hd, const double* s_params, const int64_t* z_params,
                                  const int32_t* mul_table, int32_t p_signed, void* out,
                                  int64_t out_stride, void* stream) {
  clear_error();
  if (!qkv || !mul_table || !out || !s_params || !z_params || B < 0 || T <= 0 ||
      T > kAttnMaxT || H <= 0 || hd <= 0 || hd > kAttnMaxHd || hd % 4 ||
      qkv_stride < 3 * H * hd || out_stride < H * hd ||
      (reinterpret_cast<uintptr_t>(qkv) & 3) || qkv_stride % 4) {
    set_error(kBadArgument, "qa_attention_bytes_dev: bad arguments");
    return last_status();
  }
  if (B == 0) return 0;
  AttnParams a;
  a.qkv = static_cast<const uint8_t*>(qkv);
  a.qkv_stride = qkv_stride;
  a.qkv_signed = qkv_signed ? 1 : 0;
  a.z_qkv = z_qkv;
  a.s_qkv = s_qkv;
  a.T = (int)T;
  a.H = (int)H;
  a.hd = (int)hd;
  a.D = (int)(H * hd);
  // s_params: scale of S, Mul output, P, O; z_params: (zp, qmin, qmax) of
  // S, P, O and the Mul output zero point
  a.S = make_quant_k(s_params[0], z_params[0], z_params[1], z_params[2]);
  a.s_m = s_params[1];
  a.z_m = z_params[9];
  a.P = make_quant_k(s_params[2], z_params[3], z_params[4], z_params[5]);
  a.O = make_quant_k(s_params[3], z_params[6], z_params[7], z_params[8]);
  a.p_signed = p_signed ? 1 : 0;
  a.mul_table = mul_table;
  a.out = static_cast<uint8_t*>(out);
  a.out_stride = out_stride;
  const int tp = ((int)T + 3) & ~3;
  const int kw = (int)hd / 4 + 1;
  const size_t smem = (size_t)T * (hd / 4) * 4 + (size_t)T * kw * 4 + (size_t)hd * tp +
                      (size_t)(2 * T + hd) * 4 + (size_t)(kAttnThreads / 32) * tp + 384 * 4 + 64;
  static size_t attr_bytes[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && (dev < 0 || dev >= 64 || attr_bytes[dev] < smem)) {
    if (cuda_failed(cudaFuncSetAttribute(attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "cudaFuncSetAttribute(attention)"))
      return last_status();
    if (dev >= 0 && dev < 64) attr_bytes[dev] = smem;
  }
  const int64_t grid = B * H;
  if (grid > 0x7FFFFFFF) {
    set_error(kUnsupported, "qa_attention_bytes_dev: too many heads");
    return last_status();
  }
  return launch_ex(attention_kernel, dim3((unsigned)grid), dim3(kAttnThreads), smem,
                   (cudaStream_t)stream, true, a)
             ? 0
             : last_status();
}

QA_API int qa_gather_table_dev(const void* x, int64_t x_stride, int32_t x_signed, int64_t every,
                               int64_t first, const int32_t* table, void* out, int64_t out_stride,
                               int64_t rows, int64_t D, void* stream) {
  clear_error();
  if (!x || !table || !out || rows < 0 || D <= 0 || every <= 0 || first < 0 || x_stride < D ||
      out_stride < D) {
    set_error(kBadArgument, "qa_gather_table_dev: bad arguments");
    return last_status();
  }
  if (rows == 0) return 0;
  return launch_ex(gather_table_kernel, dim3(grid_for(rows * D, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_stride,
                   (int)x_signed, every, first, table, static_cast<uint8_t*>(out), out_stride,
                   rows, D)
             ? 0
             : last_status();
}

QA_API int qa_dequantize_rows_dev(const void* x, int64_t x_stride, int32_t x_signed, int64_t zp,
                                  double scale, int32_t* q_out, float* f_out, int64_t rows,
                                  int64_t C, void* stream) {
  clear_error();
  if (!x || (!q_out && !f_out) || rows < 0 || C <= 0 || x_stride < C) {
    set_error(kBadArgument, "qa_dequantize_rows_dev: bad arguments");
    return last_status();
  }
  if (rows == 0) return 0;
  return launch_ex(dequant_rows_kernel, dim3(grid_for(rows * C, 256)), dim3(256), 0,
                   (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_stride,
                   (int)x_signed, zp, scale, q_out, f_out, rows, C)
             ? 0
             : last_status();
}
