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

#include <algorithm>
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

// The same with sixteen features per thread (D % 16 == 0, 16-byte aligned
// rows): one 16-byte load of x and of the output, the 384-entry term table
// in shared memory, the position terms as four 16-byte loads.
template <bool kSigned>
__global__ void __launch_bounds__(256)
    vit_embed16_kernel(const uint8_t* __restrict__ x, int64_t x_stride,
                       const int32_t* __restrict__ ta, const int32_t* __restrict__ pos,
                       const uint8_t* __restrict__ cls_row, int32_t qmin, int32_t qmax,
                       uint8_t* __restrict__ out, int64_t out_stride, int64_t B, int T, int D) {
  __shared__ int32_t s_ta[384];
  for (int i = threadIdx.x; i < 384; i += blockDim.x) s_ta[i] = ta[i];
  __syncthreads();
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int dq = D / 16;
  const int64_t total = B * T * dq;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / dq;
    const int j = (int)(i - row * dq);
    const int64_t n = row / T;
    const int t = (int)(row - n * T);
    uint4 v;
    if (t == 0) {
      v = *reinterpret_cast<const uint4*>(cls_row + 16 * j);
    } else {
      const uint4 xv = *reinterpret_cast<const uint4*>(
          x + (n * (T - 1) + t - 1) * x_stride + 16 * j);
      const int4* pp = reinterpret_cast<const int4*>(pos + (int64_t)t * D + 16 * j);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
      uint32_t ow[4];
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int4 p4 = __ldg(pp + k4);
        const int32_t pv[4] = {p4.x, p4.y, p4.z, p4.w};
        uint32_t w = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t b = (xw[k4] >> (8 * e)) & 0xFFu;
          const int32_t a = kSigned ? (int32_t)(int8_t)b : (int32_t)b;
          // int64: the two int32 terms may sum past int32
          const int64_t sum = (int64_t)s_ta[a + 128] + pv[e];
          const int32_t sv = (int32_t)(sum < qmin ? qmin : (sum > qmax ? qmax : sum));
          w |= ((uint32_t)sv & 0xFFu) << (8 * e);
        }
        ow[k4] = w;
      }
      v = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    *reinterpret_cast<uint4*>(out + row * out_stride + 16 * j) = v;
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

// Rows of D % 16 == 0 features, D <= 16 * 16 * kLnChunks, 16-byte aligned
// rows: sixteen lanes per row, each holding up to kLnChunks 16-byte chunks
// in registers.  The dequantized value of each byte comes from a float64
// table kept in 32 copies, one per lane (entry b of lane l at b * 32 + l,
// so a warp's lookups never share a bank).  The float64 row sum of those
// values is exact in any order (every value is a float32 multiple of the
// same scale and the sum spans fewer than 53 bits), so the mean is the
// reference's to the bit; the variance sum runs in another order than
// NumPy's.  With gamma all ones and beta all zeros (x * 1 + 0 == x) the
// output depends on the input byte alone, so each row builds a 256-entry
// output table over its byte range and its elements look it up; otherwise
// gamma and beta are applied per element in float64.
__device__ __forceinline__ uint32_t word_of(const uint4& v, int g) {
  return g == 0 ? v.x : g == 1 ? v.y : g == 2 ? v.z : v.w;
}

constexpr int kLnChunks = 4;
constexpr int kLnThreads = 256;
constexpr int kLnMaxD = 16 * 16 * kLnChunks;
constexpr int kLnRows = kLnThreads / 16;  // rows in flight per block

size_t layernorm_rows16_smem(int D) {
  return (size_t)256 * 32 * 8 + (size_t)2 * D * 8 + (size_t)kLnRows * 256;
}

__global__ void __launch_bounds__(kLnThreads, 2)
    layernorm_rows16_kernel(const uint8_t* __restrict__ x, int64_t x_stride, int x_signed,
                            int64_t zp_in, double s_in, const float* __restrict__ gamma,
                            const float* __restrict__ beta, double eps, QuantK o,
                            uint8_t* __restrict__ out, int64_t out_stride, int64_t rows, int D) {
  extern __shared__ __align__(16) double ln_smem[];
  double* s_v = ln_smem;            // [256][32]
  double* s_g = s_v + 256 * 32;     // [D]
  double* s_b = s_g + D;            // [D]
  uint8_t* s_out = reinterpret_cast<uint8_t*>(s_b + D);  // [kLnRows][256]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  {
    const double vb = (double)dequant(x_signed ? (int32_t)(int8_t)tid : tid, zp_in, s_in);
    double2* row = reinterpret_cast<double2*>(s_v + tid * 32);
#pragma unroll
    for (int c = 0; c < 16; ++c) row[c] = make_double2(vb, vb);
  }
  int ident = 1;
  for (int d = tid; d < D; d += kLnThreads) {
    const double g = (double)gamma[d], b = beta ? (double)beta[d] : 0.0;
    s_g[d] = g;
    s_b[d] = b;
    ident &= (g == 1.0 && b == 0.0) ? 1 : 0;
  }
  const bool affine = !__syncthreads_and(ident);
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  const int l16 = lane & 15, sub = lane >> 4;
  const int chunks = D / 16;
  const double rD = (double)D;
  const double* v_l = s_v + lane;  // this lane's copy: entry b at v_l[b * 32]
  uint8_t* tab = s_out + (warp * 2 + sub) * 256;
  for (int64_t pair = (int64_t)blockIdx.x * (kLnThreads / 32) + warp; 2 * pair < rows;
       pair += (int64_t)gridDim.x * (kLnThreads / 32)) {
    const int64_t row = 2 * pair + sub;
    const bool valid = row < rows;  // both halves of the warp run every shuffle
    uint4 c[kLnChunks];
#pragma unroll
    for (int i = 0; i < kLnChunks; ++i) {
      const int j = l16 + 16 * i;
      c[i] = (valid && j < chunks) ? *reinterpret_cast<const uint4*>(x + row * x_stride + 16 * j)
                                   : make_uint4(0u, 0u, 0u, 0u);
    }
    // pass 1: sum, and the byte range (as the bytes' integer values)
    double sum = 0.0;
    uint32_t bmin = x_signed ? 0x7F7F7F7Fu : 0xFFFFFFFFu, bmax = x_signed ? 0x80808080u : 0u;
#pragma unroll
    for (int i = 0; i < kLnChunks; ++i)
      if (l16 + 16 * i < chunks) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t w = word_of(c[i], g);
          sum += (v_l[(w & 0xFFu) * 32] + v_l[((w >> 8) & 0xFFu) * 32]) +
                 (v_l[((w >> 16) & 0xFFu) * 32] + v_l[(w >> 24) * 32]);
          if (x_signed) {
            bmin = __vmins4(bmin, w);
            bmax = __vmaxs4(bmax, w);
          } else {
            bmin = __vminu4(bmin, w);
            bmax = __vmaxu4(bmax, w);
          }
        }
      }
#pragma unroll
    for (int o_ = 8; o_ > 0; o_ >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o_);
    const double mean = sum / rD;
    double sq0 = 0.0, sq1 = 0.0;
#pragma unroll
    for (int i = 0; i < kLnChunks; ++i)
      if (l16 + 16 * i < chunks) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t w = word_of(c[i], g);
          const double a0 = v_l[(w & 0xFFu) * 32] - mean, a1 = v_l[((w >> 8) & 0xFFu) * 32] - mean;
          const double a2 = v_l[((w >> 16) & 0xFFu) * 32] - mean, a3 = v_l[(w >> 24) * 32] - mean;
          sq0 = fma(a0, a0, sq0);
          sq1 = fma(a1, a1, sq1);
          sq0 = fma(a2, a2, sq0);
          sq1 = fma(a3, a3, sq1);
        }
      }
    double sq = sq0 + sq1;
#pragma unroll
    for (int o_ = 8; o_ > 0; o_ >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o_);
    // the reference divides by the deviation; one reciprocal and a product
    // differ from that quotient by at most one float64 ulp, which reaches
    // the float32 result only on a float32 rounding boundary
    const double inv = 1.0 / sqrt(sq / rD + eps);
    uint8_t* orow = out + row * out_stride;
    if (!affine) {
      // the row's byte range [lo, hi] as integer values
      int lo, hi;
      if (x_signed) {
        lo = min(min((int)(int8_t)bmin, (int)(int8_t)(bmin >> 8)),
                 min((int)(int8_t)(bmin >> 16), (int)(int8_t)(bmin >> 24)));
        hi = max(max((int)(int8_t)bmax, (int)(int8_t)(bmax >> 8)),
                 max((int)(int8_t)(bmax >> 16), (int)(int8_t)(bmax >> 24)));
      } else {
        lo = (int)min(min(bmin & 0xFFu, (bmin >> 8) & 0xFFu), min((bmin >> 16) & 0xFFu, bmin >> 24));
        hi = (int)max(max(bmax & 0xFFu, (bmax >> 8) & 0xFFu), max((bmax >> 16) & 0xFFu, bmax >> 24));
      }
#pragma unroll
      for (int o_ = 8; o_ > 0; o_ >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o_));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o_));
      }
      for (int v = lo + l16; v <= hi; v += 16) {
        const uint32_t b = (uint32_t)v & 0xFFu;
        tab[b] = (uint8_t)quantize_value((float)((v_l[b * 32] - mean) * inv), o);
      }
      __syncwarp();
      if (valid) {
#pragma unroll
        for (int i = 0; i < kLnChunks; ++i) {
          const int j = l16 + 16 * i;
          if (j < chunks) {
            uint32_t ow[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint32_t w = word_of(c[i], g);
              ow[g] = pack_bytes(tab[w & 0xFFu], tab[(w >> 8) & 0xFFu], tab[(w >> 16) & 0xFFu],
                                 tab[w >> 24]);
            }
            *reinterpret_cast<uint4*>(orow + 16 * j) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          }
        }
      }
      __syncwarp();  // the table is rebuilt for the next row
    } else if (valid) {
#pragma unroll
      for (int i = 0; i < kLnChunks; ++i) {
        const int j = l16 + 16 * i;
        if (j < chunks) {
          uint32_t ow[4];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t w = word_of(c[i], g);
            uint32_t q[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int d = 16 * j + 4 * g + e;
              const double y = (v_l[((w >> (8 * e)) & 0xFFu) * 32] - mean) * inv * s_g[d] + s_b[d];
              q[e] = (uint32_t)quantize_value((float)y, o);
            }
            ow[g] = pack_bytes(q[0], q[1], q[2], q[3]);
          }
          *reinterpret_cast<uint4*>(orow + 16 * j) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
    }
  }
}

// ------------------------------------------------------------ attention --
// One CTA per (image, head, 128-query tile).  q, k, v are the head's columns
// of the QKV rows (k and v at +D and +2D); all three share the QKV
// quantization.
//   S = quant_S(deq(q) . deq(k)^T)          (activation x activation MatMul)
//   M = mul_table[S]                          (Mul by the 1/sqrt(hd) constant)
//   P = quant_P(softmax(deq_M(M)))            (float64, along the keys)
//   O = quant_O(deq_P(P) . deq(v))            (second MatMul)
// written to out[(n * T + t) * out_stride + h * hd + d] (the head merge
// Transpose + Reshape).  Both products run on the tensor cores over the raw
// bytes (tcgen05.mma kind::i8, M = 128 query rows, accumulators in TMEM);
// the zero points come off with row and column byte sums, so each dot
// product is the exact integer sum of the centred bytes, scaled in double
// and rounded to float32 like the reference's float32 MatMul result.
//
// Softmax: thread (row, column half) reads its scores straight from TMEM.
// The softmax input is a byte b (M's quantized value), so exp only ever sees
// 256 arguments: E[b] = exp(x(b) - x_top) with x_top the largest x over the
// byte range is a 256-entry table per CTA, and p = E[b] / sum_row E, which
// equals exp(x - max_row) / sum_row exp(x - max_row) up to the last bit of
// a double (the common factor exp(max_row - x_top) cancels).  When the byte
// range of x spans more than 600 (E would leave the normal doubles) the
// kernel takes exp(x - max_row) per element instead.
//
// Quantizing S, P and O: the reference quantizes a float32 value
// (rint((double)x / scale)); the fast path forms m = x / scale in float32
// from the integer dot product (or the table value) and one float constant,
// within 2^-14 of the reference's quotient wherever the clamp does not
// decide, and keeps it when m lies farther than 2^-12 from a half-integer;
// other elements take the double-precision definition (outlined, rare).
//
// Operand layouts (no swizzle, K-major): a 16-byte K slice of all R rows is
// one block of R * 16 bytes (row r at r * 16), so core matrices are 128
// bytes apart along M/N and R * 16 bytes apart along K.  Padded rows, keys
// and head dimensions hold raw 0 bytes and add nothing to the raw sums.
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxT = 256, kAttnMaxHd = 128;
constexpr int kAttnTile = 128;       // query rows per CTA
constexpr uint64_t kAttnBudget = 4000000000ull;  // bounded waits (~2 s)
constexpr int kAttnTimeoutCode = 0x7005;
constexpr double kAttnTableSpan = 600.0;  // largest x range the exp table covers
constexpr double kAttnFloatSpan = 80.0;   // ... and its float copy (normal floats)
constexpr float kAttnTieBand = 0.499755859375f;  // 0.5 - 2^-12

struct AttnParams {
  const uint8_t* qkv;
  int64_t qkv_stride;
  int qkv_signed;
  int32_t z_qkv;
  double s_qkv;
  int T, H, hd, D;
  int tiles;               // query tiles per head
  int hdp, hdn, nk, tk;    // hd to 32 (S K-dim), hd to 16 (O N-dim), T to 16 (S N-dim), T to 32
  int vec_in, vec_out;     // 16-byte row segments of qkv / out
  uint32_t tmem_cols;
  QuantK S;                 // scores quantization
  const int32_t* mul_table; // [384]: Mul output for S byte value v at v + 128
  int64_t z_m;              // Mul output (softmax input) quantization
  double s_m;
  QuantK P;                 // softmax output quantization
  int p_signed;
  QuantK O;                 // second MatMul output quantization
  float c_s, c_o;           // s_qkv^2 / S.scale, P.scale * s_qkv / O.scale (NaN: no fast path)
  uint8_t* out;
  int64_t out_stride;
  int* status;
};

// rint(clamp(m, lo, hi)) + zp, and whether m is far enough from a
// half-integer for that to be the reference's value (m must not be NaN).
__device__ __forceinline__ bool quant_fast(float m, const QuantK& k, int32_t& q) {
  const float mc = fminf(fmaxf(m, k.lo), k.hi);
  const float t = __fadd_rn(mc, k.magic_zp);
  const float r = __fsub_rn(t, k.magic_zp);
  q = (int32_t)(__float_as_uint(t) - 0x4B400000u);
  return fabsf(mc - r) < kAttnTieBand;
}

// The definitions the fast paths fall back to.
__device__ __noinline__ int32_t quant_dot_exact(int32_t dot, double scale2, const QuantK& k) {
  return quantize_value((float)((double)dot * scale2), k);
}
__device__ __noinline__ int32_t quant_prob_exact(double e, double rsum, const QuantK& k) {
  return quantize_value((float)(e * rsum), k);
}

// Sixteen scores of one key chunk -> their quantized S values (low byte of
// each tb word: the float bits of rint(m) + zp + 1.5 * 2^23, or the value
// itself where the exact definition decided).  One warp vote per chunk sends
// the lanes with an element near a rounding tie to the exact path.
template <bool kMagicS>
__device__ __forceinline__ void score_bytes(const uint32_t (&v)[16], const int4* kz4, int32_t rowc,
                                            float c_s, bool fast_s, double ss, const QuantK& S,
                                            uint32_t (&tb)[16]) {
  uint32_t okm = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int4 kz = kz4[g];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * g + e;
      const int32_t kze = e == 0 ? kz.x : e == 1 ? kz.y : e == 2 ? kz.z : kz.w;
      const int32_t dot = (int32_t)v[i] - kze + rowc;
      const float df = kMagicS ? __int_as_float(0x4B400000 + dot) - 12582912.0f
                               : __int2float_rn(dot);
      const float mc = fminf(fmaxf(df * c_s, S.lo), S.hi);
      const float t = __fadd_rn(mc, S.magic_zp);
      const float rr = __fsub_rn(t, S.magic_zp);
      okm |= (fabsf(mc - rr) < kAttnTieBand ? 1u : 0u) << i;
      tb[i] = __float_as_uint(t);
    }
  }
  if (!fast_s) okm = 0;
  if (__any_sync(0xffffffffu, okm != 0xFFFFu)) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int4 kz = kz4[g];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * g + e;
        if (!((okm >> i) & 1u)) {
          const int32_t kze = e == 0 ? kz.x : e == 1 ? kz.y : e == 2 ? kz.z : kz.w;
          tb[i] = (uint32_t)quant_dot_exact((int32_t)v[i] - kze + rowc, ss, S);
        }
      }
    }
  }
}

// Sixteen probabilities of one key chunk from its score bytes `bw`: the
// float bits of rint(m) + zp + 1.5 * 2^23 per element (the exact path's
// value is stored in the same form).
__device__ __forceinline__ void prob_bytes(uint4 bw, const double* s_ex, const float* s_exf,
                                           const float* s_xm, bool table, bool fast_p, float r_f,
                                           double rsum, float mx, const QuantK& P,
                                           uint32_t (&tp)[16]) {
  uint32_t okm = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t word = word_of(bw, g);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * g + e;
      const float mc = fminf(fmaxf(s_exf[(word >> (8 * e)) & 0xFFu] * r_f, P.lo), P.hi);
      const float t = __fadd_rn(mc, P.magic_zp);
      const float rr = __fsub_rn(t, P.magic_zp);
      okm |= (fabsf(mc - rr) < kAttnTieBand ? 1u : 0u) << i;
      tp[i] = __float_as_uint(t);
    }
  }
  if (!fast_p) okm = 0;
  if (__any_sync(0xffffffffu, okm != 0xFFFFu)) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t word = word_of(bw, g);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * g + e;
        if (!((okm >> i) & 1u)) {
          const uint32_t b = (word >> (8 * e)) & 0xFFu;
          const double ev = table ? s_ex[b] : exp((double)s_xm[b] - (double)mx);
          tp[i] = (uint32_t)quant_prob_exact(ev, rsum, P) + 0x4B400000u;
        }
      }
    }
  }
}

__device__ __forceinline__ int32_t byte_sum4(uint4 v, int is_signed) {
  int32_t s = 0;
  s = dp4a_any(v.x, 0x01010101u, s, is_signed, 0);
  s = dp4a_any(v.y, 0x01010101u, s, is_signed, 0);
  s = dp4a_any(v.z, 0x01010101u, s, is_signed, 0);
  return dp4a_any(v.w, 0x01010101u, s, is_signed, 0);
}

template <bool kMagicS>
__global__ void __launch_bounds__(kAttnThreads, 2)
    attention_kernel(const __grid_constant__ AttnParams a) {
  extern __shared__ __align__(128) uint8_t attn_smem[];
  const int T = a.T, hd = a.hd, hdp = a.hdp, hdn = a.hdn, nk = a.nk, tk = a.tk;
  uint8_t* s_q = attn_smem;                   // hdp / 16 slices of 128 rows
  uint8_t* s_k = s_q + kAttnTile * hdp;       // hdp / 16 slices of nk rows
  uint8_t* s_vt = s_k + nk * hdp;             // tk / 16 slices of hdn rows (v transposed)
  uint8_t* s_p = s_vt + hdn * tk;             // tk / 16 slices of 128 rows
  double* s_ex = reinterpret_cast<double*>(s_p + kAttnTile * tk);  // [264] exp table, [256] = 0
  float* s_exf = reinterpret_cast<float*>(s_ex + 264);             // [264] its float copy
  float* s_xm = s_exf + 264;                                        // [256] softmax input of b
  int32_t* s_kz = reinterpret_cast<int32_t*>(s_xm + 256);          // [256] z * sum k (per key)
  int32_t* s_qsum = s_kz + 256;                                    // [128]
  int32_t* s_vz = s_qsum + kAttnTile;                              // [128] per head dimension
  double* s_part = reinterpret_cast<double*>(s_vz + kAttnMaxHd);   // [2][128] row sums
  float* s_rmax = reinterpret_cast<float*>(s_part + 2 * kAttnTile);  // [2][128] row maxima
  int32_t* s_psum = reinterpret_cast<int32_t*>(s_rmax + 2 * kAttnTile);  // [2][128]
  float* s_red = reinterpret_cast<float*>(s_psum + 2 * kAttnTile);       // [2][8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_red + 16);              // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quarter = warp & 3, half = warp >> 2;
  const int tile = blockIdx.x % a.tiles, nh = blockIdx.x / a.tiles;
  const int n = nh / a.H, h = nh - n * a.H;
  const int row0 = tile * kAttnTile;
  const uint32_t bar_s = ptx::smem_addr(bars), bar_o = bar_s + 8u;
  const int32_t z = a.z_qkv;

  // ---- launch-constant tables (before waiting on the producer of qkv) ----
  {
    const int b = tid;  // 256 threads, one byte value each
    const int v = a.S.qmin_i < 0 ? (int)(int8_t)b : b;
    const bool in_range = v >= a.S.qmin_i && v <= a.S.qmax_i;
    const float xm = dequant(a.mul_table[v + 128], a.z_m, a.s_m);
    s_xm[b] = xm;
    float hi = in_range ? xm : -INFINITY, lo = in_range ? xm : INFINITY;
#pragma unroll
    for (int o_ = 16; o_ > 0; o_ >>= 1) {
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o_));
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o_));
    }
    if (lane == 0) {
      s_red[warp] = hi;
      s_red[8 + warp] = lo;
    }
    if (tid < 8) {
      s_ex[256 + tid] = 0.0;  // padded keys
      s_exf[256 + tid] = 0.f;
    }
  }
  if (tid == 0) {
    ptx::mbar_init(bar_s, 1);
    ptx::mbar_init(bar_o, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(ptx::smem_addr(s_tmem), a.tmem_cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *s_tmem;
  float x_top = s_red[0], x_low = s_red[8];
#pragma unroll
  for (int w = 1; w < 8; ++w) {
    x_top = fmaxf(x_top, s_red[w]);
    x_low = fminf(x_low, s_red[8 + w]);
  }
  const double span = (double)x_top - (double)x_low;
  const bool table = span <= kAttnTableSpan;
  const bool table_f = span <= kAttnFloatSpan && a.P.inv == a.P.inv;
  if (table) {
    const double e = exp((double)s_xm[tid] - (double)x_top);
    s_ex[tid] = e;
    s_exf[tid] = (float)e;
  }

  ptx::pdl_launch_dependents();
  ptx::pdl_wait();

  // ---- stage q (this tile's rows), k and v (all keys) in the MMA layouts ----
  const uint8_t* base = a.qkv + (int64_t)n * T * a.qkv_stride + (int64_t)h * hd;
  const int qs = hdp / 16;
  for (int i = tid; i < (kAttnTile + nk) * qs; i += kAttnThreads) {
    const int r = i / qs, j = i - r * qs;
    const bool is_q = r < kAttnTile;
    const int rr = is_q ? r : r - kAttnTile;
    const int t = is_q ? row0 + rr : rr;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < T) {
      const uint8_t* src = base + (int64_t)t * a.qkv_stride + (is_q ? 0 : a.D) + 16 * j;
      if (a.vec_in) {
        if (16 * j < hd) v = *reinterpret_cast<const uint4*>(src);
      } else {
        uint32_t w4[4];
#pragma unroll
        for (int w = 0; w < 4; ++w)
          w4[w] = 16 * j + 4 * w < hd ? *reinterpret_cast<const uint32_t*>(src + 4 * w) : 0u;
        v = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
    }
    uint8_t* dst = is_q ? s_q + j * (kAttnTile * 16) : s_k + j * (nk * 16);
    *reinterpret_cast<uint4*>(dst + rr * 16) = v;
  }
  const int dgs = hdn / 4;
  for (int i = tid; i < (tk / 4) * dgs; i += kAttnThreads) {
    const int kb = i / dgs, dg = i - kb * dgs;
    const int k0 = 4 * kb, d0 = 4 * dg;
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      w[q] = (k0 + q < T && d0 < hd)
                 ? *reinterpret_cast<const uint32_t*>(base + (int64_t)(k0 + q) * a.qkv_stride +
                                                      2 * a.D + d0)
                 : 0u;
    // 4 x 4 byte transpose: word j gets byte j of each key's word
    const uint32_t t0 = __byte_perm(w[0], w[1], 0x5140), t1 = __byte_perm(w[0], w[1], 0x7362);
    const uint32_t t2 = __byte_perm(w[2], w[3], 0x5140), t3 = __byte_perm(w[2], w[3], 0x7362);
    uint8_t* dst = s_vt + (k0 / 16) * (hdn * 16) + d0 * 16 + (k0 & 15);
    *reinterpret_cast<uint32_t*>(dst) = __byte_perm(t0, t2, 0x5410);
    *reinterpret_cast<uint32_t*>(dst + 16) = __byte_perm(t0, t2, 0x7632);
    *reinterpret_cast<uint32_t*>(dst + 32) = __byte_perm(t1, t3, 0x5410);
    *reinterpret_cast<uint32_t*>(dst + 48) = __byte_perm(t1, t3, 0x7632);
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();

  // ---- S = q k^T (raw bytes) on the tensor cores ----
  if (tid == 0) {
    ptx::tc_fence_after();
    const uint32_t idesc = ptx::idesc_i8(kAttnTile, nk, a.qkv_signed, a.qkv_signed);
    const uint32_t qa = ptx::smem_addr(s_q), ka = ptx::smem_addr(s_k);
    for (int kk = 0; kk < hdp / 32; ++kk)
      ptx::mma_i8(tmem,
                  ptx::smem_desc_kmajor_plain(qa + kk * 2 * (kAttnTile * 16), kAttnTile * 16, 128),
                  ptx::smem_desc_kmajor_plain(ka + kk * 2 * (nk * 16), nk * 16, 128), idesc,
                  kk > 0 ? 1u : 0u);
    ptx::mma_commit(bar_s);
  }
  // byte sums for the zero-point terms, while the MMA runs
  for (int i = tid; i < kAttnTile + nk + hdn; i += kAttnThreads) {
    if (i < kAttnTile) {
      int32_t s = 0;
      for (int j = 0; j < qs; ++j)
        s += byte_sum4(*reinterpret_cast<const uint4*>(s_q + j * (kAttnTile * 16) + i * 16),
                       a.qkv_signed);
      s_qsum[i] = s;
    } else if (i < kAttnTile + nk) {
      const int r = i - kAttnTile;
      int32_t s = 0;
      for (int j = 0; j < qs; ++j)
        s += byte_sum4(*reinterpret_cast<const uint4*>(s_k + j * (nk * 16) + r * 16),
                       a.qkv_signed);
      s_kz[r] = z * s;
    } else {
      const int d = i - kAttnTile - nk;
      int32_t s = 0;
      for (int j = 0; j < tk / 16; ++j)
        s += byte_sum4(*reinterpret_cast<const uint4*>(s_vt + j * (hdn * 16) + d * 16),
                       a.qkv_signed);
      s_vz[d] = a.P.zp_i * s - T * a.P.zp_i * z;
    }
  }
  __syncthreads();
  if (!ptx::mbar_wait(bar_s, 0, kAttnBudget)) {
    *s_abort = 1;
    if (a.status) atomicExch(a.status, kAttnTimeoutCode);
  }
  __syncthreads();
  ptx::tc_fence_after();
  const bool ok = !*s_abort;

  // ---- softmax rows: this thread owns row r, score chunks [c_beg, c_end) ----
  const int r = quarter * 32 + lane;
  const int t1 = row0 + r;
  const bool warp_live = ok && row0 + quarter * 32 < T;  // warp-uniform
  const int nchunks = nk / 16;
  const int c_split = (nchunks + 1) / 2;
  const int c_beg = half ? c_split : 0, c_end = half ? nchunks : c_split;
  const uint32_t lane_base = ((uint32_t)(quarter * 32)) << 16;
  const double ss = a.s_qkv * a.s_qkv;
  const float c_s = a.c_s;
  const bool fast_s = c_s == c_s;
  const int32_t rowc = hd * z * z - z * s_qsum[r];
  // pass 1: scores -> bytes b (kept in the P buffer at their P positions),
  // with the row's partial exp-table sum (or its maximum without the table)
  double part = 0.0;
  float mx = -INFINITY;
  if (warp_live) {
#pragma unroll 1
    for (int cc = c_beg; cc < c_end; ++cc) {
      uint32_t v[16], tb[16];
      ptx::tmem_ld16(tmem + lane_base + (uint32_t)(cc * 16), v);
      ptx::tmem_ld_wait(v);
      score_bytes<kMagicS>(v, reinterpret_cast<const int4*>(s_kz + cc * 16), rowc, c_s,
                           fast_s, ss, a.S, tb);
      const int lim = T - cc * 16;  // columns of this chunk that are real keys
      if (table) {
        if (lim >= 16) {
          double p0 = 0.0, p1 = 0.0;
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            p0 += s_ex[tb[i] & 0xFFu];
            p1 += s_ex[tb[i + 1] & 0xFFu];
          }
          part += p0 + p1;
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) part += s_ex[i < lim ? (tb[i] & 0xFFu) : 256u];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < lim) mx = fmaxf(mx, s_xm[tb[i] & 0xFFu]);
      }
      *reinterpret_cast<uint4*>(s_p + cc * (kAttnTile * 16) + r * 16) =
          make_uint4(pack_bytes(tb[0], tb[1], tb[2], tb[3]), pack_bytes(tb[4], tb[5], tb[6], tb[7]),
                     pack_bytes(tb[8], tb[9], tb[10], tb[11]),
                     pack_bytes(tb[12], tb[13], tb[14], tb[15]));
    }
  }
  if (!table) {  // CTA-uniform: the row maximum, then the sum of exp(x - max)
    s_rmax[half * kAttnTile + r] = mx;
    __syncthreads();
    mx = fmaxf(s_rmax[r], s_rmax[kAttnTile + r]);
    if (warp_live) {
#pragma unroll 1
      for (int cc = c_beg; cc < c_end; ++cc) {
        const uint4 bw = *reinterpret_cast<const uint4*>(s_p + cc * (kAttnTile * 16) + r * 16);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t word = word_of(bw, g);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (cc * 16 + 4 * g + e < T)
              part += exp((double)s_xm[(word >> (8 * e)) & 0xFFu] - (double)mx);
        }
      }
    }
  }
  s_part[half * kAttnTile + r] = part;
  __syncthreads();
  const double rsum = 1.0 / (s_part[r] + s_part[kAttnTile + r]);
  const float r_f = (float)(rsum * a.P.inv);  // P.inv: 1 / P.scale in float
  const bool fast_p = table_f && fabsf(r_f) <= 3.0e38f;
  // pass 2: P bytes over the b bytes
  int32_t psum = 0;
  if (warp_live) {
#pragma unroll 1
    for (int cc = c_beg; cc < c_end; ++cc) {
      uint4* slot = reinterpret_cast<uint4*>(s_p + cc * (kAttnTile * 16) + r * 16);
      uint32_t tp[16];
      prob_bytes(*slot, s_ex, s_exf, s_xm, table, fast_p, r_f, rsum, mx, a.P, tp);
      const int lim = T - cc * 16;
      if (lim < 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          tp[i] = i < lim ? tp[i] : 0x4B400000u;  // padded keys: value 0 (raw byte 0)
      }
      // each word is value + 0x4B400000 (low byte 0): the value's byte is the
      // word's, and the sixteen offsets cancel modulo 2^32
      uint32_t bsum = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) bsum += tp[i];
      psum += (int32_t)(bsum - 16u * 0x4B400000u);
      *slot = make_uint4(pack_bytes(tp[0], tp[1], tp[2], tp[3]),
                         pack_bytes(tp[4], tp[5], tp[6], tp[7]),
                         pack_bytes(tp[8], tp[9], tp[10], tp[11]),
                         pack_bytes(tp[12], tp[13], tp[14], tp[15]));
    }
  }
  // key slices past the score columns (tk > nk) hold zeros
  for (int cc = nchunks + half; cc < tk / 16; cc += 2)
    *reinterpret_cast<uint4*>(s_p + cc * (kAttnTile * 16) + r * 16) = make_uint4(0u, 0u, 0u, 0u);
  s_psum[half * kAttnTile + r] = psum;
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();

  // ---- O = P v (raw bytes) into the score columns ----
  if (tid == 0 && ok) {
    ptx::tc_fence_after();
    const uint32_t idesc = ptx::idesc_i8(kAttnTile, hdn, a.p_signed, a.qkv_signed);
    const uint32_t pa = ptx::smem_addr(s_p), va = ptx::smem_addr(s_vt);
    for (int kk = 0; kk < tk / 32; ++kk)
      ptx::mma_i8(tmem,
                  ptx::smem_desc_kmajor_plain(pa + kk * 2 * (kAttnTile * 16), kAttnTile * 16, 128),
                  ptx::smem_desc_kmajor_plain(va + kk * 2 * (hdn * 16), hdn * 16, 128), idesc,
                  kk > 0 ? 1u : 0u);
    ptx::mma_commit(bar_o);
  }
  if (ok && !ptx::mbar_wait(bar_o, 0, kAttnBudget)) {
    *s_abort = 1;
    if (a.status) atomicExch(a.status, kAttnTimeoutCode);
  }
  __syncthreads();
  ptx::tc_fence_after();

  // ---- epilogue: O row r, head-dimension chunks of this half ----
  if (warp_live && !*s_abort) {
    const int ochunks = hdn / 16, o_split = (ochunks + 1) / 2;
    const int o_beg = half ? o_split : 0, o_end = half ? ochunks : o_split;
    const int32_t prow = psum + s_psum[(1 - half) * kAttnTile + r];
    const int32_t rowo = z * prow;
    const double sp = a.P.scale * a.s_qkv;
    const float c_o = a.c_o;
    const bool fast_o = c_o == c_o;
    uint8_t* orow = a.out + ((int64_t)n * T + t1) * a.out_stride + (int64_t)h * hd;
#pragma unroll 1
    for (int oc = o_beg; oc < o_end; ++oc) {
      uint32_t v[16];
      ptx::tmem_ld16(tmem + lane_base + (uint32_t)(oc * 16), v);
      ptx::tmem_ld_wait(v);
      uint32_t ow[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t oq[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = oc * 16 + 4 * g + e;
          const int32_t dot = (int32_t)v[4 * g + e] - rowo - s_vz[d];
          int32_t q;
          if (!(fast_o && quant_fast(__int2float_rn(dot) * c_o, a.O, q)))
            q = quant_dot_exact(dot, sp, a.O);
          oq[e] = (uint32_t)q;
        }
        ow[g] = pack_bytes(oq[0], oq[1], oq[2], oq[3]);
      }
      if (t1 < T) {
        if (a.vec_out) {
          *reinterpret_cast<uint4*>(orow + oc * 16) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        } else {
          for (int j = 0; j < 16 && oc * 16 + j < hd; ++j)
            orow[oc * 16 + j] = (uint8_t)(ow[j >> 2] >> (8 * (j & 3)));
        }
      }
    }
  }

  // after an abort, wait (bounded) for the MMAs still in flight before the
  // CTA's shared memory and TMEM are released
  if (tid == 0 && *s_abort) {
    ptx::mbar_wait(bar_s, 0, kAttnBudget);
    if (ok) ptx::mbar_wait(bar_o, 0, kAttnBudget);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, a.tmem_cols);
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
  const bool vec = D % 16 == 0 && x_stride % 16 == 0 && out_stride % 16 == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                     reinterpret_cast<uintptr_t>(pos) | reinterpret_cast<uintptr_t>(cls_row)) &
                    15) == 0 &&
                   qmin >= -128 && qmax <= 255 && T < (1 << 30) && D < (1 << 30);
  if (vec) {
    auto kern = x_signed ? vit_embed16_kernel<true> : vit_embed16_kernel<false>;
    return launch_ex(kern, dim3(grid_for(B * T * (D / 16), 256)), dim3(256), 0,
                     (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_stride, ta,
                     pos, static_cast<const uint8_t*>(cls_row), (int32_t)qmin, (int32_t)qmax,
                     static_cast<uint8_t*>(out), out_stride, B, (int)T, (int)D)
               ? 0
               : last_status();
  }
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
  const bool rows16 = D % 16 == 0 && D <= kLnMaxD && x_stride % 16 == 0 &&
                      out_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (rows16) {
    const size_t smem = layernorm_rows16_smem((int)D);
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      if (cuda_failed(cudaFuncSetAttribute(layernorm_rows16_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)layernorm_rows16_smem(kLnMaxD)),
                      "cudaFuncSetAttribute(layernorm)"))
        return last_status();
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int64_t blocks = std::min<int64_t>((rows + 15) / 16, 2 * (int64_t)sm_count());
    return launch_ex(layernorm_rows16_kernel, dim3((unsigned)blocks), dim3(kLnThreads), smem,
                     (cudaStream_t)stream, true, static_cast<const uint8_t*>(x), x_stride,
                     (int)x_signed, zp_in, scale_in, gamma, beta, eps, o,
                     static_cast<uint8_t*>(out), out_stride, rows, (int)D)
               ? 0
               : last_status();
  }
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
  // s_params: scale of S, Mul output, P, O; z_params: (zp, qmin, qmax) of
  // S, P, O and the Mul output zero point
  const bool qkv_ok = qkv_signed ? (z_qkv >= -128 && z_qkv <= 127) : (z_qkv >= 0 && z_qkv <= 255);
  if (!qkv_ok || !byte_range_host(z_params[1], z_params[2]) ||
      !byte_range_host(z_params[4], z_params[5]) || !byte_range_host(z_params[7], z_params[8]) ||
      (p_signed != 0) != (z_params[4] < 0) || z_params[3] < z_params[4] ||
      z_params[3] > z_params[5]) {
    set_error(kUnsupported, "qa_attention_bytes_dev: quantization ranges must be 8-bit");
    return last_status();
  }
  if (B == 0) return 0;
  AttnParams a;
  a.qkv = static_cast<const uint8_t*>(qkv);
  a.qkv_stride = qkv_stride;
  a.qkv_signed = qkv_signed ? 1 : 0;
  a.z_qkv = (int32_t)z_qkv;
  a.s_qkv = s_qkv;
  a.T = (int)T;
  a.H = (int)H;
  a.hd = (int)hd;
  a.D = (int)(H * hd);
  a.tiles = (int)((T + kAttnTile - 1) / kAttnTile);
  a.hdp = (int)((hd + 31) & ~31);
  a.hdn = (int)((hd + 15) & ~15);
  a.nk = (int)((T + 15) & ~15);
  a.tk = (int)((T + 31) & ~31);
  a.vec_in = (hd % 16 == 0 && qkv_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0)
                 ? 1
                 : 0;
  a.vec_out = (hd % 16 == 0 && out_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0)
                  ? 1
                  : 0;
  uint32_t cols = 32;
  while (cols < (uint32_t)a.nk || cols < (uint32_t)a.hdn) cols <<= 1;
  a.tmem_cols = cols;
  a.S = make_quant_k(s_params[0], z_params[0], z_params[1], z_params[2]);
  a.s_m = s_params[1];
  a.z_m = z_params[9];
  a.P = make_quant_k(s_params[2], z_params[3], z_params[4], z_params[5]);
  a.O = make_quant_k(s_params[3], z_params[6], z_params[7], z_params[8]);
  a.p_signed = p_signed ? 1 : 0;
  a.mul_table = mul_table;
  a.out = static_cast<uint8_t*>(out);
  a.out_stride = out_stride;
  a.status = device_status_word();
  // float constants of the fast quantize paths (NaN where the scales fall
  // outside the range their error bound covers)
  const double c_s = s_qkv * s_qkv / s_params[0], c_o = s_params[2] * s_qkv / s_params[3];
  a.c_s = (a.S.inv == a.S.inv && std::isfinite(c_s) && c_s > 1e-30 && c_s < 1e30) ? (float)c_s
                                                                                  : std::nanf("");
  a.c_o = (a.O.inv == a.O.inv && std::isfinite(c_o) && c_o > 1e-30 && c_o < 1e30) ? (float)c_o
                                                                                  : std::nanf("");
  // the scores' integer dot products fit the exact float conversion by
  // exponent-field addition when |dot| < 2^22
  const bool magic_s = hd * 255 * 255 < (1 << 22);
  size_t smem = (size_t)kAttnTile * a.hdp + (size_t)a.nk * a.hdp + (size_t)a.hdn * a.tk +
                (size_t)kAttnTile * a.tk + 264 * 8 + 264 * 4 + 256 * 4 + 256 * 4 +
                kAttnTile * 4 + kAttnMaxHd * 4 + 2 * kAttnTile * 8 + 2 * kAttnTile * 4 +
                2 * kAttnTile * 4 + 16 * 4 + 2 * 8 + 16;
  auto kern = magic_s ? attention_kernel<true> : attention_kernel<false>;
  // at most 512 / tmem_cols CTAs per SM, so that every allocation succeeds at once
  const size_t per_sm = 227 * 1024;
  const size_t ctas = 512 / cols;
  if (ctas < 8 && smem * (ctas + 1) <= per_sm) smem = per_sm / (ctas + 1) + 1024;
  static size_t attr_bytes[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  size_t* attr = (dev >= 0 && dev < 64) ? &attr_bytes[magic_s ? 1 : 0][dev] : nullptr;
  if (smem > 48 * 1024 && (!attr || *attr < smem)) {
    if (cuda_failed(
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
            "cudaFuncSetAttribute(attention)"))
      return last_status();
    if (attr) *attr = smem;
  }
  const int64_t grid = B * H * a.tiles;
  if (grid > 0x7FFFFFFF) {
    set_error(kUnsupported, "qa_attention_bytes_dev: too many heads");
    return last_status();
  }
  return launch_ex(kern, dim3((unsigned)grid), dim3(kAttnThreads), smem,
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

// ===================================== activation x activation MatMul ==
// The reference's float fallback for a MatMul of two activations
// (quant_layers.py:195-205: dequantize both, float_ops.py MatMul in float32,
// quantize):  Y[b, m, n] = clamp(rint(sa * sb * S / so) + zo, qmin, qmax)
// with S = sum_k (A[b, m, k] - za) * (B[b, k, n] - zb) exact in int32 (the
// host bounds K * max|a - za| * max|b - zb| < 2^31).  Only the reference's
// float32 summation rounds differently, so the outputs agree within one
// output step.  Operands are byte tensors addressed by strides (a transposed
// operand is the same bytes with its strides swapped); a CTA of 256 threads
// computes a 64 x 64 output tile, each thread 4 x 4 outputs, from 32-wide K
// slices staged as int32 in shared memory.
namespace qa {
namespace {
constexpr int kMmTile = 64, kMmK = 32;

struct MatMulActParams {
  const uint8_t* a;
  int64_t a_sb, a_sm, a_sk;
  const uint8_t* b;
  int64_t b_sb, b_sk, b_sn;
  int32_t a_signed, b_signed, za, zb;
  uint8_t* y;
  int64_t y_stride;
  int32_t M, N, K;
  double ratio;  // sa * sb, and the output grid
  double so;
  int32_t zo, qmin, qmax;
};

__device__ __forceinline__ int32_t byte_value(const uint8_t* p, int is_signed) {
  return is_signed ? (int32_t)(int8_t)*p : (int32_t)*p;
}

__global__ void __launch_bounds__(256) matmul_act_kernel(const MatMulActParams p) {
  __shared__ int32_t sa[kMmK][kMmTile + 1];
  __shared__ int32_t sb[kMmK][kMmTile + 1];
  ptx::pdl_wait();
  const int bz = blockIdx.z;
  const int m0 = blockIdx.y * kMmTile, n0 = blockIdx.x * kMmTile;
  const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;
  const uint8_t* A = p.a + (int64_t)bz * p.a_sb;
  const uint8_t* B = p.b + (int64_t)bz * p.b_sb;
  int32_t acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += kMmK) {
    for (int i = tid; i < kMmK * kMmTile; i += 256) {
      const int kk = i / kMmTile, r = i % kMmTile;
      const int k = k0 + kk;
      const int m = m0 + r, n = n0 + r;
      sa[kk][r] = (k < p.K && m < p.M)
                      ? byte_value(A + (int64_t)m * p.a_sm + (int64_t)k * p.a_sk, p.a_signed) - p.za
                      : 0;
      sb[kk][r] = (k < p.K && n < p.N)
                      ? byte_value(B + (int64_t)k * p.b_sk + (int64_t)n * p.b_sn, p.b_signed) - p.zb
                      : 0;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kMmK; ++kk) {
      int32_t av[4], bv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        av[u] = sa[kk][tm + 16 * u];
        bv[u] = sb[kk][tn + 16 * u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < 4; ++w) acc[u][w] += av[u] * bv[w];
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int m = m0 + tm + 16 * u;
    if (m >= p.M) continue;
    uint8_t* row = p.y + ((int64_t)bz * p.M + m) * p.y_stride;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int n = n0 + tn + 16 * w;
      if (n >= p.N) continue;
      double v = rint((double)acc[u][w] * p.ratio / p.so) + (double)p.zo;
      v = fmin(fmax(v, (double)p.qmin), (double)p.qmax);
      row[n] = (uint8_t)((int32_t)v & 0xFF);
    }
  }
}
}  // namespace
}  // namespace qa

QA_API int qa_matmul_act_bytes_dev(const void* a, int32_t a_signed, int64_t a_sb, int64_t a_sm,
                                   int64_t a_sk, int64_t za, double sa, const void* b,
                                   int32_t b_signed, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                                   int64_t zb, double sb, void* y, int64_t y_stride,
                                   int64_t batch, int64_t M, int64_t N, int64_t K, double so,
                                   int64_t zo, int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  if (!a || !b || !y || batch < 0 || M < 0 || N < 0 || K < 0 || y_stride < N ||
      !(so > 0.0) || qmin > qmax || qmin < -128 || qmax > 255) {
    set_error(kBadArgument, "qa_matmul_act_bytes_dev: bad arguments");
    return last_status();
  }
  // exact int32 sums: K * max|a - za| * max|b - zb| < 2^31
  const double ma = 255.0 + (double)std::llabs(za), mb = 255.0 + (double)std::llabs(zb);
  if ((double)K * ma * mb >= 2147483648.0 || M > 0x7FFFFFFF || N > 0x7FFFFFFF ||
      batch > 65535 || (M + kMmTile - 1) / kMmTile > 65535) {
    set_error(kUnsupported, "qa_matmul_act_bytes_dev: sizes beyond the kernel's exact range");
    return last_status();
  }
  if (batch == 0 || M == 0 || N == 0) return 0;
  MatMulActParams p;
  p.a = static_cast<const uint8_t*>(a);
  p.a_sb = a_sb;
  p.a_sm = a_sm;
  p.a_sk = a_sk;
  p.b = static_cast<const uint8_t*>(b);
  p.b_sb = b_sb;
  p.b_sk = b_sk;
  p.b_sn = b_sn;
  p.a_signed = a_signed ? 1 : 0;
  p.b_signed = b_signed ? 1 : 0;
  p.za = (int32_t)za;
  p.zb = (int32_t)zb;
  p.y = static_cast<uint8_t*>(y);
  p.y_stride = y_stride;
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.ratio = sa * sb;
  p.so = so;
  p.zo = (int32_t)zo;
  p.qmin = (int32_t)qmin;
  p.qmax = (int32_t)qmax;
  const dim3 grid((unsigned)((N + kMmTile - 1) / kMmTile), (unsigned)((M + kMmTile - 1) / kMmTile),
                  (unsigned)batch);
  return launch_ex(matmul_act_kernel, grid, dim3(256), 0, (cudaStream_t)stream, true, p)
             ? 0
             : last_status();
}
