// Memory-bound integer kernels behind the reference's element-wise entry
// points (qa_kernels.cpp:287-386): requantize (int32 / int64 accumulators),
// rescale, add, mul, lut, quantize_f32 and dequantize_f32.
//
// Each has a host-pointer ABI wrapper (the drop-in, synchronous) and a
// device-pointer entry point (`*_dev`, enqueued on a caller stream) used by
// the device-resident executor.  All index arithmetic is 64-bit; all
// requantization goes through qa_fixedpoint.cuh, bit-exact with the
// reference's 128-bit `mbqm`.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "qa_common.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_host_call.cuh"

namespace qa {

// ------------------------------------------------------------ kernels --

// clamp(mbqm(x + pre[c], mult[c], shift[c]) + post[c] + zp): the exact
// high-word form when the channel's multiplier and shift allow it (the
// usual case: M0 in [2^30, 2^31)), else the 128-bit mbqm.
__device__ __forceinline__ int64_t requant_channel(int64_t x, int64_t c,
                                                   const int64_t* __restrict__ mult,
                                                   const int64_t* __restrict__ shift,
                                                   const int64_t* __restrict__ pre,
                                                   const int64_t* __restrict__ post, int64_t zp,
                                                   int64_t qmin, int64_t qmax) {
  const int64_t pb = pre ? __ldg(pre + c) : 0;
  const int64_t qb = (post ? __ldg(post + c) : 0) + zp;
  const int64_t m = __ldg(mult + c), s = __ldg(shift + c);
  const int64_t v = x + pb;
  // the sum x + pre stays exact in int64 (|x| < 2^63 - |pre| for the inputs
  // the reference accepts); the bias add may not overflow the clamp bounds
  if (hi32_applies(m, 31 + s) && qb > -(1ll << 62) && qb < (1ll << 62))
    return requant_hi32(v, m, (int)(31 + s), qb, qmin, qmax);
  return requant_exact(v, m, s, qb, qmin, qmax);
}

// The 128-bit form out of line: channels outside the high-word form are
// rare, and inlining it would double the vector kernels' registers.
__device__ __noinline__ int64_t requant_exact_slow(int64_t x, int64_t m, int64_t s, int64_t bias,
                                                   int64_t lo, int64_t hi) {
  return requant_exact(x, m, s, bias, lo, hi);
}

// acc viewed as [outer, C, inner]; channel = (i / inner) % C.
template <typename TAcc>
__global__ void requantize_kernel(const TAcc* __restrict__ acc, int32_t* __restrict__ out,
                                  int64_t total, int64_t C, int64_t inner,
                                  const int64_t* __restrict__ mult,
                                  const int64_t* __restrict__ shift,
                                  const int64_t* __restrict__ pre,
                                  const int64_t* __restrict__ post, int64_t zp,
                                  int64_t qmin, int64_t qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t c = (inner == 1 ? i : i / inner) % C;
    out[i] = (int32_t)requant_channel((int64_t)acc[i], c, mult, shift, pre, post, zp, qmin, qmax);
  }
}

// Four consecutive elements per thread with 16-byte int32 loads and stores
// (total % 4 == 0, 16-byte aligned pointers).
__global__ void requantize_i32x4_kernel(const int32_t* __restrict__ acc, int32_t* __restrict__ out,
                                        int64_t quads, int64_t C, int64_t inner,
                                        const int64_t* __restrict__ mult,
                                        const int64_t* __restrict__ shift,
                                        const int64_t* __restrict__ pre,
                                        const int64_t* __restrict__ post, int64_t zp,
                                        int64_t qmin, int64_t qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto one = [&](const int4 v, const int64_t i) {
    const int32_t a[4] = {v.x, v.y, v.z, v.w};
    int32_t o[4];
    if (inner % 4 == 0) {
      // the quad lies in one channel (NCHW accumulators): its parameters once;
      // 32-bit division when the element index fits (a 64-bit one costs
      // several times the instructions)
      const int64_t c = quads < (1ll << 30)
                            ? (int64_t)((uint32_t)(4 * i) / (uint32_t)inner % (uint32_t)C)
                            : (4 * i / inner) % C;
      const int64_t pb = pre ? __ldg(pre + c) : 0;
      const int64_t qb = (post ? __ldg(post + c) : 0) + zp;
      const int64_t m = __ldg(mult + c), s = __ldg(shift + c);
      const bool hi = hi32_applies(m, 31 + s) && qb > -(1ll << 62) && qb < (1ll << 62);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        o[k] = (int32_t)(hi ? requant_hi32((int64_t)a[k] + pb, m, (int)(31 + s), qb, qmin, qmax)
                            : requant_exact_slow((int64_t)a[k] + pb, m, s, qb, qmin, qmax));
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int64_t e = 4 * i + k;
        const int64_t c = (inner == 1 ? e : e / inner) % C;
        o[k] = (int32_t)requant_channel((int64_t)a[k], c, mult, shift, pre, post, zp, qmin,
                                        qmax);
      }
    }
    return make_int4(o[0], o[1], o[2], o[3]);
  };
  const int4* src = reinterpret_cast<const int4*>(acc);
  int4* dst = reinterpret_cast<int4*>(out);
  // four loads in flight per thread before any arithmetic
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < quads; i += 4 * stride) {
    int4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) dst[i + u * stride] = one(v[u], i + u * stride);
  }
  for (; i < quads; i += stride) dst[i] = one(__ldg(src + i), i);
}

// Rows of C channels (inner == 1, C % 4 == 0) with a grid whose stride in
// quads is a multiple of C / 4 (or that visits each quad once): every quad a
// thread visits holds the same four channels, so their parameters and the
// choice of requantize form are taken once, outside the loop.
__global__ void requantize_rows_i32x4_kernel(const int32_t* __restrict__ acc,
                                             int32_t* __restrict__ out, int64_t quads, int64_t C,
                                             const int64_t* __restrict__ mult,
                                             const int64_t* __restrict__ shift,
                                             const int64_t* __restrict__ pre,
                                             const int64_t* __restrict__ post, int64_t zp,
                                             int64_t qmin, int64_t qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i0 >= quads) return;
  const int64_t c0 = 4 * (i0 % (C / 4));
  // per channel: the high-word form's 31-bit multiplier and total shift, or
  // ts = 0 for the exact form (its parameters are re-read on that cold path)
  int64_t pb[4], qb[4];
  int32_t m32[4], ts[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    pb[k] = pre ? __ldg(pre + c0 + k) : 0;
    qb[k] = (post ? __ldg(post + c0 + k) : 0) + zp;
    const int64_t m = __ldg(mult + c0 + k), sh = __ldg(shift + c0 + k);
    const bool hi = hi32_applies(m, 31 + sh) && qb[k] > -(1ll << 62) && qb[k] < (1ll << 62);
    m32[k] = hi ? (int32_t)m : 0;
    ts[k] = hi ? (int32_t)(31 + sh) : 0;
  }
  const int4* src = reinterpret_cast<const int4*>(acc);
  int4* dst = reinterpret_cast<int4*>(out);
  auto one = [&](const int4 v) {
    const int32_t a[4] = {v.x, v.y, v.z, v.w};
    int32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      o[k] = (int32_t)(ts[k] ? requant_hi32((int64_t)a[k] + pb[k], m32[k], ts[k], qb[k], qmin,
                                            qmax)
                             : requant_exact_slow((int64_t)a[k] + pb[k], __ldg(mult + c0 + k),
                                                  __ldg(shift + c0 + k), qb[k], qmin, qmax));
    return make_int4(o[0], o[1], o[2], o[3]);
  };
  // four loads in flight per thread before any arithmetic (the quads a
  // thread visits all hold its four channels)
  int64_t i = i0;
  for (; i + 3 * stride < quads; i += 4 * stride) {
    int4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) dst[i + u * stride] = one(v[u]);
  }
  for (; i < quads; i += stride) dst[i] = one(__ldg(src + i));
}

// NCHW planes (inner % 4 == 0): a block walks whole (image, channel) planes,
// so the channel's parameters are taken once per plane; each thread keeps
// up to four of the plane's quads in flight (predicated at the plane's end).
__global__ void requantize_planes_i32x4_kernel(const int32_t* __restrict__ acc,
                                               int32_t* __restrict__ out, int64_t planes,
                                               int64_t C, int64_t plane_quads,
                                               const int64_t* __restrict__ mult,
                                               const int64_t* __restrict__ shift,
                                               const int64_t* __restrict__ pre,
                                               const int64_t* __restrict__ post, int64_t zp,
                                               int64_t qmin, int64_t qmax) {
  const int64_t bd = blockDim.x;
  for (int64_t pl = blockIdx.x; pl < planes; pl += gridDim.x) {
    const int64_t c = pl % C;
    const int64_t pb = pre ? __ldg(pre + c) : 0;
    const int64_t qb = (post ? __ldg(post + c) : 0) + zp;
    const int64_t m = __ldg(mult + c), sh = __ldg(shift + c);
    const bool hi = hi32_applies(m, 31 + sh) && qb > -(1ll << 62) && qb < (1ll << 62);
    const int4* src = reinterpret_cast<const int4*>(acc) + pl * plane_quads;
    int4* dst = reinterpret_cast<int4*>(out) + pl * plane_quads;
    for (int64_t q = threadIdx.x; q < plane_quads; q += 4 * bd) {
      int4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (q + u * bd < plane_quads) v[u] = __ldg(src + q + u * bd);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (q + u * bd >= plane_quads) break;
        const int32_t a[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        int32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = (int32_t)(hi ? requant_hi32((int64_t)a[k] + pb, m, (int)(31 + sh), qb, qmin,
                                             qmax)
                              : requant_exact_slow((int64_t)a[k] + pb, m, sh, qb, qmin, qmax));
        dst[q + u * bd] = make_int4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

__global__ void rescale_kernel(const int32_t* __restrict__ x, int32_t* __restrict__ out,
                               int64_t n, int64_t zp_in, int64_t m, int64_t s,
                               int64_t zp_out, int64_t qmin, int64_t qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = (int32_t)requant_exact((int64_t)x[i] - zp_in, m, s, zp_out, qmin, qmax);
}

__global__ void add_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b,
                           int32_t* __restrict__ out, int64_t n, int64_t za, int64_t ma,
                           int64_t sa, int64_t zb, int64_t mb, int64_t sb, int64_t sign,
                           int64_t zp_out, int64_t qmin, int64_t qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const I128 ta = mbqm((int64_t)a[i] - za, ma, sa);
    I128 tb = mbqm((int64_t)b[i] - zb, mb, sb);
    // sign * tb on 128 bits (the reference multiplies the i128 by sign)
    if (sign == -1) {
      tb = neg_i128(tb);
    } else if (sign != 1) {
      // general sign: low 128 bits of tb * sign
      const uint64_t lo = tb.lo * (uint64_t)sign;
      const int64_t hi = (int64_t)(__umul64hi(tb.lo, (uint64_t)sign) +
                                   (uint64_t)tb.hi * (uint64_t)sign -
                                   (sign < 0 ? tb.lo : 0));
      tb = I128{lo, hi};
    }
    const I128 v = add_i128_i64(add_i128(ta, tb), zp_out);
    out[i] = (int32_t)clamp_i128(v, qmin, qmax);
  }
}

__global__ void mul_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b,
                           int32_t* __restrict__ out, int64_t n, int64_t za, int64_t zb,
                           int64_t m, int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t prod = (int64_t)((uint64_t)((int64_t)a[i] - za) * (uint64_t)((int64_t)b[i] - zb));
    out[i] = (int32_t)requant_exact(prod, m, s, zp_out, qmin, qmax);
  }
}

__global__ void lut_kernel(const int32_t* __restrict__ x, int32_t* __restrict__ out, int64_t n,
                           int64_t offset, const int32_t* __restrict__ lut, int64_t len) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t idx = (int64_t)x[i] - offset;
    idx = idx < 0 ? 0 : (idx >= len ? len - 1 : idx);
    out[i] = __ldg(lut + idx);
  }
}

// q = clamp(rint(x / scale) + zp) in IEEE double (division and rint are
// correctly rounded on the GPU exactly as on the host).  The reference's
// final double->int32 truncation is x86 cvttsd2si, which maps NaN and
// out-of-range values to INT32_MIN; the GPU conversion would give 0 or
// saturate, so that case is made explicit.
__device__ __forceinline__ int32_t quantize_one(float xv, double scale, double zp,
                                                double qmin, double qmax) {
  double v = rint((double)xv / scale) + zp;
  if (v < qmin) v = qmin;
  if (qmax < v) v = qmax;
  if (!(v >= -2147483648.0 && v < 2147483648.0)) return INT32_MIN;
  return (int32_t)v;
}

__global__ void quantize_kernel(const float* __restrict__ x, int32_t* __restrict__ q, int64_t n,
                                double scale, double zp, double qmin, double qmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    q[i] = quantize_one(x[i], scale, zp, qmin, qmax);
}

__global__ void dequantize_kernel(const int32_t* __restrict__ q, float* __restrict__ x,
                                  int64_t n, double scale, int64_t zp) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    x[i] = (float)((double)((int64_t)q[i] - zp) * scale);
}

// ------------------------------------------------------- launch helpers --
constexpr int kThreads = 256;

template <typename TAcc>
static bool launch_requantize(const TAcc* acc, int32_t* out, int64_t outer, int64_t C,
                              int64_t inner, const int64_t* mult, const int64_t* shift,
                              const int64_t* pre, const int64_t* post, int64_t zp,
                              int64_t qmin, int64_t qmax, cudaStream_t st) {
  const int64_t total = outer * C * inner;
  if (total <= 0) return true;
  if (sizeof(TAcc) == 4 && total % 4 == 0 &&
      ((reinterpret_cast<uintptr_t>(acc) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const int64_t quads = total / 4;
    if (inner == 1 && C % 4 == 0) {
      // grid stride a multiple of C / 4 quads: blocks a multiple of
      // (C / 4) / gcd(C / 4, kThreads)
      int64_t a = C / 4, b = kThreads;
      while (b) { const int64_t t = a % b; a = b; b = t; }
      const int64_t unit = (C / 4) / a;
      int64_t grid = grid_for(quads, kThreads, 2);
      if (grid * kThreads < quads) grid -= grid % unit;
      if (grid >= 1) {
        requantize_rows_i32x4_kernel<<<(unsigned)grid, kThreads, 0, st>>>(
            reinterpret_cast<const int32_t*>(acc), out, quads, C, mult, shift, pre, post, zp,
            qmin, qmax);
        return !cuda_failed(cudaGetLastError(), "requantize launch");
      }
    }
    if (inner % 4 == 0 && inner / 4 >= 32) {
      // threads: a quarter of the plane's quads (four in flight each), in warps
      const int64_t pq = inner / 4;
      const int threads = (int)std::min<int64_t>(256, ((pq + 3) / 4 + 31) / 32 * 32);
      const int64_t planes = outer * C;
      // one block per plane (the block scheduler balances the waves)
      const unsigned grid = (unsigned)std::min<int64_t>(planes, 0x7FFFFFFF);
      requantize_planes_i32x4_kernel<<<grid, threads, 0, st>>>(
          reinterpret_cast<const int32_t*>(acc), out, planes, C, pq, mult, shift, pre, post, zp,
          qmin, qmax);
      return !cuda_failed(cudaGetLastError(), "requantize launch");
    }
    requantize_i32x4_kernel<<<grid_for(total / 4, kThreads, 2), kThreads, 0, st>>>(
        reinterpret_cast<const int32_t*>(acc), out, total / 4, C, inner, mult, shift, pre, post,
        zp, qmin, qmax);
    return !cuda_failed(cudaGetLastError(), "requantize launch");
  }
  requantize_kernel<TAcc><<<grid_for(total, kThreads, 4), kThreads, 0, st>>>(
      acc, out, total, C, inner, mult, shift, pre, post, zp, qmin, qmax);
  return !cuda_failed(cudaGetLastError(), "requantize launch");
}

template <typename TAcc>
static void host_requantize(const TAcc* acc, int32_t* out, int64_t outer, int64_t C,
                            int64_t inner, const int64_t* mult, const int64_t* shift,
                            const int64_t* pre, const int64_t* post, int64_t zp,
                            int64_t qmin, int64_t qmax) {
  clear_error();
  const int64_t total = outer * C * inner;
  QA_REQUIRE(outer >= 0 && C >= 0 && inner >= 0, "requantize: negative size");
  if (total == 0) return;
  HostCall hc;
  auto s_acc = hc.input(acc, total);
  auto s_out = hc.output(out, total);
  auto s_m = hc.input(mult, C);
  auto s_s = hc.input(shift, C);
  auto s_pre = hc.input(pre, pre ? C : 0);
  auto s_post = hc.input(post, post ? C : 0);
  if (!hc.upload()) return;
  if (!launch_requantize<TAcc>(hc.dev(s_acc), hc.dev(s_out), outer, C, inner, hc.dev(s_m),
                               hc.dev(s_s), pre ? hc.dev(s_pre) : nullptr,
                               post ? hc.dev(s_post) : nullptr, zp, qmin, qmax, hc.stream()))
    return;
  hc.download();
}

}  // namespace qa

using namespace qa;

// =========================================================== host ABI ==
QA_API void qa_requantize_i32(const int32_t* acc, int32_t* out, int64_t outer, int64_t C,
                              int64_t inner, const int64_t* mult, const int64_t* shift,
                              const int64_t* pre_bias, const int64_t* post_bias, int64_t zp,
                              int64_t qmin, int64_t qmax) {
  host_requantize<int32_t>(acc, out, outer, C, inner, mult, shift, pre_bias, post_bias, zp,
                           qmin, qmax);
}

QA_API void qa_requantize_i64(const int64_t* acc, int32_t* out, int64_t outer, int64_t C,
                              int64_t inner, const int64_t* mult, const int64_t* shift,
                              const int64_t* pre_bias, const int64_t* post_bias, int64_t zp,
                              int64_t qmin, int64_t qmax) {
  host_requantize<int64_t>(acc, out, outer, C, inner, mult, shift, pre_bias, post_bias, zp,
                           qmin, qmax);
}

QA_API void qa_rescale(const int32_t* x, int32_t* out, int64_t n, int64_t zp_in, int64_t m,
                       int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax) {
  clear_error();
  QA_REQUIRE(n >= 0, "rescale: negative size");
  if (n == 0) return;
  HostCall hc;
  auto s_dx = hc.input(x, n);
  auto s_dout = hc.output(out, n);
  if (!hc.upload()) return;
  rescale_kernel<<<grid_for(n, kThreads, 4), kThreads, 0, hc.stream()>>>(hc.dev(s_dx), hc.dev(s_dout), n, zp_in, m,
                                                                          s, zp_out, qmin, qmax);
  if (cuda_failed(cudaGetLastError(), "rescale launch")) return;
  hc.download();
}

QA_API void qa_add(const int32_t* a, const int32_t* b, int32_t* out, int64_t n, int64_t za,
                   int64_t ma, int64_t sa, int64_t zb, int64_t mb, int64_t sb, int64_t sign,
                   int64_t zp_out, int64_t qmin, int64_t qmax) {
  clear_error();
  QA_REQUIRE(n >= 0, "add: negative size");
  if (n == 0) return;
  HostCall hc;
  auto s_da = hc.input(a, n);
  auto s_db = hc.input(b, n);
  auto s_dout = hc.output(out, n);
  if (!hc.upload()) return;
  add_kernel<<<grid_for(n, kThreads, 4), kThreads, 0, hc.stream()>>>(
      hc.dev(s_da), hc.dev(s_db), hc.dev(s_dout), n, za, ma, sa, zb, mb, sb, sign, zp_out, qmin, qmax);
  if (cuda_failed(cudaGetLastError(), "add launch")) return;
  hc.download();
}

QA_API void qa_mul(const int32_t* a, const int32_t* b, int32_t* out, int64_t n, int64_t za,
                   int64_t zb, int64_t m, int64_t s, int64_t zp_out, int64_t qmin,
                   int64_t qmax) {
  clear_error();
  QA_REQUIRE(n >= 0, "mul: negative size");
  if (n == 0) return;
  HostCall hc;
  auto s_da = hc.input(a, n);
  auto s_db = hc.input(b, n);
  auto s_dout = hc.output(out, n);
  if (!hc.upload()) return;
  mul_kernel<<<grid_for(n, kThreads, 4), kThreads, 0, hc.stream()>>>(hc.dev(s_da), hc.dev(s_db), hc.dev(s_dout), n, za, zb, m,
                                                                      s, zp_out, qmin, qmax);
  if (cuda_failed(cudaGetLastError(), "mul launch")) return;
  hc.download();
}

QA_API void qa_lut(const int32_t* x, int32_t* out, int64_t n, int64_t offset,
                   const int32_t* lut, int64_t lut_len) {
  clear_error();
  QA_REQUIRE(n >= 0, "lut: negative size");
  if (n == 0) return;
  QA_REQUIRE(lut_len > 0 && lut != nullptr, "lut: empty table");
  HostCall hc;
  auto s_dx = hc.input(x, n);
  auto s_dl = hc.input(lut, lut_len);
  auto s_dout = hc.output(out, n);
  if (!hc.upload()) return;
  lut_kernel<<<grid_for(n, kThreads, 4), kThreads, 0, hc.stream()>>>(hc.dev(s_dx), hc.dev(s_dout), n, offset, hc.dev(s_dl),
                                                                      lut_len);
  if (cuda_failed(cudaGetLastError(), "lut launch")) return;
  hc.download();
}

QA_API void qa_quantize_f32(const float* x, int32_t* q, int64_t n, double scale, int64_t zp,
                            int64_t qmin, int64_t qmax) {
  clear_error();
  QA_REQUIRE(n >= 0, "quantize_f32: negative size");
  if (n == 0) return;
  HostCall hc;
  auto s_dx = hc.input(x, n);
  auto s_dq = hc.output(q, n);
  if (!hc.upload()) return;
  quantize_kernel<<<grid_for(n, kThreads, 4), kThreads, 0, hc.stream()>>>(
      hc.dev(s_dx), hc.dev(s_dq), n, scale, (double)zp, (double)qmin, (double)qmax);
  if (cuda_failed(cudaGetLastError(), "quantize launch")) return;
  hc.download();
}

QA_API void qa_dequantize_f32(const int32_t* q, float* x, int64_t n, double scale, int64_t zp) {
  clear_error();
  QA_REQUIRE(n >= 0, "dequantize_f32: negative size");
  if (n == 0) return;
  HostCall hc;
  auto s_dq = hc.input(q, n);
  auto s_dx = hc.output(x, n);
  if (!hc.upload()) return;
  dequantize_kernel<<<grid_for(n, kThreads, 4), kThreads, 0, hc.stream()>>>(hc.dev(s_dq), hc.dev(s_dx), n, scale,
                                                                             zp);
  if (cuda_failed(cudaGetLastError(), "dequantize launch")) return;
  hc.download();
}

// ====================================================== device-pointer ==
QA_API int qa_requantize_i32_dev(const int32_t* acc, int32_t* out, int64_t outer, int64_t C,
                                 int64_t inner, const int64_t* mult, const int64_t* shift,
                                 const int64_t* pre_bias, const int64_t* post_bias, int64_t zp,
                                 int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  return launch_requantize<int32_t>(acc, out, outer, C, inner, mult, shift, pre_bias, post_bias,
                                    zp, qmin, qmax, (cudaStream_t)stream)
             ? 0
             : last_status();
}

QA_API int qa_requantize_i64_dev(const int64_t* acc, int32_t* out, int64_t outer, int64_t C,
                                 int64_t inner, const int64_t* mult, const int64_t* shift,
                                 const int64_t* pre_bias, const int64_t* post_bias, int64_t zp,
                                 int64_t qmin, int64_t qmax, void* stream) {
  clear_error();
  return launch_requantize<int64_t>(acc, out, outer, C, inner, mult, shift, pre_bias, post_bias,
                                    zp, qmin, qmax, (cudaStream_t)stream)
             ? 0
             : last_status();
}
