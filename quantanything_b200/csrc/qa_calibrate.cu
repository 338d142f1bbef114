// Device-resident float pass of calibration with the per-tensor range
// reductions fused into the kernels that produce each tensor.
//
// The reference calibrates by running the float graph (float_ops.py; its
// convolutions and GEMMs through qa_conv_f32 / qa_gemm_f32) and recording
// min / max of every layer output (quant_layers.py:130-137, _min_max
// :39-43) and of every graph input (quant_container.py:141-149).  Here the
// float tensors stay in device memory and every kernel below that writes a
// tensor also folds the values it writes into that tensor's range slot:
// two uint32 words {min key, max key} updated with atomicMin / atomicMax on
// an order-preserving encoding of float32 (key(a) < key(b) iff a < b for
// non-NaN values; NaN encodes above +inf, so a NaN shows up in the max
// word).  A slot starts at {0xFFFFFFFF, 0}.  Pass a null range pointer to
// skip the reduction.  All tensors are dense float32 unless strides say
// otherwise; every entry point enqueues on `stream` and returns 0 or an
// error status.
#include <cuda_runtime.h>

#include <cstdint>

#include "qa_common.cuh"
#include "qa_direct.cuh"

namespace qa {
namespace {

constexpr int kMaxRank = 6;
constexpr int kThreads = 256;

struct Strided {
  int64_t shape[kMaxRank];
  int64_t a[kMaxRank];  // element strides of the first operand
  int64_t b[kMaxRank];  // second operand / destination
};

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Folds this thread's (lo, hi) keys into `range` with one atomic pair per warp.
__device__ __forceinline__ void fold_range(uint32_t* range, uint32_t lo, uint32_t hi) {
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  if ((threadIdx.x & 31) == 0) {
    if (lo != 0xffffffffu) atomicMin(range, lo);
    if (hi != 0u) atomicMax(range + 1, hi);
  }
}

// Abramowitz & Stegun 7.1.26 in float64, odd in x (the erf of the float
// graph's Erf / Gelu nodes).
__device__ __forceinline__ double erf_as(double x) {
  const double ax = fabs(x);
  const double t = 1.0 / (1.0 + 0.3275911 * ax);
  const double poly =
      t * (0.254829592 +
           t * (-0.284496736 + t * (1.421413741 + t * (-1.453152027 + t * 1.061405429))));
  const double r = 1.0 - poly * exp(-ax * ax);
  return x > 0 ? r : (x < 0 ? -r : 0.0);
}

enum MapOp : int {
  kCopy = 0, kSigmoid, kRelu, kLeakyRelu, kTanh, kHardSigmoid, kHardSwish, kElu, kSoftplus,
  kAbs, kNeg, kSqrt, kExp, kErf, kGeluErf, kGeluTanh, kClip, kMapOps
};

__device__ __forceinline__ float map_value(int op, float x, float p0, float p1) {
  switch (op) {
    case kSigmoid: return (float)(1.0 / (1.0 + exp(-(double)x)));
    case kRelu: return x > 0.f ? x : (x == x ? 0.f : x);
    case kLeakyRelu: return x >= 0.f ? x : p0 * x;
    case kTanh: return tanhf(x);
    case kHardSigmoid: return fminf(fmaxf(__fadd_rn(__fmul_rn(p0, x), p1), 0.f), 1.f);
    case kHardSwish: return x * fminf(fmaxf(x / 6.0f + 0.5f, 0.f), 1.f);
    case kElu: return x > 0.f ? x : (float)((double)p0 * expm1((double)fminf(x, 0.f)));
    case kSoftplus: {
      const double d = x;
      return (float)(fmax(d, 0.0) + log1p(exp(-fabs(d))));
    }
    case kAbs: return fabsf(x);
    case kNeg: return -x;
    case kSqrt: return sqrtf(x);
    case kExp: return (float)exp((double)x);
    case kErf: return (float)erf_as((double)x);
    case kGeluErf: {
      const double d = x;
      return (float)(0.5 * d * (1.0 + erf_as(d / 1.4142135623730951)));
    }
    case kGeluTanh: {
      const double d = x;
      const double inner = 0.7978845608028654 * (d + 0.044715 * d * d * d);
      return (float)(0.5 * d * (1.0 + tanh(inner)));
    }
    case kClip: return fminf(fmaxf(x, p0), p1);
    default: return x;
  }
}

__global__ void map_kernel(const float* __restrict__ x, float* y, int64_t n, int op, float p0,
                           float p1, uint32_t* range) {
  uint32_t lo = 0xffffffffu, hi = 0u;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = map_value(op, x[i], p0, p1);
    y[i] = v;
    const uint32_t k = order_key(v);
    lo = min(lo, k);
    hi = max(hi, k);
  }
  if (range) fold_range(range, lo, hi);
}

enum BinOp : int { kAdd = 0, kSub, kMul, kDiv, kMax, kMin, kPow, kBinOps };

__device__ __forceinline__ float bin_value(int op, float a, float b) {
  switch (op) {
    case kAdd: return a + b;
    case kSub: return a - b;
    case kMul: return a * b;
    case kDiv: return a / b;
    case kMax: return (a != a || b != b) ? a + b : fmaxf(a, b);
    case kMin: return (a != a || b != b) ? a + b : fminf(a, b);
    case kPow: return (float)pow((double)a, (double)b);
    default: return a;
  }
}

// y (dense, `shape`) = op(a, b), a and b addressed by broadcast strides.
__global__ void binary_kernel(const float* a, const float* b, float* y, int rank, Strided s,
                              int64_t n, int op, uint32_t* range) {
  uint32_t lo = 0xffffffffu, hi = 0u;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t r = i, oa = 0, ob = 0;
    for (int d = rank - 1; d >= 0; --d) {
      const int64_t c = r % s.shape[d];
      r /= s.shape[d];
      oa += c * s.a[d];
      ob += c * s.b[d];
    }
    const float v = bin_value(op, a[oa], b[ob]);
    y[i] = v;
    const uint32_t k = order_key(v);
    lo = min(lo, k);
    hi = max(hi, k);
  }
  if (range) fold_range(range, lo, hi);
}

// y[offset_y + sum c_d * s.b[d]] = x[sum c_d * s.a[d]] over `shape`.
__global__ void copy_kernel(const float* x, float* y, int rank, Strided s, int64_t n,
                            uint32_t* range) {
  uint32_t lo = 0xffffffffu, hi = 0u;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t r = i, ox = 0, oy = 0;
    for (int d = rank - 1; d >= 0; --d) {
      const int64_t c = r % s.shape[d];
      r /= s.shape[d];
      ox += c * s.a[d];
      oy += c * s.b[d];
    }
    const float v = x[ox];
    y[oy] = v;
    const uint32_t k = order_key(v);
    lo = min(lo, k);
    hi = max(hi, k);
  }
  if (range) fold_range(range, lo, hi);
}

__global__ void fill_kernel(float* y, int64_t n, float value, uint32_t* range) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = value;
  if (range && blockIdx.x == 0 && threadIdx.x == 0 && n > 0) {
    atomicMin(range, order_key(value));
    atomicMax(range + 1, order_key(value));
  }
}

__global__ void range_kernel(const float* __restrict__ x, int64_t n, uint32_t* range) {
  uint32_t lo = 0xffffffffu, hi = 0u;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t k = order_key(x[i]);
    lo = min(lo, k);
    hi = max(hi, k);
  }
  fold_range(range, lo, hi);
}

// Batched C[z] = alpha * A[z] . B[z]: 64 x 64 tile per CTA, 16-deep K
// slices through shared memory, 4 x 4 outputs per thread, float32 sums.
constexpr int kGT = 64, kGK = 16;
__global__ void __launch_bounds__(256)
    gemm_f32_kernel(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    int64_t a_batch, int64_t a_m, int64_t a_k, int64_t b_batch, int64_t b_k,
                    int64_t b_n, float alpha, uint32_t* range) {
  __shared__ float As[kGK][kGT + 4];
  __shared__ float Bs[kGK][kGT + 4];
  const int64_t z = blockIdx.z;
  const float* Ab = A + z * a_batch;
  const float* Bb = B + z * b_batch;
  float* Cb = C + z * M * N;
  const int64_t m0 = (int64_t)blockIdx.y * kGT, n0 = (int64_t)blockIdx.x * kGT;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kGK) {
    for (int i = threadIdx.x; i < kGK * kGT; i += 256) {
      const int kk = i / kGT, mm = i % kGT;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? Ab[gm * a_m + gk * a_k] : 0.f;
      const int64_t gn = n0 + mm;
      Bs[kk][mm] = (gn < N && gk < K) ? Bb[gk * b_k + gn * b_n] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kGK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  uint32_t lo = 0xffffffffu, hi = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gm < M && gn < N) {
        const float v = alpha == 1.f ? acc[i][j] : alpha * acc[i][j];
        Cb[gm * N + gn] = v;
        const uint32_t k = order_key(v);
        lo = min(lo, k);
        hi = max(hi, k);
      }
    }
  }
  if (range) fold_range(range, lo, hi);
}

// Softmax over the last axis, float64, max subtracted; one warp per row.
__global__ void softmax_f32_kernel(const float* __restrict__ x, float* y, int64_t rows,
                                   int64_t cols, uint32_t* range) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t lo = 0xffffffffu, hi = 0u;
  if (warp < rows) {
    const float* xr = x + warp * cols;
    float* yr = y + warp * cols;
    double m = -INFINITY;
    for (int64_t c = lane; c < cols; c += 32) m = fmax(m, (double)xr[c]);
    for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s = 0.0;
    for (int64_t c = lane; c < cols; c += 32) s += exp((double)xr[c] - m);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    for (int64_t c = lane; c < cols; c += 32) {
      const float v = (float)(exp((double)xr[c] - m) / s);
      yr[c] = v;
      const uint32_t k = order_key(v);
      lo = min(lo, k);
      hi = max(hi, k);
    }
  }
  if (range) fold_range(range, lo, hi);
}

// LayerNormalization over the last D values, float64 mean / variance, then
// * gamma (+ beta) in float64; one warp per row.
__global__ void layernorm_f32_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                     const float* __restrict__ beta, float* y, int64_t rows,
                                     int64_t D, double eps, uint32_t* range) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t lo = 0xffffffffu, hi = 0u;
  if (warp < rows) {
    const float* xr = x + warp * D;
    float* yr = y + warp * D;
    double s = 0.0;
    for (int64_t c = lane; c < D; c += 32) s += (double)xr[c];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const double mean = s / (double)D;
    double v = 0.0;
    for (int64_t c = lane; c < D; c += 32) {
      const double d = (double)xr[c] - mean;
      v += d * d;
    }
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const double inv = sqrt(v / (double)D + eps);
    for (int64_t c = lane; c < D; c += 32) {
      double t = ((double)xr[c] - mean) / inv * (double)gamma[c];
      if (beta) t += (double)beta[c];
      const float f = (float)t;
      yr[c] = f;
      const uint32_t k = order_key(f);
      lo = min(lo, k);
      hi = max(hi, k);
    }
  }
  if (range) fold_range(range, lo, hi);
}

// MaxPool on NCHW, padding reads -inf (float_ops MaxPool on float tensors).
__global__ void maxpool_f32_kernel(const float* __restrict__ x, float* y, int64_t NC, int64_t H,
                                   int64_t W, int kh, int kw, int sh, int sw, int pt, int pl,
                                   int dh, int dw, int64_t OH, int64_t OW, uint32_t* range) {
  uint32_t lo = 0xffffffffu, hi = 0u;
  const int64_t n = NC * OH * OW;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t ox = i % OW, oy = (i / OW) % OH, p = i / (OW * OH);
    const float* xp = x + p * H * W;
    float m = -INFINITY;
    for (int a = 0; a < kh; ++a) {
      const int64_t iy = oy * sh - pt + (int64_t)a * dh;
      for (int b = 0; b < kw; ++b) {
        const int64_t ix = ox * sw - pl + (int64_t)b * dw;
        const float v = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? xp[iy * W + ix] : -INFINITY;
        m = (v != v || m != m) ? v + m : fmaxf(m, v);
      }
    }
    y[i] = m;
    const uint32_t k = order_key(m);
    lo = min(lo, k);
    hi = max(hi, k);
  }
  if (range) fold_range(range, lo, hi);
}

// Mean over each of NC planes of HW values (GlobalAveragePool); one warp
// per plane, float64 sum.
__global__ void plane_mean_kernel(const float* __restrict__ x, float* y, int64_t NC, int64_t HW,
                                  uint32_t* range) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t lo = 0xffffffffu, hi = 0u;
  if (warp < NC) {
    double s = 0.0;
    for (int64_t c = lane; c < HW; c += 32) s += (double)x[warp * HW + c];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float v = (float)(s / (double)HW);
    if (lane == 0) y[warp] = v;
    lo = hi = order_key(v);
  }
  if (range) fold_range(range, lo, hi);
}

// Range keys -> float32 pairs (lo, -hi), the form one MIN all-reduce combines;
// a slot nothing was folded into gives (+inf, +inf).
__global__ void range_decode_kernel(const uint32_t* range, float* out, int64_t count) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    for (int w = 0; w < 2; ++w) {
      const uint32_t k = range[2 * i + w];
      const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
      // an untouched slot {0xFFFFFFFF, 0} reads as (+inf, -inf)
      const float f = (w == 0 && k == 0xffffffffu) ? INFINITY
                      : (w == 1 && k == 0u)        ? -INFINITY
                                                   : __uint_as_float(u);
      out[2 * i + w] = w ? -f : f;
    }
  }
}

bool load_strided(Strided& s, int rank, const int64_t* shape, const int64_t* a,
                  const int64_t* b, int64_t& n, const char* what) {
  if (rank < 0 || rank > kMaxRank) {
    set_error(kBadArgument, std::string(what) + ": rank must lie in [0, 6]");
    return false;
  }
  n = 1;
  for (int d = 0; d < rank; ++d) {
    if (shape[d] < 0) {
      set_error(kBadArgument, std::string(what) + ": negative extent");
      return false;
    }
    s.shape[d] = shape[d];
    s.a[d] = a[d];
    s.b[d] = b[d];
    n *= shape[d];
  }
  return true;
}

inline unsigned warps_grid(int64_t rows) {
  const int64_t blocks = (rows * 32 + kThreads - 1) / kThreads;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

}  // namespace
}  // namespace qa

using namespace qa;

QA_API int qa_f32_map_dev(const float* x, float* y, int64_t n, int32_t op, float p0, float p1,
                          uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(op >= 0 && op < kMapOps, "qa_f32_map_dev: unknown op", last_status());
  QA_REQUIRE(n >= 0, "qa_f32_map_dev: negative size", last_status());
  if (n == 0) return 0;
  return launch_ex(map_kernel, dim3(grid_for(n, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, y, n, (int)op, p0, p1, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_binary_dev(const float* a, const float* b, float* y, int32_t rank,
                             const int64_t* shape, const int64_t* a_strides,
                             const int64_t* b_strides, int32_t op, uint32_t* range,
                             void* stream) {
  clear_error();
  QA_REQUIRE(op >= 0 && op < kBinOps, "qa_f32_binary_dev: unknown op", last_status());
  Strided s = {};
  int64_t n = 0;
  if (!load_strided(s, rank, shape, a_strides, b_strides, n, "qa_f32_binary_dev"))
    return last_status();
  if (n == 0) return 0;
  return launch_ex(binary_kernel, dim3(grid_for(n, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, a, b, y, (int)rank, s, n, (int)op, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_copy_dev(const float* x, float* y, int32_t rank, const int64_t* shape,
                           const int64_t* x_strides, const int64_t* y_strides, uint32_t* range,
                           void* stream) {
  clear_error();
  Strided s = {};
  int64_t n = 0;
  if (!load_strided(s, rank, shape, x_strides, y_strides, n, "qa_f32_copy_dev"))
    return last_status();
  if (n == 0) return 0;
  return launch_ex(copy_kernel, dim3(grid_for(n, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, y, (int)rank, s, n, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_fill_dev(float* y, int64_t n, float value, uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(n >= 0, "qa_f32_fill_dev: negative size", last_status());
  if (n == 0) return 0;
  return launch_ex(fill_kernel, dim3(grid_for(n, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, y, n, value, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_range_dev(const float* x, int64_t n, uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(range && n >= 0, "qa_f32_range_dev: bad argument", last_status());
  if (n == 0) return 0;
  return launch_ex(range_kernel, dim3(grid_for(n, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, n, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_range_decode_dev(const uint32_t* range, float* out, int64_t count,
                                   void* stream) {
  clear_error();
  QA_REQUIRE(range && out && count >= 0, "qa_f32_range_decode_dev: bad argument",
             last_status());
  if (count == 0) return 0;
  return launch_ex(range_decode_kernel, dim3(grid_for(count, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, range, out, count)
             ? 0
             : last_status();
}

QA_API int qa_f32_gemm_dev(const float* A, const float* B, float* C, int64_t batch, int64_t M,
                           int64_t N, int64_t K, int64_t a_batch, int64_t a_m, int64_t a_k,
                           int64_t b_batch, int64_t b_k, int64_t b_n, float alpha,
                           uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "qa_f32_gemm_dev: negative size",
             last_status());
  QA_REQUIRE(batch <= 65535 && (M + kGT - 1) / kGT <= 65535,
             "qa_f32_gemm_dev: batch or M too large for the tile grid", last_status());
  if (batch == 0 || M == 0 || N == 0) return 0;
  const dim3 grid((unsigned)((N + kGT - 1) / kGT), (unsigned)((M + kGT - 1) / kGT),
                  (unsigned)batch);
  return launch_ex(gemm_f32_kernel, grid, dim3(256), 0, (cudaStream_t)stream, false, A, B, C, M,
                   N, K, a_batch, a_m, a_k, b_batch, b_k, b_n, alpha, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_conv_dev(const float* x, const float* w, float* y, int64_t N, int64_t C,
                           int64_t H, int64_t W, int64_t Cout, int64_t KH, int64_t KW,
                           int64_t SH, int64_t SW, int64_t PH, int64_t PW, int64_t DH,
                           int64_t DW, int64_t G, int64_t OH, int64_t OW, void* stream) {
  // the same CUDA-core kernel as qa_conv_f32 (bit-identical sums), on
  // device pointers; the bias and the range follow as a broadcast Add
  clear_error();
  const ConvGeom g{N, C, H, W, Cout, KH, KW, SH, SW, PH, PW, DH, DW, G, OH, OW};
  if (!validate_conv(g)) return last_status();
  if (N * Cout * OH * OW == 0) return 0;
  return launch_conv_direct<float, float, float, float>(x, w, y, g, (cudaStream_t)stream)
             ? 0
             : last_status();
}

QA_API int qa_f32_softmax_dev(const float* x, float* y, int64_t rows, int64_t cols,
                              uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(rows >= 0 && cols >= 1, "qa_f32_softmax_dev: bad shape", last_status());
  if (rows == 0) return 0;
  return launch_ex(softmax_f32_kernel, dim3(warps_grid(rows)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, y, rows, cols, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_layernorm_dev(const float* x, const float* gamma, const float* beta, float* y,
                                int64_t rows, int64_t D, double eps, uint32_t* range,
                                void* stream) {
  clear_error();
  QA_REQUIRE(gamma && rows >= 0 && D >= 1, "qa_f32_layernorm_dev: bad argument",
             last_status());
  if (rows == 0) return 0;
  return launch_ex(layernorm_f32_kernel, dim3(warps_grid(rows)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, gamma, beta, y, rows, D, eps, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_maxpool_dev(const float* x, float* y, int64_t NC, int64_t H, int64_t W,
                              int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t pt,
                              int64_t pl, int64_t dh, int64_t dw, int64_t OH, int64_t OW,
                              uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(kh >= 1 && kw >= 1 && sh >= 1 && sw >= 1 && dh >= 1 && dw >= 1 && pt >= 0 &&
                 pl >= 0 && kh <= 64 && kw <= 64,
             "qa_f32_maxpool_dev: bad window", last_status());
  const int64_t n = NC * OH * OW;
  if (n <= 0) return 0;
  return launch_ex(maxpool_f32_kernel, dim3(grid_for(n, kThreads)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, y, NC, H, W, (int)kh, (int)kw, (int)sh,
                   (int)sw, (int)pt, (int)pl, (int)dh, (int)dw, OH, OW, range)
             ? 0
             : last_status();
}

QA_API int qa_f32_plane_mean_dev(const float* x, float* y, int64_t NC, int64_t HW,
                                 uint32_t* range, void* stream) {
  clear_error();
  QA_REQUIRE(NC >= 0 && HW >= 1, "qa_f32_plane_mean_dev: bad shape", last_status());
  if (NC == 0) return 0;
  return launch_ex(plane_mean_kernel, dim3(warps_grid(NC)), dim3(kThreads), 0,
                   (cudaStream_t)stream, false, x, y, NC, HW, range)
             ? 0
             : last_status();
}
