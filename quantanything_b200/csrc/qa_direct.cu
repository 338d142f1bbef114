// CUDA-core contraction kernels: exact for every geometry the ABI accepts.
//
//  * gemm_tiled:  C[M,N] = A[M,K]·B[K,N] with a 64x64 block tile staged in
//    shared memory and a 4x4 register tile per thread.  The int32xint32 ->
//    int64 instantiation is the "wide" route (qa_gemm_i32_i64,
//    qa_kernels.cpp:260): every MAC is one 32x32+64 wide multiply-add.
//  * conv_direct: one output element per thread, any groups / strides /
//    dilations / asymmetric padding (qa_kernels.cpp:141-185 semantics).  It
//    serves the wide conv route and the grouped / depthwise convolutions
//    that do not map onto tensor-core tiles.
//
// Narrow (int32 accumulator) instantiations accumulate in uint32 so the
// modulo-2^32 wrap of the CPU library is reproduced without signed overflow.
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "qa_common.cuh"
#include "qa_direct.cuh"
#include "qa_host_call.cuh"

namespace qa {

template <typename TAcc>
struct AccOf {
  using type = TAcc;
};
template <>
struct AccOf<int32_t> {
  using type = uint32_t;
};
template <>
struct AccOf<int64_t> {
  using type = uint64_t;
};

template <typename TAcc, typename T>
__device__ __forceinline__ typename AccOf<TAcc>::type widen(T v) {
  using U = typename AccOf<TAcc>::type;
  if constexpr (std::is_floating_point<TAcc>::value) {
    return (U)v;
  } else {
    return (U)(TAcc)v;  // sign-extend then reinterpret as unsigned
  }
}

constexpr int kTile = 64, kTK = 16, kGemmThreads = 256;

template <typename TA, typename TB, typename TAcc>
__global__ void __launch_bounds__(kGemmThreads)
    gemm_tiled_kernel(const TA* __restrict__ A, const TB* __restrict__ B, TAcc* __restrict__ C,
                      int64_t M, int64_t N, int64_t K) {
  using U = typename AccOf<TAcc>::type;
  __shared__ TA sA[kTK][kTile + 1];
  __shared__ TB sB[kTK][kTile];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t row0 = (int64_t)blockIdx.y * kTile, col0 = (int64_t)blockIdx.x * kTile;
  U acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;
  for (int64_t k0 = 0; k0 < K; k0 += kTK) {
    for (int e = threadIdx.x; e < kTK * kTile; e += kGemmThreads) {
      const int r = e / kTK, kk = e % kTK;  // A tile: rows r, k kk
      const int64_t gr = row0 + r, gk = k0 + kk;
      sA[kk][r] = (gr < M && gk < K) ? A[gr * K + gk] : TA(0);
      const int kb = e / kTile, c = e % kTile;  // B tile: k kb, col c
      const int64_t gkb = k0 + kb, gc = col0 + c;
      sB[kb][c] = (gkb < K && gc < N) ? B[gkb * N + gc] : TB(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kTK; ++kk) {
      U a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = widen<TAcc>(sA[kk][ty * 4 + i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = widen<TAcc>(sB[kk][tx * 4 + j]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + ty * 4 + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = col0 + tx * 4 + j;
      if (c < N) C[r * N + c] = (TAcc)acc[i][j];
    }
  }
}

// TX: the operand type the input is cast to before multiplying (int16 on
// the narrow path, like the CPU library's im2col cast).
template <typename TIn, typename TX, typename TW, typename TAcc>
__global__ void conv_direct_kernel(const TIn* __restrict__ x, const TW* __restrict__ w,
                                   TAcc* __restrict__ y, ConvGeom g) {
  using U = typename AccOf<TAcc>::type;
  const int64_t total = g.N * g.Cout * g.OH * g.OW;
  const int64_t Cg = g.C / g.G, Cog = g.Cout / g.G;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int64_t ox = idx % g.OW;
    int64_t t = idx / g.OW;
    const int64_t oy = t % g.OH;
    t /= g.OH;
    const int64_t co = t % g.Cout;
    const int64_t n = t / g.Cout;
    const int64_t grp = co / Cog;
    const TIn* xb = x + (n * g.C + grp * Cg) * g.H * g.W;
    const TW* wb = w + co * Cg * g.KH * g.KW;
    U s = 0;
    for (int64_t ky = 0; ky < g.KH; ++ky) {
      const int64_t iy = oy * g.SH - g.PH + ky * g.DH;
      if (iy < 0 || iy >= g.H) continue;
      for (int64_t kx = 0; kx < g.KW; ++kx) {
        const int64_t ix = ox * g.SW - g.PW + kx * g.DW;
        if (ix < 0 || ix >= g.W) continue;
        const TIn* xp = xb + iy * g.W + ix;
        const TW* wp = wb + ky * g.KW + kx;
        for (int64_t ci = 0; ci < Cg; ++ci)
          s += widen<TAcc>((TX)__ldg(xp + ci * g.H * g.W)) *
               widen<TAcc>(__ldg(wp + ci * g.KH * g.KW));
      }
    }
    y[idx] = (TAcc)s;
  }
}

template <typename TA, typename TB, typename TAcc>
bool launch_gemm_tiled(const TA* A, const TB* B, TAcc* C, int64_t M, int64_t N, int64_t K,
                       cudaStream_t st) {
  if (M <= 0 || N <= 0) return true;
  if (K <= 0) {
    return !cuda_failed(cudaMemsetAsync(C, 0, (size_t)(M * N) * sizeof(TAcc), st),
                        "cudaMemsetAsync(gemm K=0)");
  }
  const int64_t gy = (M + kTile - 1) / kTile, gx = (N + kTile - 1) / kTile;
  if (gy > 65535) {
    set_error(kUnsupported, "gemm: M too large for the CUDA-core tile grid");
    return false;
  }
  gemm_tiled_kernel<TA, TB, TAcc><<<dim3((unsigned)gx, (unsigned)gy), kGemmThreads, 0, st>>>(
      A, B, C, M, N, K);
  return !cuda_failed(cudaGetLastError(), "gemm_tiled launch");
}

template <typename TIn, typename TX, typename TW, typename TAcc>
bool launch_conv_direct(const TIn* x, const TW* w, TAcc* y, const ConvGeom& g, cudaStream_t st) {
  const int64_t total = g.N * g.Cout * g.OH * g.OW;
  if (total <= 0) return true;
  conv_direct_kernel<TIn, TX, TW, TAcc><<<grid_for(total, 256), 256, 0, st>>>(x, w, y, g);
  return !cuda_failed(cudaGetLastError(), "conv_direct launch");
}

template bool launch_gemm_tiled<float, float, float>(const float*, const float*, float*, int64_t,
                                                     int64_t, int64_t, cudaStream_t);
template bool launch_gemm_tiled<int16_t, int16_t, int32_t>(const int16_t*, const int16_t*,
                                                           int32_t*, int64_t, int64_t, int64_t,
                                                           cudaStream_t);
template bool launch_gemm_tiled<int32_t, int32_t, int64_t>(const int32_t*, const int32_t*,
                                                           int64_t*, int64_t, int64_t, int64_t,
                                                           cudaStream_t);
template bool launch_conv_direct<float, float, float, float>(const float*, const float*, float*,
                                                             const ConvGeom&, cudaStream_t);
template bool launch_conv_direct<int32_t, int16_t, int16_t, int32_t>(const int32_t*,
                                                                     const int16_t*, int32_t*,
                                                                     const ConvGeom&,
                                                                     cudaStream_t);
template bool launch_conv_direct<int32_t, int32_t, int32_t, int64_t>(const int32_t*,
                                                                     const int32_t*, int64_t*,
                                                                     const ConvGeom&,
                                                                     cudaStream_t);

bool validate_conv(const ConvGeom& g) {
  if (g.N < 0 || g.C <= 0 || g.H < 0 || g.W < 0 || g.Cout <= 0 || g.KH <= 0 || g.KW <= 0 ||
      g.SH <= 0 || g.SW <= 0 || g.DH <= 0 || g.DW <= 0 || g.G <= 0 || g.OH < 0 || g.OW < 0 ||
      g.PH < 0 || g.PW < 0) {
    set_error(kBadArgument, "conv: invalid geometry");
    return false;
  }
  if (g.C % g.G || g.Cout % g.G) {
    set_error(kBadArgument, "conv: channels not divisible by groups");
    return false;
  }
  return true;
}

}  // namespace qa
