// Host-pointer ABI of the contraction entry points (qa_kernels.cpp:252-284):
// qa_gemm_{f32,i16_i32,i32_i64} and qa_conv_{f32,i32_i16_i32,i32_i32_i64}.
//
// Routing:
//  * narrow int16 GEMM / conv with tensor-core friendly shapes -> the
//    tcgen05 byte-split kernels (qa_umma.cu), exact int32 results;
//  * everything else (wide int64, float, grouped / depthwise convs, tiny
//    channel counts) -> the exact CUDA-core kernels (qa_direct.cu).
#include <cuda_runtime.h>

#include <cstdint>

#include "qa_common.cuh"
#include "qa_direct.cuh"
#include "qa_host_call.cuh"
#include "qa_umma.cuh"

using namespace qa;

namespace {

template <typename TA, typename TB, typename TAcc>
void host_gemm(int64_t M, int64_t N, int64_t K, const TA* A, const TB* B, TAcc* C,
               const char* name) {
  clear_error();
  QA_REQUIRE(M >= 0 && N >= 0 && K >= 0, std::string(name) + ": negative size");
  if (M == 0 || N == 0) return;
  HostCall hc;
  auto sa = hc.input(A, M * K);
  auto sb = hc.input(B, K * N);
  auto sc = hc.output(C, M * N);
  if (!hc.upload()) return;
  bool ok;
  if constexpr (std::is_same<TA, int16_t>::value) {
    ok = umma_gemm_i16_i32_abi(hc.dev(sa), hc.dev(sb), hc.dev(sc), M, N, K, hc.stream());
  } else {
    ok = launch_gemm_tiled<TA, TB, TAcc>(hc.dev(sa), hc.dev(sb), hc.dev(sc), M, N, K,
                                         hc.stream());
  }
  if (!ok) return;
  hc.download();
}

template <typename TIn, typename TX, typename TW, typename TAcc>
void host_conv(const TIn* x, const TW* w, TAcc* y, const ConvGeom& g, const char* name) {
  clear_error();
  if (!validate_conv(g)) return;
  const int64_t nx = g.N * g.C * g.H * g.W;
  const int64_t nw = g.Cout * (g.C / g.G) * g.KH * g.KW;
  const int64_t ny = g.N * g.Cout * g.OH * g.OW;
  if (ny == 0) return;
  HostCall hc;
  auto sx = hc.input(x, nx);
  auto sw = hc.input(w, nw);
  auto sy = hc.output(y, ny);
  if (!hc.upload()) return;
  bool ok;
  if constexpr (std::is_same<TX, int16_t>::value) {
    ok = umma_conv_i16_i32_abi(hc.dev(sx), hc.dev(sw), hc.dev(sy), g, hc.stream());
  } else {
    ok = launch_conv_direct<TIn, TX, TW, TAcc>(hc.dev(sx), hc.dev(sw), hc.dev(sy), g,
                                               hc.stream());
  }
  if (!ok) return;
  (void)name;
  hc.download();
}

}  // namespace

QA_API void qa_gemm_f32(int64_t M, int64_t N, int64_t K, const float* A, const float* B,
                        float* C) {
  host_gemm<float, float, float>(M, N, K, A, B, C, "qa_gemm_f32");
}

QA_API void qa_gemm_i16_i32(int64_t M, int64_t N, int64_t K, const int16_t* A, const int16_t* B,
                            int32_t* C) {
  host_gemm<int16_t, int16_t, int32_t>(M, N, K, A, B, C, "qa_gemm_i16_i32");
}

QA_API void qa_gemm_i32_i64(int64_t M, int64_t N, int64_t K, const int32_t* A, const int32_t* B,
                            int64_t* C) {
  host_gemm<int32_t, int32_t, int64_t>(M, N, K, A, B, C, "qa_gemm_i32_i64");
}

#define QA_CONV_PARAMS                                                                     \
  int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cout, int64_t KH, int64_t KW,       \
      int64_t SH, int64_t SW, int64_t PH, int64_t PW, int64_t DH, int64_t DW, int64_t G,  \
      int64_t OH, int64_t OW
#define QA_CONV_GEOM \
  ConvGeom { N, C, H, W, Cout, KH, KW, SH, SW, PH, PW, DH, DW, G, OH, OW }

QA_API void qa_conv_f32(const float* x, const float* w, float* y, QA_CONV_PARAMS) {
  host_conv<float, float, float, float>(x, w, y, QA_CONV_GEOM, "qa_conv_f32");
}

QA_API void qa_conv_i32_i16_i32(const int32_t* x, const int16_t* w, int32_t* y,
                                QA_CONV_PARAMS) {
  host_conv<int32_t, int16_t, int16_t, int32_t>(x, w, y, QA_CONV_GEOM, "qa_conv_i32_i16_i32");
}

QA_API void qa_conv_i32_i32_i64(const int32_t* x, const int32_t* w, int64_t* y,
                                QA_CONV_PARAMS) {
  host_conv<int32_t, int32_t, int32_t, int64_t>(x, w, y, QA_CONV_GEOM, "qa_conv_i32_i32_i64");
}
