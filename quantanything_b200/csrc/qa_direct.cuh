// Geometry of an NCHW/OIHW convolution exactly as the reference ABI passes it
// (qa_kernels.cpp:108-110, ConvShape), plus the CUDA-core launchers.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace qa {

struct ConvGeom {
  int64_t N, C, H, W, Cout, KH, KW, SH, SW, PH, PW, DH, DW, G, OH, OW;
};

bool validate_conv(const ConvGeom& g);

template <typename TA, typename TB, typename TAcc>
bool launch_gemm_tiled(const TA* A, const TB* B, TAcc* C, int64_t M, int64_t N, int64_t K,
                       cudaStream_t st);

template <typename TIn, typename TX, typename TW, typename TAcc>
bool launch_conv_direct(const TIn* x, const TW* w, TAcc* y, const ConvGeom& g, cudaStream_t st);

}  // namespace qa
