// Tensor-core (tcgen05 kind::i8) implicit-GEMM kernel, its operand packing
// kernels and the host routes that use it.  See qa_umma.cuh for the design.
//
// CTA = 6 warps:
//   warps 0-3  gather the activation K-block tiles with cp.async (one row per
//              thread), then drain TMEM in the epilogue (warp w owns TMEM
//              lanes 32w..32w+31, i.e. output rows 32w..32w+31);
//   warp 4     allocates TMEM; its lane 0 issues the MMAs;
//   warp 5     lane 0 issues the weight-tile TMA loads.
// Pipeline: kStages shared-memory stages with full/empty mbarriers; the MMA
// thread releases a stage with tcgen05.commit.  All waits are bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "qa_common.cuh"
#include "qa_direct.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_ptx.cuh"
#include "qa_umma.cuh"
#include "qa_fused_epilogue.cuh"

namespace qa {

// int32 accumulators out: NCHW conv layout, or row-major GEMM rows
enum EpiMode : int { kEpiAcc32Nchw = 0, kEpiAcc32Row = 1 };

constexpr int kBM = 128;          // tile rows (TMEM lanes)
constexpr int kBKBytes = 128;     // K-block bytes (one 128-byte swizzle row)
constexpr int kProducerThreads = 128;
constexpr int kCtaThreads = 192;
constexpr uint64_t kWaitBudgetCycles = 4000000000ull;  // ~2 s at 1.9 GHz
constexpr int kTimeoutCode = 0x7001;

struct ConvTileParams {
  const uint8_t* a[2];      // activation planes (NHWC bytes)
  int64_t pix_stride;       // bytes between consecutive pixels of a plane
  int64_t group_a_off;      // byte offset between groups (grid.z)
  uint32_t pad_word[2];     // 4-byte pattern for taps outside the image
  int32_t a_signed;         // single-plane activations: s8 (1) or u8 (0)
  int32_t H, W, Cin;        // Cin: bytes per pixel consumed per tap (multiple of chunk)
  int32_t KH, KW, SH, SW, PH, PW, DH, DW, OH, OW;
  int64_t M;                // rows = images * OH * OW
  int32_t K;                // valid K bytes = KH*KW*Cin
  int32_t num_kb;           // K-blocks
  int32_t b_plane_rows;     // weight rows between planes in the tensor map
  int32_t b_group_rows;     // weight rows between groups
  int32_t n_valid;          // valid output columns per group
  // int32 accumulator outputs (ABI modes)
  int32_t* y;
  int64_t y_ctot;           // NCHW: channels of y; row mode: leading dimension
  int64_t ohw;
  int32_t* status;          // device error word
  int32_t stage_params;     // persistent 16-bit kernel: every CTA keeps one column
                            // tile (grid a multiple of the column tiles), so its
                            // channel parameters are staged in shared memory once
  FusedEpilogue epi;
};

template <int BN, int PA, int PB>
struct TileShape {
  static constexpr int kAPlaneBytes = kBM * kBKBytes;           // 16 KB
  static constexpr int kBPlaneBytes = BN * kBKBytes;
  static constexpr int kStageBytes = PA * kAPlaneBytes + PB * kBPlaneBytes;
  static constexpr int kNumAcc = (PA == 1 && PB == 1) ? 1 : 3;
  static constexpr int kTmemCols = (kNumAcc * BN <= 32)    ? 32
                                   : (kNumAcc * BN <= 64)  ? 64
                                   : (kNumAcc * BN <= 128) ? 128
                                   : (kNumAcc * BN <= 256) ? 256
                                                           : 512;
  static_assert(kNumAcc * BN <= 512, "TMEM columns");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
};

template <int BN, int PA, int PB, int kStages>
constexpr size_t umma_smem_bytes() {
  return 1024 /* alignment slack */ + (size_t)kStages * TileShape<BN, PA, PB>::kStageBytes +
         (2 * kStages + 1) * 8 + 16;
}

template <int BN, int PA, int PB, int kChunk, int kEpi, int kStages>
__global__ void __launch_bounds__(kCtaThreads, 1)
    umma_conv_kernel(const __grid_constant__ ConvTileParams p,
                     const __grid_constant__ CUtensorMap tmap_b) {
  using TS = TileShape<BN, PA, PB>;

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment of the swizzled tiles (the swizzle pattern is a
  // function of the shared address bits 4..9).
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + kStages * TS::kStageBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (kStages + s); };
  const uint32_t done_bar = bar_base + 8u * (2 * kStages);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + kStages * TS::kStageBytes +
                                                 (2 * kStages + 1) * 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  auto a_tile = [&](int s, int pl) {
    return base + s * TS::kStageBytes + pl * TS::kAPlaneBytes;
  };
  auto b_tile = [&](int s, int pl) {
    return base + s * TS::kStageBytes + PA * TS::kAPlaneBytes + pl * TS::kBPlaneBytes;
  };

  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int64_t m0 = (int64_t)blockIdx.x * kBM;
  const int n0 = blockIdx.y * BN;
  const int grp = blockIdx.z;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(full_bar(s), kProducerThreads + 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    ptx::mbar_init(done_bar, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc(ptx::smem_addr(s_tmem), TS::kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 5 && lane == 0) ptx::prefetch_tmap(&tmap_b);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  auto fail = [&]() {
    *s_abort = 1;
    if (p.status) atomicExch(p.status, kTimeoutCode);
  };
  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (ptx::mbar_wait(bar, parity, kWaitBudgetCycles)) return true;
    fail();
    return false;
  };

  if (warp < 4) {
    // ------------------------------------------------ activation gather --
    const int r = tid;  // tile row
    const int64_t m = m0 + r;
    const bool row_ok = m < p.M;
    int64_t img = 0, iy0 = 0, ix0 = 0;
    if (row_ok) {
      const int64_t ohw = (int64_t)p.OH * p.OW;
      img = m / ohw;
      const int64_t rem = m - img * ohw;
      const int64_t oy = rem / p.OW, ox = rem - (rem / p.OW) * p.OW;
      iy0 = oy * p.SH - p.PH;
      ix0 = ox * p.SW - p.PW;
    }
    const int64_t img_off = img * (int64_t)p.H * p.W * p.pix_stride + grp * p.group_a_off;
    const uint32_t row_off = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    const uint32_t sw = (uint32_t)(r & 7);
    for (int kb = 0; kb < p.num_kb; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages) wait(empty_bar(s), ((kb / kStages) - 1) & 1);
      const bool live = !*s_abort;
      const int k0 = kb * kBKBytes;
      int tap = k0 / p.Cin;
      int c = k0 - tap * p.Cin;
      int ky = tap / p.KW, kx = tap - (tap / p.KW) * p.KW;
#pragma unroll 4
      for (int kk = 0; kk < kBKBytes; kk += kChunk) {
        const int k = k0 + kk;
        const int64_t iy = iy0 + (int64_t)ky * p.DH, ix = ix0 + (int64_t)kx * p.DW;
        const bool in_k = k < p.K;
        const bool inside = row_ok && in_k && iy >= 0 && iy < p.H && ix >= 0 && ix < p.W;
        const int64_t off = img_off + (iy * p.W + ix) * p.pix_stride + c;
        const uint32_t soff = row_off + ((((uint32_t)kk >> 4) ^ sw) << 4) + ((uint32_t)kk & 15u);
#pragma unroll
        for (int pl = 0; pl < PA; ++pl) {
          const uint32_t dst = a_tile(s, pl) + soff;
          if (!live) continue;
          if (inside) {
            if (kChunk == 16)
              ptx::cp_async_16(dst, p.a[pl] + off, 16);
            else
              ptx::cp_async_4(dst, p.a[pl] + off, 4);
          } else if (row_ok && in_k && p.pad_word[pl] != 0u) {
            // tap outside the image: the raw zero point (centred value 0)
            uint8_t* d = smem + (dst - base);
            if (kChunk == 16)
              *reinterpret_cast<uint4*>(d) =
                  make_uint4(p.pad_word[pl], p.pad_word[pl], p.pad_word[pl], p.pad_word[pl]);
            else
              *reinterpret_cast<uint32_t*>(d) = p.pad_word[pl];
          } else {
            if (kChunk == 16)
              ptx::cp_async_16(dst, p.a[pl], 0);
            else
              ptx::cp_async_4(dst, p.a[pl], 0);
          }
        }
        c += kChunk;
        if (c >= p.Cin) {
          c = 0;
          if (++kx == p.KW) {
            kx = 0;
            ++ky;
          }
        }
      }
      // the zero-point padding stores are generic-proxy writes
      if (p.pad_word[0] | p.pad_word[1]) ptx::fence_proxy_async_smem();
      ptx::cp_async_mbar_arrive_noinc(full_bar(s));
    }
    ptx::cp_async_wait_all();
  } else if (warp == 5) {
    // ------------------------------------------------- weight TMA loads --
    if (lane == 0) {
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !wait(empty_bar(s), ((kb / kStages) - 1) & 1)) break;
        if (*s_abort) break;
        ptx::mbar_arrive_expect_tx(full_bar(s), PB * TS::kBPlaneBytes);
#pragma unroll
        for (int q = 0; q < PB; ++q)
          ptx::tma_load_2d(b_tile(s, q), &tmap_b, full_bar(s), kb * kBKBytes,
                           q * p.b_plane_rows + grp * p.b_group_rows + n0);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int s = kb % kStages;
        if (!wait(full_bar(s), (kb / kStages) & 1)) break;
        ptx::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBKBytes / 32; ++kk) {
#pragma unroll
          for (int pa = 0; pa < PA; ++pa) {
#pragma unroll
            for (int pb = 0; pb < PB; ++pb) {
              // accumulator of this plane pair: 0 = lo*lo, 1 = cross, 2 = hi*hi
              const int acc = (PA == 1) ? 0 : (pa + pb);
              const bool first_writer = (PA == 1) || !(pa == 1 && pb == 0);
              const uint32_t accumulate = (kb > 0 || kk > 0 || !first_writer) ? 1u : 0u;
              // operand signedness: 8-bit single plane is signed unless the
              // caller says otherwise; split planes are (lo: u8, hi: s8)
              const int a_signed = (PA == 1) ? p.a_signed : pa;
              const int b_signed = (PB == 1) ? 1 : pb;
              const uint32_t idesc = ptx::idesc_i8(kBM, BN, a_signed, b_signed);
              const uint64_t ad = ptx::smem_desc_sw128(a_tile(s, pa) + kk * 32);
              const uint64_t bd = ptx::smem_desc_sw128(b_tile(s, pb) + kk * 32);
              ptx::mma_i8(tmem + acc * BN, ad, bd, idesc, accumulate);
            }
          }
        }
        ptx::mma_commit(empty_bar(s));
      }
      ptx::mma_commit(done_bar);
    }
  }

  if (warp < 4) {
    // ----------------------------------------------------------- epilogue --
    const bool ok = wait(done_bar, 0);
    __syncwarp();
    ptx::tc_fence_after();
    const int r = tid;
    const int64_t m = m0 + r;
    const bool row_ok = ok && m < p.M;
    const uint32_t lane_base = tmem + (((uint32_t)warp * 32u) << 16);
    int64_t img = 0, pix = 0;
    if (row_ok) {
      const int64_t ohw = (int64_t)p.OH * p.OW;
      img = m / ohw;
      pix = m - img * ohw;
    }
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t v[TS::kNumAcc][16];
#pragma unroll
      for (int a = 0; a < TS::kNumAcc; ++a) ptx::tmem_ld16(lane_base + a * BN + c0, v[a]);
      ptx::tmem_ld_wait();
      if (!row_ok) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = n0 + c0 + j;  // column within the group
        if (n >= p.n_valid) continue;
        if constexpr (kEpi == kEpiAcc32Nchw || kEpi == kEpiAcc32Row) {
          uint32_t acc;
          if constexpr (TS::kNumAcc == 1) {
            acc = v[0][j];
          } else {
            acc = v[0][j] + (v[1][j] << 8) + (v[2][j] << 16);  // modulo 2^32
          }
          if constexpr (kEpi == kEpiAcc32Nchw) {
            const int64_t co = (int64_t)grp * p.n_valid + n;
            p.y[(img * p.y_ctot + co) * p.ohw + pix] = (int32_t)acc;
          } else {
            p.y[m * p.y_ctot + n] = (int32_t)acc;
          }
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, TS::kTmemCols);
  }
}

// ===================================================== host utilities ==

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

// Tiled tensor map of any rank (dims / box innermost first, strides in
// bytes for dims 1..rank-1), no interleave, no swizzle, zero fill.  Returns
// false with the error recorded.
bool encode_tiled_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error(kCudaError, "cuTensorMapEncodeTiled unavailable");
    return false;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  CUresult r = fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(kCudaError, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return false;
  }
  return true;
}

// 2-D uint8 tensor map over [rows, row_bytes] (rows `row_stride` bytes
// apart) with a 128 x box_rows box in the 128-byte swizzle; bytes past
// row_bytes and rows past `rows` read as zero.
bool make_rows_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                    int64_t row_stride, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error(kCudaError, "cuTensorMapEncodeTiled unavailable");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride & 15) || row_bytes > row_stride) {
    set_error(kBadArgument, "row tensor map: base / row stride not 16-byte aligned");
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(kCudaError, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return false;
  }
  return true;
}

bool make_weight_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                      int box_rows) {
  return make_rows_tmap(map, base, rows, row_bytes, row_bytes, box_rows);
}

template <int BN, int PA, int PB, int kChunk, int kEpi, int kStages>
bool launch_umma(const ConvTileParams& prm, const CUtensorMap& tmap, int64_t n_tiles,
                 int64_t groups, cudaStream_t st) {
  auto kern = umma_conv_kernel<BN, PA, PB, kChunk, kEpi, kStages>;
  const size_t smem = umma_smem_bytes<BN, PA, PB, kStages>();
  static bool attr_set[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem),
                    "cudaFuncSetAttribute(smem)"))
      return false;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t m_tiles = (prm.M + kBM - 1) / kBM;
  if (m_tiles > 0x7FFFFFFF || n_tiles > 65535 || groups > 65535) {
    set_error(kUnsupported, "umma: grid too large");
    return false;
  }
  kern<<<dim3((unsigned)m_tiles, (unsigned)n_tiles, (unsigned)groups), kCtaThreads, smem, st>>>(
      prm, tmap);
  return !cuda_failed(cudaGetLastError(), "umma_conv_kernel launch");
}

// ---------------------------------------------------- packing kernels ----

// int16 [rows, K] row-major (or int32 cast to int16) -> two byte planes
// [rows, Kp] (lo: v & 0xFF, hi: v >> 8), zero padded to Kp.
template <typename TIn>
__global__ void split_rows_kernel(const TIn* __restrict__ src, uint8_t* __restrict__ lo,
                                  uint8_t* __restrict__ hi, int64_t rows, int64_t K,
                                  int64_t Kp) {
  const int64_t total = rows * Kp;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / Kp, k = i - r * Kp;
    const int16_t v = k < K ? (int16_t)src[r * K + k] : (int16_t)0;
    lo[i] = (uint8_t)(v & 0xFF);
    hi[i] = (uint8_t)(v >> 8);
  }
}

// int16 B[K, N] row-major -> planes [Np, Kp] (transposed, zero padded).
__global__ void split_transpose_kernel(const int16_t* __restrict__ B, uint8_t* __restrict__ lo,
                                       uint8_t* __restrict__ hi, int64_t K, int64_t N,
                                       int64_t Np, int64_t Kp) {
  const int64_t total = Np * Kp;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t n = i / Kp, k = i - n * Kp;
    const int16_t v = (k < K && n < N) ? B[k * N + n] : (int16_t)0;
    lo[i] = (uint8_t)(v & 0xFF);
    hi[i] = (uint8_t)(v >> 8);
  }
}

// int32 NCHW (cast to int16) -> NHWC planes with Cp channels (zero padded).
__global__ void split_nchw_to_nhwc_kernel(const int32_t* __restrict__ x, uint8_t* __restrict__ lo,
                                          uint8_t* __restrict__ hi, int64_t N, int64_t C,
                                          int64_t HW, int64_t Cp) {
  const int64_t total = N * HW * Cp;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t c = i % Cp;
    const int64_t t = i / Cp;
    const int64_t pix = t % HW, n = t / HW;
    const int16_t v = c < C ? (int16_t)x[(n * C + c) * HW + pix] : (int16_t)0;
    lo[i] = (uint8_t)(v & 0xFF);
    hi[i] = (uint8_t)(v >> 8);
  }
}

// int16 OIHW weights [G*Cog, Cg, KH, KW] -> planes [G][Cogp][KH*KW*Cgp]
// with K ordered (ky, kx, c).
__global__ void split_weights_kernel(const int16_t* __restrict__ w, uint8_t* __restrict__ lo,
                                     uint8_t* __restrict__ hi, int64_t G, int64_t Cog,
                                     int64_t Cogp, int64_t Cg, int64_t Cgp, int64_t KH,
                                     int64_t KW, int64_t Kp) {
  const int64_t total = G * Cogp * Kp;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t Kv = KH * KW * Cgp;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t k = i % Kp;
    const int64_t row = i / Kp;
    const int64_t o = row % Cogp, g = row / Cogp;
    int16_t v = 0;
    if (o < Cog && k < Kv) {
      const int64_t tap = k / Cgp, c = k - tap * Cgp;
      const int64_t ky = tap / KW, kx = tap - ky * KW;
      if (c < Cg) v = w[(((g * Cog + o) * Cg + c) * KH + ky) * KW + kx];
    }
    lo[i] = (uint8_t)(v & 0xFF);
    hi[i] = (uint8_t)(v >> 8);
  }
}

static inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Scratch for the packed planes of an ABI call: a per-thread grow-only
// buffer separate from the HostCall arena (which holds the call's operands).
static uint8_t* pack_scratch(size_t bytes) {
  static thread_local uint8_t* buf = nullptr;
  static thread_local size_t cap = 0;
  static thread_local int dev = -1;
  int cur = 0;
  cudaGetDevice(&cur);
  if (buf && (bytes > cap || dev != cur)) {
    cudaDeviceSynchronize();
    cudaFree(buf);
    buf = nullptr;
    cap = 0;
  }
  if (!buf) {
    size_t want = bytes < (size_t(32) << 20) ? (size_t(32) << 20) : bytes;
    if (cuda_failed(cudaMalloc(&buf, want), "cudaMalloc(pack scratch)")) return nullptr;
    cap = want;
    dev = cur;
  }
  return buf;
}

constexpr int kSplitBN = 64;
constexpr int kSplitStages = 4;

bool umma_gemm_i16_i32_abi(const int16_t* A, const int16_t* B, int32_t* C, int64_t M, int64_t N,
                           int64_t K, cudaStream_t st) {
  if (K == 0 || M * N == 0 || K > (int64_t(1) << 24)) {
    return launch_gemm_tiled<int16_t, int16_t, int32_t>(A, B, C, M, N, K, st);
  }
  const int64_t Kp = round_up(K, 16);
  const int64_t Np = round_up(N, kSplitBN);
  const size_t a_bytes = align256((size_t)(M * Kp)), b_bytes = align256((size_t)(Np * Kp));
  uint8_t* scratch = pack_scratch(2 * a_bytes + 2 * b_bytes);
  if (!scratch) return false;
  uint8_t *a_lo = scratch, *a_hi = scratch + a_bytes;
  uint8_t *b_lo = a_hi + a_bytes, *b_hi = b_lo + b_bytes;
  split_rows_kernel<int16_t><<<grid_for(M * Kp, 256), 256, 0, st>>>(A, a_lo, a_hi, M, K, Kp);
  split_transpose_kernel<<<grid_for(Np * Kp, 256), 256, 0, st>>>(B, b_lo, b_hi, K, N, Np, Kp);
  if (cuda_failed(cudaGetLastError(), "split launch")) return false;
  // the two weight planes are consecutive [Np, Kp] blocks of one tensor map
  CUtensorMap tmap;
  if (!make_weight_tmap(&tmap, b_lo, 2 * Np, Kp, kSplitBN)) return false;
  if ((size_t)(b_hi - b_lo) != (size_t)(Np * Kp)) {
    // planes must be contiguous for the single tensor map: repack offsets
    set_error(kBadArgument, "internal: weight planes not contiguous");
    return false;
  }
  ConvTileParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.a[0] = a_lo;
  prm.a[1] = a_hi;
  prm.pix_stride = Kp;
  prm.H = prm.W = 1;
  prm.Cin = (int32_t)Kp;
  prm.KH = prm.KW = prm.SH = prm.SW = prm.DH = prm.DW = 1;
  prm.OH = prm.OW = 1;
  prm.M = M;
  prm.K = (int32_t)Kp;
  prm.num_kb = (int32_t)((Kp + kBKBytes - 1) / kBKBytes);
  prm.b_plane_rows = (int32_t)Np;
  prm.n_valid = (int32_t)N;
  prm.y = C;
  prm.y_ctot = N;
  prm.ohw = 1;
  prm.status = device_status_word();
  return launch_umma<kSplitBN, 2, 2, 16, kEpiAcc32Row, kSplitStages>(prm, tmap, Np / kSplitBN, 1,
                                                                      st);
}

bool umma_conv_i16_i32_abi(const int32_t* x, const int16_t* w, int32_t* y, const ConvGeom& g,
                           cudaStream_t st) {
  const int64_t Cg = g.C / g.G, Cog = g.Cout / g.G;
  const bool tiles_fit = (g.G == 1) || (Cg % 16 == 0);
  const int64_t Cgp = g.G == 1 ? round_up(g.C, 16) : Cg;
  const int64_t Kv = g.KH * g.KW * Cgp;
  if (!tiles_fit || Kv > (int64_t(1) << 24) || g.H * g.W == 0) {
    return launch_conv_direct<int32_t, int16_t, int16_t, int32_t>(x, w, y, g, st);
  }
  const int64_t Cp = g.G == 1 ? Cgp : g.C;
  const int64_t HW = g.H * g.W;
  const int64_t Kp = round_up(Kv, 16);
  const int64_t Cogp = round_up(Cog, kSplitBN);
  const size_t a_bytes = align256((size_t)(g.N * HW * Cp));
  const size_t b_bytes = (size_t)(g.G * Cogp * Kp);  // planes must be contiguous
  uint8_t* scratch = pack_scratch(2 * a_bytes + align256(2 * b_bytes));
  if (!scratch) return false;
  uint8_t *a_lo = scratch, *a_hi = scratch + a_bytes;
  uint8_t *b_lo = a_hi + a_bytes, *b_hi = b_lo + b_bytes;
  split_nchw_to_nhwc_kernel<<<grid_for(g.N * HW * Cp, 256), 256, 0, st>>>(x, a_lo, a_hi, g.N,
                                                                           g.C, HW, Cp);
  split_weights_kernel<<<grid_for(g.G * Cogp * Kp, 256), 256, 0, st>>>(
      w, b_lo, b_hi, g.G, Cog, Cogp, Cg, Cgp, g.KH, g.KW, Kp);
  if (cuda_failed(cudaGetLastError(), "split launch")) return false;
  CUtensorMap tmap;
  if (!make_weight_tmap(&tmap, b_lo, 2 * g.G * Cogp, Kp, kSplitBN)) return false;
  ConvTileParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.a[0] = a_lo;
  prm.a[1] = a_hi;
  prm.pix_stride = Cp;
  prm.group_a_off = Cg;
  prm.H = (int32_t)g.H;
  prm.W = (int32_t)g.W;
  prm.Cin = (int32_t)Cgp;
  prm.KH = (int32_t)g.KH;
  prm.KW = (int32_t)g.KW;
  prm.SH = (int32_t)g.SH;
  prm.SW = (int32_t)g.SW;
  prm.PH = (int32_t)g.PH;
  prm.PW = (int32_t)g.PW;
  prm.DH = (int32_t)g.DH;
  prm.DW = (int32_t)g.DW;
  prm.OH = (int32_t)g.OH;
  prm.OW = (int32_t)g.OW;
  prm.M = g.N * g.OH * g.OW;
  prm.K = (int32_t)Kv;
  prm.num_kb = (int32_t)((Kp + kBKBytes - 1) / kBKBytes);
  prm.b_plane_rows = (int32_t)(g.G * Cogp);
  prm.b_group_rows = (int32_t)Cogp;
  prm.n_valid = (int32_t)Cog;
  prm.y = y;
  prm.y_ctot = g.Cout;
  prm.ohw = g.OH * g.OW;
  prm.status = device_status_word();
  if (prm.M == 0) return true;
  return launch_umma<kSplitBN, 2, 2, 16, kEpiAcc32Nchw, kSplitStages>(prm, tmap, Cogp / kSplitBN,
                                                                       g.G, st);
}

}  // namespace qa

namespace qa {

// Byte-split tensor-core GEMM with caller-provided plane storage: the same
// packing and kernel as umma_gemm_i16_i32_abi, but the four byte planes are
// laid out in `planes` (planes_bytes long) and the timeout status goes to
// `status`, so nothing here allocates.  Returns false (error recorded) when
// the planes do not fit.
size_t umma_gemm_planes_bytes(int64_t M, int64_t N, int64_t K) {
  const int64_t Kp = round_up(K, 16);
  const int64_t Np = round_up(N, kSplitBN);
  return 2 * align256((size_t)(M * Kp)) + 2 * (size_t)(Np * Kp);
}

bool umma_gemm_i16_i32_into(const int16_t* A, const int16_t* B, int32_t* C, int64_t M,
                            int64_t N, int64_t K, uint8_t* planes, size_t planes_bytes,
                            int32_t* status, cudaStream_t st) {
  if (K == 0 || M * N == 0) {
    return launch_gemm_tiled<int16_t, int16_t, int32_t>(A, B, C, M, N, K, st);
  }
  if (K > (int64_t(1) << 24) || umma_gemm_planes_bytes(M, N, K) > planes_bytes) {
    set_error(kBadArgument, "byte planes exceed the provided scratch");
    return false;
  }
  const int64_t Kp = round_up(K, 16);
  const int64_t Np = round_up(N, kSplitBN);
  const size_t a_bytes = align256((size_t)(M * Kp));
  uint8_t *a_lo = planes, *a_hi = planes + a_bytes;
  uint8_t *b_lo = a_hi + a_bytes, *b_hi = b_lo + Np * Kp;
  split_rows_kernel<int16_t><<<grid_for(M * Kp, 256), 256, 0, st>>>(A, a_lo, a_hi, M, K, Kp);
  split_transpose_kernel<<<grid_for(Np * Kp, 256), 256, 0, st>>>(B, b_lo, b_hi, K, N, Np, Kp);
  if (cuda_failed(cudaGetLastError(), "split launch")) return false;
  CUtensorMap tmap;
  if (!make_weight_tmap(&tmap, b_lo, 2 * Np, Kp, kSplitBN)) return false;
  ConvTileParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.a[0] = a_lo;
  prm.a[1] = a_hi;
  prm.pix_stride = Kp;
  prm.H = prm.W = 1;
  prm.Cin = (int32_t)Kp;
  prm.KH = prm.KW = prm.SH = prm.SW = prm.DH = prm.DW = 1;
  prm.OH = prm.OW = 1;
  prm.M = M;
  prm.K = (int32_t)Kp;
  prm.num_kb = (int32_t)((Kp + kBKBytes - 1) / kBKBytes);
  prm.b_plane_rows = (int32_t)Np;
  prm.n_valid = (int32_t)N;
  prm.y = C;
  prm.y_ctot = N;
  prm.ohw = 1;
  prm.status = status;
  return launch_umma<kSplitBN, 2, 2, 16, kEpiAcc32Row, kSplitStages>(prm, tmap, Np / kSplitBN, 1,
                                                                      st);
}

}  // namespace qa

// ============================================ 16-bit resident layers ==

#include "../../include/qa_kernels.h"

namespace qa {

// Persistent, warp-specialized form of the byte-split kernel for the
// resident 16-bit layers.  One CTA per SM walks a strided list of
// (128-row, BN-column) output tiles; roles:
//   warps 0-3  gather both activation planes of every K-block (cp.async,
//              one tile row per thread, K-block bytes past K skipped: the
//              packed weights are zero there);
//   warp 4     allocates TMEM; lane 0 issues four MMAs per 32-byte K-step
//              (lo*lo, lo*hi, hi*lo, hi*hi) into one of two accumulator
//              sets of three int32 accumulators, K-steps past K skipped;
//   warp 5     lane 0 loads both weight planes of every K-block by TMA;
//   warps 6-13 two epilogue warpgroups, one per accumulator set (even
//              tiles / odd tiles; TMEM lane quarter = warp % 4), run the
//              16-bit epilogue while the MMAs fill the other set.
// kSmemLut: the layer's activation table (65536 int16 entries at most) is
// copied into shared memory at the start, so each lookup is a shared-memory
// read (a few bank conflicts) instead of a gather of 32 L1 sectors per warp;
// the table takes 128 KB, so such layers run two stages instead of four.
// Every mbarrier wait is bounded; on expiry the kernel records
// kTimeoutCode in the status word, stops issuing work and exits.
constexpr int kP16Threads = 448;
constexpr int kP16LutEntries = 65536;

// kWP: weight byte planes.  2 for int16 weights (lo u8, hi s8): four MMAs
// per K-step into three accumulators (shifts 0, 8, 16).  3 for the 17-bit
// centred weights of uint16 graphs, w = b0 + 256 b1 + 65536 b2 (b0, b1 u8,
// b2 s8 in {-1, 0}): six MMAs into four accumulators (shifts 0, 8, 16, 24).
// Two accumulator sets (double buffering, one epilogue warpgroup per set)
// when they fit the 512 TMEM columns, else one set that both epilogue
// warpgroups drain half of each tile's columns.
template <int BN, bool kSmemLut, int kWP>
struct P16Layout {
  static constexpr int kAccs = kWP == 3 ? 4 : 3;  // accumulators per set
  static constexpr int kSetCols = kAccs * BN;      // one accumulator set
  static constexpr int kSets = 2 * kSetCols <= 512 ? 2 : 1;
  static constexpr int kAPlane = kBM * kBKBytes;  // 16 KB
  static constexpr int kBPlane = BN * kBKBytes;
  static constexpr int kStage = 2 * kAPlane + kWP * kBPlane;
  static constexpr int kLutBytes = kSmemLut ? kP16LutEntries * 2 : 0;
  static constexpr int kParamBytes = BN * (int)sizeof(ChanParams16);  // one column tile
  static constexpr int kFit = (232448 - 1024 - 256 - kLutBytes - kParamBytes) / kStage;
  static constexpr int kStages =
      kWP == 2 ? (kSmemLut ? 2 : (BN >= 128 ? 3 : 4)) : (kFit < 4 ? kFit : 4);
  static constexpr int kCols = kSets * kSetCols;
  static constexpr int kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                   : kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "accumulator sets must fit TMEM");
  static_assert(kStages >= 2, "at least two stages must fit shared memory");
  static_assert(!(kSmemLut && BN >= 128), "the shared-memory table leaves one stage at BN 128");
  static constexpr size_t kBarOff = (size_t)kStages * kStage + kLutBytes + kParamBytes;
  static constexpr size_t kSmem = 1024 + kBarOff + (2 * kStages + 4) * 8 + 16;
  static_assert(kSmem <= 232448, "shared memory per CTA");
};

template <int BN, int kChunk, bool kSmemLut, int kWP>
__global__ void __launch_bounds__(kP16Threads, 1)
    umma16_persistent_kernel(const __grid_constant__ ConvTileParams p,
                             const __grid_constant__ CUtensorMap tmap_b, int64_t n_tiles,
                             int64_t total_tiles) {
  using L = P16Layout<BN, kSmemLut, kWP>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + (uint32_t)L::kBarOff;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (S + s); };
  auto accf_bar = [&](int b) { return bar_base + 8u * (2 * S + b); };
  auto acce_bar = [&](int b) { return bar_base + 8u * (2 * S + 2 + b); };
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::kBarOff + (2 * S + 4) * 8);
  int16_t* s_lut = reinterpret_cast<int16_t*>(smem + (size_t)S * L::kStage);
  ChanParams16* s_par =
      reinterpret_cast<ChanParams16*>(smem + (size_t)S * L::kStage + L::kLutBytes);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  auto a_tile = [&](int s, int pl) { return base + s * L::kStage + pl * L::kAPlane; };
  auto b_tile = [&](int s, int pl) {
    return base + s * L::kStage + 2 * L::kAPlane + pl * L::kBPlane;
  };

  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(full_bar(s), kProducerThreads + 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(accf_bar(b), 1);
      ptx::mbar_init(acce_bar(b), L::kSets == 2 ? 128 : 256);
    }
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc(ptx::smem_addr(s_tmem), L::kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 5 && lane == 0) ptx::prefetch_tmap(&tmap_b);
  if constexpr (kSmemLut) {
    // the host guarantees lut_len <= 65536 and a 16-byte aligned table
    const int64_t n16 = (p.epi.lut_len * 2 + 15) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(p.epi.lut16);
    uint4* dst = reinterpret_cast<uint4*>(s_lut);
    for (int64_t i = tid; i < n16; i += kP16Threads) dst[i] = __ldg(src + i);
  }
  int par_hi = 1;
  if (p.stage_params) {
    // this CTA's column tile (the host made the grid a multiple of n_tiles)
    const int nb0 = (int)(blockIdx.x % n_tiles) * BN;
    for (int c = tid; c < BN; c += kP16Threads) {
      const int n = nb0 + c < p.n_valid ? nb0 + c : nb0;
      const int64_t mv = p.epi.mult[n], sv = p.epi.shift[n];
      ChanParams16 cp;
      cp.bias = p.epi.bias ? p.epi.bias[n] : 0;
      cp.mult = mv;
      cp.ts = (int32_t)(31 + sv);
      cp.hi = (p.epi.fast || hi32_applies(mv, 31 + sv)) ? 1 : 0;
      par_hi &= cp.hi;
      s_par[c] = cp;
    }
  }
  ptx::tc_fence_before();
  const bool par_all_hi = __syncthreads_and(par_hi) != 0;
  ptx::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  auto fail = [&]() {
    *s_abort = 1;
    if (p.status) atomicExch(p.status, kTimeoutCode);
  };
  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (ptx::mbar_wait_sleep(bar, parity, kWaitBudgetCycles)) return true;
    fail();
    return false;
  };
  const int64_t first = blockIdx.x, step = gridDim.x;

  if (warp < 4) {
    // ------------------------------------------------ activation gather --
    // offsets within one image fit 32 bits (host-checked H*W*pix_stride)
    const int r = tid;
    const uint32_t row_off = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    const uint32_t sw = (uint32_t)(r & 7);
    const int64_t ohw = (int64_t)p.OH * p.OW;
    const int pix_stride = (int)p.pix_stride;
    int64_t g = 0;
    for (int64_t t = first; t < total_tiles; t += step) {
      const int64_t m = (t / n_tiles) * kBM + r;
      const bool row_ok = m < p.M;
      int iy0 = 0, ix0 = 0;
      const uint8_t* src[2] = {p.a[0], p.a[1]};
      if (row_ok) {
        const int64_t img = m / ohw;
        const int rem = (int)(m - img * ohw);
        const int oy = rem / p.OW, ox = rem - (rem / p.OW) * p.OW;
        iy0 = oy * p.SH - p.PH;
        ix0 = ox * p.SW - p.PW;
        const int64_t img_off = img * (int64_t)p.H * p.W * p.pix_stride;
        src[0] += img_off;
        src[1] += img_off;
      }
      for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
        const int s = (int)(g % S);
        if (g >= S && !wait(empty_bar(s), (uint32_t)(((g / S) - 1) & 1))) break;
        const int k0 = kb * kBKBytes;
        const int kend = p.K - k0 < kBKBytes ? p.K - k0 : kBKBytes;
        if (row_ok) {
          int tap = k0 / p.Cin;
          int c = k0 - tap * p.Cin;
          int ky = tap / p.KW, kx = tap - (tap / p.KW) * p.KW;
          for (int kk = 0; kk < kend; kk += kChunk) {
            const int iy = iy0 + ky * p.DH, ix = ix0 + kx * p.DW;
            const bool inside = iy >= 0 && iy < p.H && ix >= 0 && ix < p.W;
            const int off = (iy * p.W + ix) * pix_stride + c;
            const uint32_t soff =
                row_off + ((((uint32_t)kk >> 4) ^ sw) << 4) + ((uint32_t)kk & 15u);
#pragma unroll
            for (int pl = 0; pl < 2; ++pl) {
              const uint32_t dst = a_tile(s, pl) + soff;
              if (inside) {
                if (kChunk == 16)
                  ptx::cp_async_16(dst, src[pl] + off, 16);
                else
                  ptx::cp_async_4(dst, src[pl] + off, 4);
              } else if (p.pad_word[pl] != 0u) {
                // tap outside the image: the raw zero point (centred value 0)
                uint8_t* d = smem + (dst - base);
                if (kChunk == 16)
                  *reinterpret_cast<uint4*>(d) = make_uint4(p.pad_word[pl], p.pad_word[pl],
                                                            p.pad_word[pl], p.pad_word[pl]);
                else
                  *reinterpret_cast<uint32_t*>(d) = p.pad_word[pl];
              } else {
                if (kChunk == 16)
                  ptx::cp_async_16(dst, p.a[pl], 0);
                else
                  ptx::cp_async_4(dst, p.a[pl], 0);
              }
            }
            c += kChunk;
            if (c >= p.Cin) {
              c = 0;
              if (++kx == p.KW) {
                kx = 0;
                ++ky;
              }
            }
          }
          if (p.pad_word[0] | p.pad_word[1]) ptx::fence_proxy_async_smem();
        }
        ptx::cp_async_mbar_arrive_noinc(full_bar(s));
      }
      if (*s_abort) break;
    }
    ptx::cp_async_wait_all();
  } else if (warp == 5) {
    // ------------------------------------------------- weight TMA loads --
    if (lane == 0) {
      int64_t g = 0;
      for (int64_t t = first; t < total_tiles && !*s_abort; t += step) {
        const int n0 = (int)(t % n_tiles) * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
          const int s = (int)(g % S);
          if (g >= S && !wait(empty_bar(s), (uint32_t)(((g / S) - 1) & 1))) break;
          ptx::mbar_arrive_expect_tx(full_bar(s), kWP * L::kBPlane);
#pragma unroll
          for (int pl = 0; pl < kWP; ++pl)
            ptx::tma_load_2d(b_tile(s, pl), &tmap_b, full_bar(s), kb * kBKBytes,
                             pl * p.b_plane_rows + n0);
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      // descriptors formed once; a stage / plane / K-step offset moves only
      // the 14-bit start-address field (shared addresses stay below 256 KB)
      const uint64_t a_desc0 = ptx::smem_desc_sw128(a_tile(0, 0));
      const uint64_t b_desc0 = ptx::smem_desc_sw128(b_tile(0, 0));
      constexpr uint64_t kAPl = L::kAPlane >> 4, kBPl = L::kBPlane >> 4;
      // lo*lo (u8 x u8) -> acc 0; lo*hi, hi*lo -> acc 1; hi*hi (s8 x s8) -> acc 2
      constexpr uint32_t id_ll = ptx::idesc_i8(kBM, BN, 0, 0);
      constexpr uint32_t id_lh = ptx::idesc_i8(kBM, BN, 0, 1);
      constexpr uint32_t id_hl = ptx::idesc_i8(kBM, BN, 1, 0);
      constexpr uint32_t id_hh = ptx::idesc_i8(kBM, BN, 1, 1);
      int64_t g = 0, i = 0;
      for (int64_t t = first; t < total_tiles && !*s_abort; t += step, ++i) {
        const int b = L::kSets == 2 ? (int)(i & 1) : 0;
        const int64_t u = L::kSets == 2 ? (i >> 1) : i;  // earlier uses of set b
        if (u >= 1 && !wait(acce_bar(b), (uint32_t)((u - 1) & 1))) break;
        ptx::tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(b * L::kSetCols);
        for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
          const int s = (int)(g % S);
          if (!wait(full_bar(s), (uint32_t)((g / S) & 1))) break;
          ptx::tc_fence_after();
          const int krem = p.K - kb * kBKBytes;
          const int ksteps = krem >= kBKBytes ? kBKBytes / 32 : (krem + 31) / 32;
          const uint64_t so = (uint64_t)((uint32_t)(s * L::kStage) >> 4);
          const uint64_t al = a_desc0 + so, bl = b_desc0 + so;
#pragma unroll 4
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint64_t a0 = al + (uint64_t)(kk * 2), b0 = bl + (uint64_t)(kk * 2);
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            if constexpr (kWP == 2) {
              ptx::mma_i8(d0, a0, b0, id_ll, acc);
              ptx::mma_i8(d0 + BN, a0, b0 + kBPl, id_lh, acc);
              ptx::mma_i8(d0 + BN, a0 + kAPl, b0, id_hl, 1u);
              ptx::mma_i8(d0 + 2 * BN, a0 + kAPl, b0 + kBPl, id_hh, acc);
            } else {
              // weights b0 (u8), b1 (u8), b2 (s8): shift 0: lo*b0; 8: lo*b1 +
              // hi*b0; 16: lo*b2 + hi*b1; 24: hi*b2
              ptx::mma_i8(d0, a0, b0, id_ll, acc);
              ptx::mma_i8(d0 + BN, a0, b0 + kBPl, id_ll, acc);
              ptx::mma_i8(d0 + BN, a0 + kAPl, b0, id_hl, 1u);
              ptx::mma_i8(d0 + 2 * BN, a0, b0 + 2 * kBPl, id_lh, acc);
              ptx::mma_i8(d0 + 2 * BN, a0 + kAPl, b0 + kBPl, id_hl, 1u);
              ptx::mma_i8(d0 + 3 * BN, a0 + kAPl, b0 + 2 * kBPl, id_hh, acc);
            }
          }
          ptx::mma_commit(empty_bar(s));
        }
        ptx::mma_commit(accf_bar(b));
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    // two sets: warpgroup wg drains set wg (tiles wg, wg + 2, ...), all
    // columns; one set: both drain every tile, warpgroup wg half the columns
    const int wg = (warp - 6) / 4;
    const int b = L::kSets == 2 ? wg : 0;
    const int c_lo = L::kSets == 2 ? 0 : wg * (BN / 2);
    const int c_hi = L::kSets == 2 ? BN : c_lo + BN / 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int64_t istep = L::kSets == 2 ? 2 : 1;
    int64_t i = L::kSets == 2 ? wg : 0;
    for (int64_t t = first + i * step; t < total_tiles; t += istep * step, i += istep) {
      const int64_t u = L::kSets == 2 ? (i >> 1) : i;
      if (!wait(accf_bar(b), (uint32_t)(u & 1))) break;
      __syncwarp();
      ptx::tc_fence_after();
      const int64_t m = (t / n_tiles) * kBM + r;
      const int n_base = (int)(t % n_tiles) * BN;
      const bool row_ok = m < p.M;
      const uint32_t lane_base =
          tmem + (((uint32_t)quarter * 32u) << 16) + (uint32_t)(b * L::kSetCols);
#pragma unroll 1
      for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
        uint32_t v[L::kAccs][16];
#pragma unroll
        for (int a = 0; a < L::kAccs; ++a) ptx::tmem_ld16(lane_base + a * BN + c0, v[a]);
        ptx::tmem_ld_wait();
        const int nb = n_base + c0;
        const int cnt = p.n_valid - nb < 16 ? p.n_valid - nb : 16;
        if (!row_ok || cnt <= 0) continue;
        // each partial sum is exact in int32 (K * 255 * 255 < 2^31, host-
        // checked); the int64 combination is the reference's accumulator
        int64_t acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[j] = (int64_t)(int32_t)v[0][j] + (int64_t)(int32_t)v[1][j] * 256 +
                   (int64_t)(int32_t)v[2][j] * 65536;
          if constexpr (kWP == 3) acc[j] += (int64_t)(int32_t)v[3][j] * 16777216;
        }
        fused_epilogue_store16_run(p.epi, acc, m, nb, cnt, kSmemLut ? s_lut : nullptr,
                                   p.stage_params ? s_par + c0 : nullptr, par_all_hi);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(acce_bar(b));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, L::kTmemCols);
  }
}

template <int BN, int kChunk, bool kSmemLut, int kWP>
bool launch_umma16_persistent(const ConvTileParams& prm, const CUtensorMap& tmap,
                              int64_t n_tiles, cudaStream_t st) {
  auto kern = umma16_persistent_kernel<BN, kChunk, kSmemLut, kWP>;
  const size_t smem = P16Layout<BN, kSmemLut, kWP>::kSmem;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if (cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem),
                    "cudaFuncSetAttribute(smem)"))
      return false;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t m_tiles = (prm.M + kBM - 1) / kBM;
  const int64_t total = m_tiles * n_tiles;
  int64_t grid = total < sm_count() ? total : sm_count();
  // a grid that is a multiple of the column tiles keeps every CTA on one
  // column tile: its channel parameters are then staged once
  ConvTileParams prm2 = prm;
  const int64_t even = grid / n_tiles * n_tiles;
  if (even >= 1) {
    grid = even;
    prm2.stage_params = 1;
  }
  kern<<<(unsigned)grid, kP16Threads, smem, st>>>(prm2, tmap, n_tiles, total);
  return !cuda_failed(cudaGetLastError(), "umma16_persistent_kernel launch");
}


bool fill_fused_epilogue(FusedEpilogue& e, const qa_fused_conv_desc& d);  // qa_resident_ops.cu

namespace {

template <int kChunk, bool kSmemLut, int kWP>
bool launch_conv16_lut(int bn, const ConvTileParams& prm, const CUtensorMap& tmap,
                       int64_t n_tiles, cudaStream_t st) {
  switch (bn) {
    case 16: return launch_umma16_persistent<16, kChunk, kSmemLut, kWP>(prm, tmap, n_tiles, st);
    case 32: return launch_umma16_persistent<32, kChunk, kSmemLut, kWP>(prm, tmap, n_tiles, st);
    default:
      if constexpr (kWP == 3 && kSmemLut) {
        // three weight planes at BN 64 leave no room for the table
        set_error(kBadArgument, "qa_conv16_fused_dev: no shared-memory table at BN 64");
        return false;
      } else {
        return launch_umma16_persistent<64, kChunk, kSmemLut, kWP>(prm, tmap, n_tiles, st);
      }
  }
}

template <int kChunk, int kWP>
bool launch_conv16_bn(int bn, const ConvTileParams& prm, const CUtensorMap& tmap,
                      int64_t n_tiles, cudaStream_t st) {
  // BN = 128 keeps the table in global memory (see P16Layout)
  if (bn == 128)
    return launch_umma16_persistent<128, kChunk, false, kWP>(prm, tmap, n_tiles, st);
  // the kernel copies the table in 16-byte pieces; with three weight planes
  // only the narrow tiles leave room for it
  const bool smem_lut = prm.epi.lut && prm.epi.lut16 && prm.epi.lut_len <= kP16LutEntries &&
                        prm.epi.lut_len % 8 == 0 &&
                        (reinterpret_cast<uintptr_t>(prm.epi.lut16) & 15) == 0 &&
                        (kWP == 2 || bn <= 32);
  return smem_lut ? launch_conv16_lut<kChunk, true, kWP>(bn, prm, tmap, n_tiles, st)
                  : launch_conv16_lut<kChunk, false, kWP>(bn, prm, tmap, n_tiles, st);
}

}  // namespace

// Dense (groups == 1) 16-bit layer on the byte-split tensor-core kernel.
bool umma_conv16_fused(const qa_fused_conv16_desc& d16, cudaStream_t st) {
  const qa_fused_conv_desc& d = d16.base;
  const int64_t bn = d.block_n;
  const int64_t K = d.KH * d.KW * d.C;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(d.x);
  if (d.gap_sum) {
    set_error(kUnsupported, "qa_conv16_fused_dev: no fused GlobalAveragePool on 16-bit layers");
    return false;
  }
  if (bn != 16 && bn != 32 && bn != 64 && bn != 128) {
    set_error(kBadArgument, "qa_conv16_fused_dev: block_n must be 16, 32, 64 or 128");
    return false;
  }
  if (d.w_rows % bn || d.w_rows < d.Cout || d.w_kp % 16 || d.w_kp < K || !d.mult || !d.shift ||
      d.C % 4 || d.x_pix_stride % 4 || d.x_pix_stride < d.C || (xa & 3) ||
      (d16.x_plane & 3) || d.x_signed != 1 || (d.res && d.res_signed != 1)) {
    set_error(kBadArgument, "qa_conv16_fused_dev: bad layout");
    return false;
  }
  // each 8-bit partial product sum must stay exact in its int32 accumulator
  if (K * 255 * 255 >= (int64_t(1) << 31)) {
    set_error(kUnsupported, "qa_conv16_fused_dev: K too large for exact int32 partial sums");
    return false;
  }
  if (d.H * d.W * d.x_pix_stride >= (int64_t(1) << 31) || d.OH * d.OW >= (int64_t(1) << 31)) {
    set_error(kUnsupported, "qa_conv16_fused_dev: image too large");
    return false;
  }
  const int64_t M = d.N * d.OH * d.OW;
  if (M == 0 || d.Cout == 0) return true;
  ConvTileParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.a[0] = static_cast<const uint8_t*>(d.x);
  prm.a[1] = static_cast<const uint8_t*>(d.x) + d16.x_plane;
  prm.pix_stride = d.x_pix_stride;
  // out-of-image taps read the raw zero point (centred value 0), per plane
  prm.pad_word[0] = (uint32_t)(d.x_zp & 0xFF) * 0x01010101u;
  prm.pad_word[1] = (uint32_t)((d.x_zp >> 8) & 0xFF) * 0x01010101u;
  prm.H = (int32_t)d.H;
  prm.W = (int32_t)d.W;
  prm.Cin = (int32_t)d.C;
  prm.KH = (int32_t)d.KH;
  prm.KW = (int32_t)d.KW;
  prm.SH = (int32_t)d.SH;
  prm.SW = (int32_t)d.SW;
  prm.PH = (int32_t)d.PH;
  prm.PW = (int32_t)d.PW;
  prm.DH = (int32_t)d.DH;
  prm.DW = (int32_t)d.DW;
  prm.OH = (int32_t)d.OH;
  prm.OW = (int32_t)d.OW;
  prm.M = M;
  prm.K = (int32_t)K;
  prm.num_kb = (int32_t)((d.w_kp + kBKBytes - 1) / kBKBytes);
  prm.b_plane_rows = (int32_t)d.w_rows;
  prm.n_valid = (int32_t)d.Cout;
  prm.status = device_status_word();
  fill_fused_epilogue(prm.epi, d);
  prm.epi.res_plane = d16.res_plane;
  prm.epi.out_plane = d16.out_plane;
  prm.epi.out2_plane = d16.out2_plane;
  prm.epi.lut16 = d16.lut16;
  const int wp = d16.w_planes == 3 ? 3 : 2;
  if (d16.w_planes != 0 && d16.w_planes != 2 && d16.w_planes != 3) {
    set_error(kBadArgument, "qa_conv16_fused_dev: w_planes must be 2 or 3");
    return false;
  }
  CUtensorMap tmap;
  if (!make_weight_tmap(&tmap, d.w, wp * d.w_rows, d.w_kp, (int)bn)) return false;
  const bool wide = d.C % 16 == 0 && d.x_pix_stride % 16 == 0 && (xa & 15) == 0 &&
                    (d16.x_plane & 15) == 0;
  const int64_t n_tiles = d.w_rows / bn;
  if (wp == 3)
    return wide ? launch_conv16_bn<16, 3>((int)bn, prm, tmap, n_tiles, st)
                : launch_conv16_bn<4, 3>((int)bn, prm, tmap, n_tiles, st);
  return wide ? launch_conv16_bn<16, 2>((int)bn, prm, tmap, n_tiles, st)
              : launch_conv16_bn<4, 2>((int)bn, prm, tmap, n_tiles, st);
}

}  // namespace qa
