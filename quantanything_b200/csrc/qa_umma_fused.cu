// Persistent, warp-specialized fused 8-bit convolution / GEMM (tcgen05).
//
// One CTA per SM walks a strided list of 128-row output tiles of one
// column tile (all CTAs of a column tile share its weights).  Roles:
//   warps 0-3  thread gather (4- or 16-byte taps): one tile row per thread,
//              cp.async straight into the 128-byte swizzled K-major layout;
//              a ring of kStages 16 KB stages that runs ahead across tile
//              boundaries.  Layers fed by TMA use them as a third epilogue
//              warpgroup instead (BN >= 64);
//   warp 4     TMEM allocation; lane 0 issues tcgen05.mma (M=128, N=BN,
//              K=32) into one of the TMEM accumulators and commits;
//   warp 5     TMA loads: the weights once for the whole kernel when they
//              fit in shared memory (kResidentB), else one K-block per
//              stage; for TMA-fed layers also the activations (row tiles or
//              im2col slices, lanes 0-7 in one instruction);
//   warps 6-13 epilogue: drain the finished accumulator (the MMA meanwhile
//              fills the next one), apply the layer's integer sequence and
//              store 16-byte vectors of NHWC output.
// The K padding of every thread-gathered stage is zeroed once and never
// gathered again.  Every mbarrier wait is bounded (~2 s); a timeout sets the
// device status word, the CTA skips the remaining work, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/qa_kernels.h"
#include "qa_common.cuh"
#include "qa_fixedpoint.cuh"
#include "qa_ptx.cuh"
#include "qa_umma.cuh"

namespace qa {

bool make_weight_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                      int box_rows);
bool make_rows_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes,
                    int64_t row_stride, int box_rows);
bool fused_conv_grouped(const qa_fused_conv_desc& d, cudaStream_t st);
bool fill_fused_epilogue(FusedEpilogue& e, const qa_fused_conv_desc& d);

namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;                 // K-block bytes
constexpr int kProducers = 128;
constexpr int kEpilogueThreads = 128;    // one epilogue warpgroup
constexpr int kEpilogueWarp0 = 6;
constexpr uint64_t kBudgetCycles = 4000000000ull;  // ~2 s at 1.9 GHz
constexpr int kTimeoutCode = 0x7002;
// Byte-domain tables: every 8-bit value v in [-128, 255] at index v + 128.
constexpr int kTab = 384;

// Host-proven shortcuts of the epilogue's fixed-point steps.
struct FastFlags {
  int32_t requant;  // acc + bias fits int32, |M0| < 2^31, 1 <= ts <= 62
  int32_t add_tab;  // residual Add by two int32 tables is exact (|terms| < 2^29, sign = +-1)
  int32_t add64;    // both residual rescales: |v - z| * |m| + 2^(ts-1) < 2^62
  int32_t r64;      // concat copy rescale likewise
};

// One K-chunk of the implicit-GEMM row: tap displacement (dy, dx) and the
// byte offset of its first channel from the row's top-left input pixel;
// dy == kTapNone marks chunk positions beyond K.
struct TapEntry {
  int16_t dy, dx;
  int32_t delta;
};
constexpr int16_t kTapNone = -32768;

struct FusedParams {
  const uint8_t* a;
  int64_t pix_stride;
  uint32_t pad_word;
  int32_t a_signed;
  int32_t H, W, Cin, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW;
  int64_t M;
  int32_t K, num_kb;
  int32_t n_tap;   // chunk positions covered by the tap table (num_kb * 128 / chunk)
  int32_t slice;   // TMA gather: channel bytes per im2col load (16, 64 or 128)
  int32_t stable;  // every stage always holds the same K-block (kStages % num_kb == 0)
  int32_t n_valid;
  int32_t m_tiles, n_tiles;
  int32_t vec_ok;  // every output / residual base and stride is 16-byte aligned
  // border corrections of a nonzero input zero point under the TMA gather
  // (classes x Cout; NULL when none)
  const int32_t* pad_corr;
  const int32_t* pad_row_class;
  const int32_t* pad_col_class;
  int32_t pad_ncol, pad_classes;
  int32_t* status;
  FastFlags fast;
  FusedEpilogue epi;
  // GlobalAveragePool of this layer's output fused into the epilogue
  // (kGap): per (image, channel) sums of (v - gap_zp_in), per (image,
  // column tile) counts of the (row, column) contributions; the warp whose
  // contribution completes an (image, column tile) requantizes its pooled
  // values and zeroes the sums and the count again
  int32_t* gap_sum;  // [N][n_valid]
  int32_t* gap_cnt;  // [N][n_tiles]
  uint8_t* gap_out;
  int64_t gap_out_stride;
  int32_t gap_hw, gap_zp_in;
  int64_t gap_mult, gap_shift, gap_zp_out, gap_qmin, gap_qmax;
  int32_t gap_fast;  // (sum * M0 + 2^(ts-1)) >> ts is exact in 64 bits (host-proven)
};

__device__ __forceinline__ int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

__device__ __forceinline__ int64_t sbyte(uint32_t word, int j, int is_signed) {
  const uint32_t b = (word >> (8 * (j & 3))) & 0xFFu;
  return is_signed ? (int64_t)(int8_t)b : (int64_t)b;
}

__device__ __forceinline__ int32_t sbyte32(uint32_t word, int j, int is_signed) {
  return is_signed ? ((int32_t)(word << (24 - 8 * (j & 3))) >> 24)
                   : (int32_t)((word >> (8 * (j & 3))) & 0xFFu);
}

// Low bytes of four values, little-endian, in one word.
__device__ __forceinline__ uint32_t pack4(int32_t a, int32_t b, int32_t c, int32_t d) {
  return __byte_perm(__byte_perm((uint32_t)a, (uint32_t)b, 0x0040),
                     __byte_perm((uint32_t)c, (uint32_t)d, 0x0040), 0x5410);
}

// Four int32 values saturated to 8 bits (int8 or uint8) and packed
// little-endian: cvt.pack.sat gives sat(b) | sat(a) << 8 | c << 16.
__device__ __forceinline__ uint32_t pack_sat4(int32_t a, int32_t b, int32_t c, int32_t d,
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

template <int BN, int kChunk, bool kResidentB, int kStages>
struct Layout {
  static constexpr int kAStage = kBM * kBK;       // 16 KB
  static constexpr int kBBlock = BN * kBK;        // one K-block of weights
  // Two epilogue warpgroups.  With at least 32 columns both drain every
  // tile (group g its half of the columns); with 16 columns they alternate
  // tiles.  Accumulators: four when they fit in TMEM (BN <= 128), else two
  // (still double buffered).
  // Layers fed by TMA (kChunk <= 1) leave warps 0-3 free: with BN >= 64
  // they form a third group, so three groups split every tile's columns.
  static constexpr bool kTmaFed = kChunk <= 1;
  static constexpr int kGroups = (kTmaFed && BN >= 64) ? 3 : 2;
  static constexpr bool kSplit = BN >= 32;
  static constexpr int kAccs = BN <= 128 ? 4 : 2;
  static constexpr int kThreads = 192 + 2 * kEpilogueThreads;
  static constexpr int kCols = kAccs * BN;
  static constexpr int kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                 : kCols <= 256 ? 256 : 512;
};

// Exact (128-bit) forms, kept out of line: they run only for layers whose
// bounds the host could not prove for the 64-bit forms.
__device__ __noinline__ int64_t requant_exact_ool(int64_t x, int64_t m, int64_t s, int64_t zp,
                                                  int64_t lo, int64_t hi) {
  return requant_exact(x, m, s, zp, lo, hi);
}
__device__ __noinline__ int64_t add_exact_ool(int64_t a, int64_t q, const FusedEpilogue& e) {
  const I128 ta = mbqm(a - e.za, e.ma, e.sa);
  I128 tb = mbqm(q - e.zb, e.mb, e.sb);
  if (e.sign < 0) tb = neg_i128(tb);
  return clamp_i128(add_i128_i64(add_i128(ta, tb), e.add_zo), e.add_qmin, e.add_qmax);
}

// kChunk: bytes per gathered tap chunk of the thread gather (4 or 16), 1
// for a pointwise layer read as a row matrix by 2-D tiled TMA (one load per
// K-block, 128-byte swizzle), or 0
// for the TMA im2col gather (16-byte channel slices, no swizzle).
template <int BN, int kChunk, bool kResidentB, int kStages, bool kGap = false>
__global__ void __launch_bounds__((Layout<BN, kChunk, kResidentB, kStages>::kThreads), 1)
    fused_conv_persistent(const __grid_constant__ FusedParams p,
                          const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_a) {
  using L = Layout<BN, kChunk, kResidentB, kStages>;
  constexpr bool kTmaA = kChunk == 0;
  constexpr bool kTileA = kChunk == 1;
  constexpr int kTapBytes = (kTmaA || kTileA) ? 16 : kChunk;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);
  const int b_blocks = kResidentB ? p.num_kb : kStages;
  const uint32_t a_base = base;
  const uint32_t b_base = a_base + kStages * L::kAStage;
  uint8_t* tail = sm + kStages * L::kAStage + b_blocks * L::kBBlock;
  // per channel {bias, M0, 2^(sh-1), sh = ts - 32} of the high-word form
  int4* s_ch = reinterpret_cast<int4*>(tail);
  int64_t* s_bias = reinterpret_cast<int64_t*>(s_ch + BN);
  int64_t* s_mult = s_bias + BN;
  int64_t* s_shift = s_mult + BN;
  int64_t* s_rnd = s_shift + BN;                 // 2^(ts-1) of the 64-bit form
  int32_t* s_ts = reinterpret_cast<int32_t*>(s_rnd + BN);
  // byte-domain tables: activation, residual term a (+ zero point), residual
  // term b (signed), concat rescale
  int32_t* s_tab = s_ts + BN;
  int32_t* s_corr = s_tab + 4 * kTab;  // [pad_classes][BN] border corrections
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_corr + p.pad_classes * BN);
  // per K-chunk gather offsets, decoded once per CTA (after the barriers)
  TapEntry* s_tap = reinterpret_cast<TapEntry*>(bars + 3 * kStages + 2 * L::kAccs + 2);
  const uint32_t bar0 = ptx::smem_addr(bars);
  auto a_full = [&](int s) { return bar0 + 8u * s; };
  auto a_empty = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto b_full = [&](int s) { return bar0 + 8u * (2 * kStages + s); };
  const uint32_t acc_full0 = bar0 + 8u * (3 * kStages);
  const uint32_t acc_empty0 = acc_full0 + 8u * L::kAccs;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 3 * kStages + 2 * L::kAccs);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  ptx::pdl_launch_dependents();
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  int hi_ok = 1;  // this thread's channels all admit the high-word requantize
  const int n_tile = blockIdx.x % p.n_tiles;
  const int m_first = blockIdx.x / p.n_tiles;
  const int m_step = gridDim.x / p.n_tiles;
  const int n0 = n_tile * BN;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(a_full(s), (kTmaA || kTileA) ? 1 : kProducers);
      ptx::mbar_init(a_empty(s), 1);
      ptx::mbar_init(b_full(s), 1);
    }
    for (int b = 0; b < L::kAccs; ++b) {
      ptx::mbar_init(acc_full0 + 8u * b, 1);
      ptx::mbar_init(acc_empty0 + 8u * b,
                     L::kSplit ? L::kGroups * kEpilogueThreads : kEpilogueThreads);
    }
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc(ptx::smem_addr(s_tmem), L::kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 5 && lane == 0) {
    ptx::prefetch_tmap(&tmap_b);
    if (kTmaA || kTileA) ptx::prefetch_tmap(&tmap_a);
  }
  if (warp < 4) {
    if (!kTmaA && !kTileA) {
      // zero every activation stage once: the K padding is never gathered
      // (the TMA gather leaves it stale: it meets zero weight columns)
      uint4* z = reinterpret_cast<uint4*>(sm);
      for (int i = tid; i < kStages * L::kAStage / 16; i += kProducers) z[i] = make_uint4(0, 0, 0, 0);
      ptx::fence_proxy_async_smem();
    }
    const int tap_bytes = kTmaA ? p.slice : kTapBytes;
    for (int i = tid; i < p.n_tap; i += kProducers) {
      const int k = i * tap_bytes;
      TapEntry t{kTapNone, 0, 0};
      if (k < p.K) {
        const int tap = k / p.Cin, c = k - (k / p.Cin) * p.Cin;
        const int ky = tap / p.KW, kx = tap - (tap / p.KW) * p.KW;
        const int dy = ky * p.DH, dx = kx * p.DW;
        // the TMA gather needs the channel offset, the thread gather the
        // byte offset from the row's top-left input pixel
        t = TapEntry{(int16_t)dy, (int16_t)dx,
                     kTmaA ? (int32_t)c : (int32_t)((dy * p.W + dx) * p.pix_stride + c)};
      }
      s_tap[i] = t;
    }
  } else if (warp >= kEpilogueWarp0) {
    const FusedEpilogue& e = p.epi;
    const int et = tid - kEpilogueWarp0 * 32, nthreads = 2 * kEpilogueThreads;
    for (int c = et; c < BN; c += nthreads) {
      const int n = n0 + c;
      const bool v = n < p.n_valid;
      s_bias[c] = (v && e.bias) ? e.bias[n] : 0;
      s_mult[c] = v ? e.mult[n] : 0;
      s_shift[c] = v ? e.shift[n] : 0;
      const int ts = (int)(31 + s_shift[c]);
      s_ts[c] = ts;
      s_rnd[c] = (ts >= 1 && ts <= 62) ? ((int64_t)1 << (ts - 1)) : 0;
      // (x * M0 + 2^(ts-1)) >> ts == (hi32(x * M0) + 2^(ts-33)) >> (ts - 32)
      // for ts in [33, 62]: the low word cannot carry into the rounding.
      // The output zero point rides in the rounding term (z * 2^sh added
      // before the arithmetic shift adds z after it) while the sum stays
      // in int32: |hi32| < 2^30.
      const bool hi0 = ts >= 33 && ts <= 62;
      const int sh = hi0 ? ts - 32 : 1;
      const int64_t zfold = e.zp * ((int64_t)1 << sh);
      const bool hi = hi0 && e.zp > -(1 << 20) && e.zp < (1 << 20) &&
                      (zfold < 0 ? -zfold : zfold) + ((int64_t)1 << (sh - 1)) < ((int64_t)1 << 30);
      if (v && !hi) hi_ok = 0;
      s_ch[c] = make_int4((int32_t)s_bias[c], (int32_t)s_mult[c],
                          (int32_t)(((int64_t)1 << (sh - 1)) + (hi ? zfold : 0)), sh);
    }
    for (int i = et; i < p.pad_classes * BN; i += nthreads) {
      const int cls = i / BN, n = n0 + (i - cls * BN);
      s_corr[i] = n < p.n_valid ? p.pad_corr[(int64_t)cls * p.n_valid + n] : 0;
    }
    // Every value the epilogue carries between steps is an 8-bit one (the
    // host checks the clamp ranges), so each step after the requantize is a
    // lookup in a table over [-128, 255].
    const bool add_tab = e.res && p.fast.add_tab;
    const int tsa = (int)(31 + e.sa), tsb = (int)(31 + e.sb), tsr = (int)(31 + e.r_s);
    for (int i = et; i < kTab; i += nthreads) {
      const int64_t v = i - 128;
      if (e.lut) {
        const int64_t idx = clamp64(v - e.lut_offset, 0, e.lut_len - 1);
        s_tab[i] = (int32_t)clamp64(e.lut[idx], -128, 255);
      }
      if (add_tab) {
        int64_t ta, tb;
        if (p.fast.add64) {
          ta = ((v - e.za) * e.ma + ((int64_t)1 << (tsa - 1))) >> tsa;
          tb = ((v - e.zb) * e.mb + ((int64_t)1 << (tsb - 1))) >> tsb;
        } else {
          ta = clamp_i128(mbqm(v - e.za, e.ma, e.sa), -(int64_t(1) << 40), int64_t(1) << 40);
          tb = clamp_i128(mbqm(v - e.zb, e.mb, e.sb), -(int64_t(1) << 40), int64_t(1) << 40);
        }
        s_tab[kTab + i] = (int32_t)(ta + e.add_zo);
        s_tab[2 * kTab + i] = (int32_t)(e.sign * tb);
      }
      if (e.out2) {
        int64_t r;
        if (e.r_identity) r = clamp64(v, e.r_qmin, e.r_qmax);
        else if (p.fast.r64)
          r = clamp64(((((v - e.r_zp_in) * e.r_m) + ((int64_t)1 << (tsr - 1))) >> tsr) + e.r_zp_out,
                      e.r_qmin, e.r_qmax);
        else r = requant_exact(v - e.r_zp_in, e.r_m, e.r_s, e.r_zp_out, e.r_qmin, e.r_qmax);
        s_tab[3 * kTab + i] = (int32_t)r;
      }
    }
  }
  ptx::tc_fence_before();
  const int hi_all = __syncthreads_and(hi_ok);
  ptx::tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // Static weights may stream in while the previous layer finishes; its
  // outputs (this layer's activations) are read only after pdl_wait.
  if (kResidentB && warp == 5 && lane == 0) {
    ptx::mbar_arrive_expect_tx(b_full(0), (uint32_t)(p.num_kb * L::kBBlock));
    for (int kb = 0; kb < p.num_kb; ++kb)
      ptx::tma_load_2d(b_base + kb * L::kBBlock, &tmap_b, b_full(0), kb * kBK, n0);
  }
  ptx::pdl_wait();

  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (ptx::mbar_wait_sleep(bar, parity, kBudgetCycles)) return true;
    *s_abort = 1;
    if (p.status) atomicExch(p.status, kTimeoutCode);
    return false;
  };

  if (!L::kTmaFed && warp < 4) {
    // --------------------------------------------------- activation gather --
    // Thread r owns tile row r: one output pixel whose receptive field it
    // gathers K-chunk by K-chunk using the decoded tap table (32-bit math).
    const int r = tid;
    const uint32_t row_off = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    const uint32_t sw = (uint32_t)(r & 7);
    const int ohw = p.OH * p.OW;
    constexpr int kPerBlock = kBK / kTapBytes;
    int g = 0;  // K-blocks issued by this CTA
    for (int mt = m_first; mt < p.m_tiles; mt += m_step) {
      const int m = mt * kBM + r;
      const bool row_ok = m < p.M;
      int iy0 = 0, ix0 = 0;
      const uint8_t* row_base = p.a;
      if (row_ok) {
        const int img = m / ohw, rem = m - (m / ohw) * ohw;
        const int oy = rem / p.OW, ox = rem - (rem / p.OW) * p.OW;
        iy0 = oy * p.SH - p.PH;
        ix0 = ox * p.SW - p.PW;
        row_base = p.a + ((int64_t)img * p.H * p.W + (int64_t)iy0 * p.W + ix0) * p.pix_stride;
      }
      for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
        const int s = g % kStages;
        if (g >= kStages) wait(a_empty(s), ((g / kStages) - 1) & 1);
        const bool live = !*s_abort;
        const int kend = min(kBK, p.K - kb * kBK);
        // bytes [kend, kpad) are read by the last 32-byte MMA step: zero them
        // (a stage may have held a fuller K-block of another tile before)
        // (not needed when each stage always holds this same K-block: its
        // padding stays zero from the initial clear)
        const int npos = (p.stable ? kend : min(kBK, (kend + 31) & ~31)) / kTapBytes;
        const TapEntry* tap = s_tap + kb * kPerBlock;
        const uint32_t stage = a_base + s * L::kAStage + row_off;
        bool wrote_generic = false;
        if (live) {
#pragma unroll 4
          for (int jpos = 0; jpos < npos; ++jpos) {
            const TapEntry t = tap[jpos];
            const int kk = jpos * kChunk;
            const uint32_t dst = stage + ((((uint32_t)kk >> 4) ^ sw) << 4) + ((uint32_t)kk & 15u);
            const bool in_k = t.dy != kTapNone;
            const bool inside = row_ok && in_k && (unsigned)(iy0 + t.dy) < (unsigned)p.H &&
                                (unsigned)(ix0 + t.dx) < (unsigned)p.W;
            if (inside) {
              if (kChunk == 16) ptx::cp_async_16(dst, row_base + t.delta, 16);
              else ptx::cp_async_4(dst, row_base + t.delta, 4);
            } else if (in_k && row_ok && p.pad_word) {
              wrote_generic = true;
              uint8_t* d = sm + (dst - base);
              if (kChunk == 16)
                *reinterpret_cast<uint4*>(d) = make_uint4(p.pad_word, p.pad_word, p.pad_word,
                                                          p.pad_word);
              else
                *reinterpret_cast<uint32_t*>(d) = p.pad_word;
            } else {
              if (kChunk == 16) ptx::cp_async_16(dst, p.a, 0);
              else ptx::cp_async_4(dst, p.a, 0);
            }
          }
        }
        // zero-point padding written with plain stores must reach the async
        // proxy; copies are tracked by the barrier itself
        if (wrote_generic) ptx::fence_proxy_async_smem();
        ptx::cp_async_mbar_arrive_noinc(a_full(s));
      }
    }
    ptx::cp_async_wait_all();
  } else if (warp == 5 && L::kTmaFed) {
    // ------------------------------------------ activation + weight loads --
    // Lanes 0-7, converged: per K-block, lane 0 posts the stage's byte
    // counts and loads the weights' K-block (when they are not resident);
    // the activations come as one 2-D load of 128 rows x 128 bytes in the
    // 128-byte swizzle (row TMA: bytes past C and rows past M read 0), or
    // as one im2col load per channel slice of a tap (lane i: slice i) that
    // brings the slice for all 128 output pixels of the tile: 16-byte slices
    // as rows of 16 bytes (slice i at byte 2048 * i), 64- and 128-byte
    // slices in the 64- / 128-byte swizzle (slice i at byte 128 * slice * i).
    const int sl = kTileA ? kBK : p.slice, per_kb = kBK / sl;
    if (lane < per_kb) {
      const int ohw = p.OH * p.OW;
      int g = 0;
      for (int mt = m_first; mt < p.m_tiles && !*s_abort; mt += m_step) {
        const int m0 = mt * kBM;
        const int img = m0 / ohw, rem = m0 - img * ohw;
        const int oy = rem / p.OW, ox = rem - oy * p.OW;
        const int w0 = ox * p.SW - p.PW, h0 = oy * p.SH - p.PH;
        for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !wait(a_empty(s), ((g / kStages) - 1) & 1)) break;
          if (!kResidentB && lane == 0) {
            ptx::mbar_arrive_expect_tx(b_full(s), (uint32_t)L::kBBlock);
            ptx::tma_load_2d(b_base + s * L::kBBlock, &tmap_b, b_full(s), kb * kBK, n0);
          }
          if (kTileA) {
            if (lane == 0) {
              ptx::mbar_arrive_expect_tx(a_full(s), (uint32_t)L::kAStage);
              ptx::tma_load_2d(a_base + s * L::kAStage, &tmap_a, a_full(s), kb * kBK, m0);
            }
          } else {
            const int nsl = min(per_kb, (p.K - kb * kBK + sl - 1) / sl);
            if (lane == 0) ptx::mbar_arrive_expect_tx(a_full(s), (uint32_t)(nsl * kBM * sl));
            if (lane < nsl) {
              const TapEntry t = s_tap[kb * per_kb + lane];
              ptx::tma_load_im2col_4d(a_base + s * L::kAStage + lane * (kBM * sl), &tmap_a,
                                      a_full(s), t.delta, w0, h0, img, (uint16_t)t.dx,
                                      (uint16_t)t.dy);
            }
          }
        }
      }
      // after an abort, wait (bounded) for the loads still in flight
      if (*s_abort && lane == 0) {
        for (int gg = max(0, g - kStages); gg < g; ++gg) {
          ptx::mbar_wait(a_full(gg % kStages), (gg / kStages) & 1, kBudgetCycles);
          if (!kResidentB)
            ptx::mbar_wait(b_full(gg % kStages), (gg / kStages) & 1, kBudgetCycles);
        }
        if (kResidentB) ptx::mbar_wait(b_full(0), 0, kBudgetCycles);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------ weight loads --
    if (lane == 0) {
      if (!kResidentB) {
        int g = 0;
        for (int mt = m_first; mt < p.m_tiles; mt += m_step) {
          for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
            const int s = g % kStages;
            if (g >= kStages && !wait(a_empty(s), ((g / kStages) - 1) & 1)) break;
            ptx::mbar_arrive_expect_tx(b_full(s), (uint32_t)L::kBBlock);
            ptx::tma_load_2d(b_base + s * L::kBBlock, &tmap_b, b_full(s), kb * kBK, n0);
          }
          if (*s_abort) break;
        }
        // after an abort, wait (bounded) for the loads still in flight
        if (*s_abort)
          for (int gg = max(0, g - kStages); gg < g; ++gg)
            ptx::mbar_wait(b_full(gg % kStages), (gg / kStages) & 1, kBudgetCycles);
      } else if (*s_abort) {
        ptx::mbar_wait(b_full(0), 0, kBudgetCycles);
      }
    }
  } else if (warp == 4) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_i8(kBM, BN, p.a_signed, 1);
      // A operand layouts: TMA gather with 16-byte slices (2048 bytes apart
      // along K, 8-row groups 128 bytes apart), 64-byte slices (8 KB apart,
      // 64-byte swizzle); row TMA / thread gather / 128-byte slices: 128-byte
      // swizzle.  a_off[kk]: the K-step's offset in 16-byte units.
      const int slice = kTmaA ? p.slice : 128;
      const uint64_t a_desc0 = slice == 16   ? ptx::smem_desc_kmajor_plain(a_base, kBM * 16, 128)
                               : slice == 64 ? ptx::smem_desc_sw64(a_base)
                                             : ptx::smem_desc_sw128(a_base);
      uint32_t a_off[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        a_off[kk] = (slice == 16   ? kk * 2 * (kBM * 16)
                     : slice == 64 ? (kk >> 1) * (kBM * 64) + (kk & 1) * 32
                                   : kk * 32) >> 4;
      const uint64_t b_desc0 = ptx::smem_desc_sw128(b_base);
      bool ok = true;
      if (kResidentB) ok = wait(b_full(0), 0);
      int g = 0, j = 0;
      for (int mt = m_first; ok && mt < p.m_tiles; mt += m_step, ++j) {
        const int ab = j % L::kAccs;
        const int use = j / L::kAccs;  // how often this accumulator was used before
        if (use >= 1 && !wait(acc_empty0 + 8u * ab, (use - 1) & 1)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem + ab * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1;
          if (!wait(a_full(s), ph)) { ok = false; break; }
          if (!kResidentB && !wait(b_full(s), ph)) { ok = false; break; }
          ptx::tc_fence_after();
          const int ksteps = (min(kBK, p.K - kb * kBK) + 31) / 32;
          // descriptors of this stage: the bases plus the stage offset (in
          // 16-byte units: the start-address field), then the K-steps'
          // offsets, so that the MMAs leave back to back
          const uint64_t ad = a_desc0 + (uint64_t)((uint32_t)(s * L::kAStage) >> 4);
          const uint64_t bd =
              b_desc0 + (uint64_t)((uint32_t)((kResidentB ? kb : s) * L::kBBlock) >> 4);
          const uint32_t acc0 = kb > 0 ? 1u : 0u;
          if (ksteps == 4) {
            ptx::mma_i8(d_tmem, ad + a_off[0], bd, idesc, acc0);
            ptx::mma_i8(d_tmem, ad + a_off[1], bd + 2, idesc, 1u);
            ptx::mma_i8(d_tmem, ad + a_off[2], bd + 4, idesc, 1u);
            ptx::mma_i8(d_tmem, ad + a_off[3], bd + 6, idesc, 1u);
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              if (kk < ksteps)
                ptx::mma_i8(d_tmem, ad + a_off[kk], bd + 2 * kk, idesc, (acc0 | kk) ? 1u : 0u);
          }
          ptx::mma_commit(a_empty(s));
        }
        if (!ok) break;
        ptx::mma_commit(acc_full0 + 8u * ab);
      }
    }
  } else if (warp >= kEpilogueWarp0 || (L::kGroups == 3 && warp < 4)) {
    // ---------------------------------------------------------- epilogue --
    // With kSplit, warpgroup `grp` drains its share of every tile's
    // 16-column chunks; otherwise the tiles j with j % kGroups == grp.
    // Each thread owns one tile row;
    // per 16-column chunk the layer-uniform branches are hoisted out of the
    // unrolled element loops, and the next chunk's TMEM load is in flight
    // while this one is processed.
    const FusedEpilogue& e = p.epi;
    const int grp = warp < 4 ? 2 : (warp - kEpilogueWarp0) / 4;
    // this group's share of the tile's 16-column chunks (kSplit)
    const int g_lo = grp * (BN / 16) / L::kGroups, g_hi = (grp + 1) * (BN / 16) / L::kGroups;
    const int gcols = L::kSplit ? (g_hi - g_lo) * 16 : BN;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter.. belong to this warp
    const int r = quarter * 32 + lane;
    const bool fast_rq = p.fast.requant;
    const bool hi_rq = fast_rq && hi_all;
    // plain requantize to the full 8-bit range: clamp and pack in one step
    // (streamed-weight variants only: the resident ones are at their
    // register limit)
    const bool pack_sat = !kGap && !kResidentB && hi_rq && !e.lut && !e.res && !e.out2 &&
                          ((e.qmin == 0 && e.qmax == 255) || (e.qmin == -128 && e.qmax == 127));
    const bool pack_signed = e.qmin < 0;
    const bool has_lut = e.lut != nullptr, add_tab = p.fast.add_tab;
    const int32_t zp32 = (int32_t)e.zp, qmin32 = (int32_t)e.qmin, qmax32 = (int32_t)e.qmax;
    const int32_t aqmin32 = (int32_t)e.add_qmin, aqmax32 = (int32_t)e.add_qmax;
    const int32_t* t_lut = s_tab + 128;
    const int32_t* t_a = s_tab + kTab + 128;
    const int32_t* t_b = s_tab + 2 * kTab + 128;
    const int32_t* t_r = s_tab + 3 * kTab + 128;
    // Everything the tile loop reads from the parameters, read once: the
    // parameter block is reached through a generic pointer here, and every
    // such read is a long-latency load.
    const uint8_t* const res_p = e.res;
    const int64_t res_stride = e.res_pix_stride;
    const int res_signed = (int)e.res_signed;
    uint8_t* const out_p = e.out;
    const int64_t out_stride = e.out_pix_stride;
    uint8_t* const out2_p = e.out2;
    const int64_t out2_stride = e.out2_pix_stride;
    const int n_valid = p.n_valid;
    const bool vec_ok = p.vec_ok != 0;
    const bool pad_corr = p.pad_corr != nullptr;
    const int64_t M = p.M;
    int32_t* const gap_sum = p.gap_sum;
    const int gap_hw = p.gap_hw, gap_zp = p.gap_zp_in;
    int j = 0;
    for (int mt = m_first; mt < p.m_tiles; mt += m_step, ++j) {
      if (!L::kSplit && j % L::kGroups != grp) continue;
      const int cbase = L::kSplit ? g_lo * 16 : 0;
      const int ab = j % L::kAccs;
      const int use = j / L::kAccs;
      const bool ok = wait(acc_full0 + 8u * ab, use & 1);
      __syncwarp();
      ptx::tc_fence_after();
      const int64_t m = (int64_t)mt * kBM + r;
      const bool row_ok = ok && m < M;
      // fused GlobalAveragePool: this row's image (rows fit 32 bits) and the
      // warp's first image; the warp's rows span at most two images
      int gimg = -1, gimg0 = -1;
      bool gtwo = false;
      if constexpr (kGap) {
        gimg = row_ok ? (int)((uint32_t)m / (uint32_t)gap_hw) : -1;
        gimg0 = __shfl_sync(0xffffffffu, gimg, 0);
        gtwo = __any_sync(0xffffffffu, gimg >= 0 && gimg != gimg0);
      }
      // border class of this output pixel (nonzero input zero point with
      // out-of-image taps read as 0 by the TMA gather)
      const int32_t* corr = nullptr;
      if (pad_corr && row_ok) {
        const int ohw = p.OH * p.OW;
        const int rem = (int)(m % ohw), oy = rem / p.OW, ox = rem - oy * p.OW;
        corr = s_corr + (p.pad_row_class[oy] * p.pad_ncol + p.pad_col_class[ox]) * BN + cbase;
      }
      // this row's first output channel in each destination
      const uint8_t* const res_row = res_p + m * res_stride + n0 + cbase;
      uint8_t* const out_row = out_p + m * out_stride + n0 + cbase;
      uint8_t* const out2_row = out2_p + m * out2_stride + n0 + cbase;
      const uint32_t lane_base = tmem + (((uint32_t)quarter * 32u) << 16) + ab * BN + cbase;
      uint32_t v[16], vn[16];
      ptx::tmem_ld16(lane_base, v);
      ptx::tmem_ld_wait(v);
#pragma unroll 1
      for (int c0 = 0; c0 < gcols; c0 += 16) {
        const int cc = cbase + c0;  // tile column of this chunk
        const bool more = c0 + 16 < gcols;
        if (more) ptx::tmem_ld16(lane_base + c0 + 16, vn);
        int32_t gq[16];  // pooled contributions v - gap_zp of this chunk (kGap)
        if constexpr (kGap) {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) gq[jj] = 0;
        }
        if (row_ok && n0 + cc < n_valid) {
          const int nval = min(16, n_valid - (n0 + cc));
          if (corr) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v[jj] += (uint32_t)corr[c0 + jj];
          }
          const bool vec = vec_ok && nval == 16;
          int32_t q[16];
          if (pack_sat) {
            int32_t t[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int4 ch = s_ch[cc + jj];
              t[jj] = (__mulhi((int32_t)v[jj] + ch.x, ch.y) + ch.z) >> ch.w;
            }
            uint32_t o[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              o[k4] = pack_sat4(t[4 * k4], t[4 * k4 + 1], t[4 * k4 + 2], t[4 * k4 + 3],
                                pack_signed);
            uint8_t* op = out_row + c0;
            if (vec) {
              *reinterpret_cast<uint4*>(op) = make_uint4(o[0], o[1], o[2], o[3]);
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                if (jj < nval) op[jj] = (uint8_t)(o[jj >> 2] >> (8 * (jj & 3)));
            }
          } else {
          // requantize
          if (hi_rq) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int4 ch = s_ch[cc + jj];
              const int32_t x = (int32_t)v[jj] + ch.x;
              const int32_t t = (__mulhi(x, ch.y) + ch.z) >> ch.w;  // zero point included
              q[jj] = min(max(t, qmin32), qmax32);
            }
          } else if (fast_rq) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int c = cc + jj;
              const int32_t x = (int32_t)v[jj] + s_ch[c].x;
              const int64_t r64 = ((int64_t)x * (int64_t)s_ch[c].y + s_rnd[c]) >> s_ts[c];
              q[jj] = (int32_t)clamp64(r64 + e.zp, e.qmin, e.qmax);
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int c = cc + jj;
              q[jj] = (int32_t)requant_exact_ool((int64_t)(int32_t)v[jj] + s_bias[c], s_mult[c],
                                                 s_shift[c], e.zp, e.qmin, e.qmax);
            }
          }
          // activation table
          if (has_lut) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) q[jj] = t_lut[q[jj]];
          }
          // residual add: out = res (operand a) + sign * ours (operand b)
          if (res_p) {
            const uint8_t* rp = res_row + c0;
            uint32_t w[4];
            if (vec) {
              const uint4 rv = *reinterpret_cast<const uint4*>(rp);
              w[0] = rv.x; w[1] = rv.y; w[2] = rv.z; w[3] = rv.w;
            } else {
#pragma unroll
              for (int k4 = 0; k4 < 4; ++k4) {
                uint32_t acc = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b)
                  if (k4 * 4 + b < nval) acc |= (uint32_t)rp[k4 * 4 + b] << (8 * b);
                w[k4] = acc;
              }
            }
            if (add_tab) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const int32_t a = sbyte32(w[jj >> 2], jj, res_signed);
                q[jj] = min(max(t_a[a] + t_b[q[jj]], aqmin32), aqmax32);
              }
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                q[jj] = (int32_t)add_exact_ool(sbyte(w[jj >> 2], jj, res_signed), q[jj], e);
            }
          }
          if constexpr (kGap) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) gq[jj] = jj < nval ? q[jj] - gap_zp : 0;
          }
          // primary store
          if (out_p) {
            uint32_t o[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              o[k4] = pack4(q[4 * k4], q[4 * k4 + 1], q[4 * k4 + 2], q[4 * k4 + 3]);
            uint8_t* op = out_row + c0;
            if (vec) {
              *reinterpret_cast<uint4*>(op) = make_uint4(o[0], o[1], o[2], o[3]);
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                if (jj < nval) op[jj] = (uint8_t)(o[jj >> 2] >> (8 * (jj & 3)));
            }
          }
          // rescaled copy into a Concat slice
          if (out2_p) {
            uint32_t o[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              o[k4] = pack4(t_r[q[4 * k4]], t_r[q[4 * k4 + 1]], t_r[q[4 * k4 + 2]],
                            t_r[q[4 * k4 + 3]]);
            uint8_t* op = out2_row + c0;
            if (vec) {
              *reinterpret_cast<uint4*>(op) = make_uint4(o[0], o[1], o[2], o[3]);
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                if (jj < nval) op[jj] = (uint8_t)(o[jj >> 2] >> (8 * (jj & 3)));
            }
          }
          }  // requantize with table steps
        }
        if constexpr (kGap) {
          // the warp's 32 rows span at most two images (gap_hw >= 32, host-
          // checked): one sum per image and column, added by lane jj
          if (n0 + cc < n_valid && gimg0 >= 0) {
            const bool first = gimg == gimg0;
            int32_t mine0 = 0, mine1 = 0;
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int32_t s0 = __reduce_add_sync(0xffffffffu, first ? gq[jj] : 0);
              if (lane == jj) mine0 = s0;
            }
            if (gtwo) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const int32_t s1 = __reduce_add_sync(0xffffffffu, first ? 0 : gq[jj]);
                if (lane == jj) mine1 = s1;
              }
            }
            const int nv = min(16, n_valid - (n0 + cc));
            if (lane < nv) {
              int32_t* sp = gap_sum + (int64_t)gimg0 * n_valid + n0 + cc + lane;
              if (mine0) atomicAdd(sp, mine0);
              if (gtwo && mine1) atomicAdd(sp + n_valid, mine1);
            }
          }
        }
        if (more) {
          ptx::tmem_ld_wait(vn);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) v[jj] = vn[jj];
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(acc_empty0 + 8u * ab);
      if constexpr (kGap) {
        // count this warp's (row, column) contributions per image; the warp
        // that completes an (image, column tile) pools it
        const int img0 = gimg0;
        const int rows0 = __popc(__ballot_sync(0xffffffffu, gimg >= 0 && gimg == img0));
        const int rows1 = __popc(__ballot_sync(0xffffffffu, gimg >= 0 && gimg != img0));
        const int tile_cols = min(BN, n_valid - n0);
        const int my_cols = max(0, min(gcols, n_valid - (n0 + cbase)));
        const int target = gap_hw * tile_cols;
        int fin = 0;
        __threadfence();
        if (lane == 0 && img0 >= 0 && my_cols > 0) {
          int32_t* cp = p.gap_cnt + (int64_t)img0 * p.n_tiles + n_tile;
          if (rows0 && atomicAdd(cp, rows0 * my_cols) + rows0 * my_cols == target) fin |= 1;
          if (rows1 && atomicAdd(cp + p.n_tiles, rows1 * my_cols) + rows1 * my_cols == target)
            fin |= 2;
        }
        fin = __shfl_sync(0xffffffffu, fin, 0);
        for (int k = 0; k < 2; ++k) {
          if (!((fin >> k) & 1)) continue;
          const int im = img0 + k;
          __threadfence();
          // every sum of this (image, column tile) is complete in L2: read
          // them all at once (L2-coherent loads), pool, zero them again
          int32_t* const srow = gap_sum + (int64_t)im * n_valid + n0;
          int32_t sv[BN / 32];
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) {
            const int c = lane + 32 * i;
            sv[i] = c < tile_cols ? __ldcg(srow + c) : 0;
          }
          uint8_t* const orow = p.gap_out + (int64_t)im * p.gap_out_stride + n0;
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) {
            const int c = lane + 32 * i;
            if (c >= tile_cols) continue;
            int64_t q;
            if (p.gap_fast) {
              const int ts = 31 + (int)p.gap_shift;
              q = clamp64((((int64_t)sv[i] * p.gap_mult + (int64_t(1) << (ts - 1))) >> ts) +
                              p.gap_zp_out,
                          p.gap_qmin, p.gap_qmax);
            } else {
              q = requant_exact_ool(sv[i], p.gap_mult, p.gap_shift, p.gap_zp_out, p.gap_qmin,
                                    p.gap_qmax);
            }
            orow[c] = (uint8_t)q;
            __stcg(srow + c, 0);
          }
          if (lane == 0) __stcg(p.gap_cnt + (int64_t)im * p.n_tiles + n_tile, 0);
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, L::kTmemCols);
  }
}

template <int BN, int kChunk, bool kResidentB, int kStages>
size_t smem_bytes(int num_kb, int pad_classes) {
  using L = Layout<BN, kChunk, kResidentB, kStages>;
  const int b_blocks = kResidentB ? num_kb : kStages;
  return 1024 + (size_t)kStages * L::kAStage + (size_t)b_blocks * L::kBBlock + BN * 16 +
         4 * BN * 8 + BN * 4 + 4 * kTab * 4 + (size_t)pad_classes * BN * 4 +
         (3 * kStages + 2 * L::kAccs + 2) * 8 +
         (size_t)num_kb * (kBK / (kChunk <= 1 ? 16 : kChunk)) * sizeof(TapEntry);
}

constexpr int kStagesFused = 4;
constexpr size_t kSmemCap = 227 * 1024;

template <int BN, int kChunk, bool kResidentB, int kStages, bool kGap = false>
bool launch_persistent(const FusedParams& prm_in, const CUtensorMap& tmap,
                       const CUtensorMap& tmap_a, cudaStream_t st) {
  auto kern = fused_conv_persistent<BN, kChunk, kResidentB, kStages, kGap>;
  const size_t smem = smem_bytes<BN, kChunk, kResidentB, kStages>(prm_in.num_kb,
                                                                   prm_in.pad_classes);
  FusedParams prm = prm_in;
  prm.stable = (kStages % prm.num_kb) == 0;
  static size_t attr_bytes[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || attr_bytes[dev] < smem) {
    if (cuda_failed(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem),
                    "cudaFuncSetAttribute(smem)"))
      return false;
    if (dev >= 0 && dev < 64) attr_bytes[dev] = smem;
  }
  const int64_t sms = sm_count();
  int64_t per_n = sms / prm.n_tiles;
  if (per_n < 1) per_n = 1;
  if (per_n > prm.m_tiles) per_n = prm.m_tiles;
  const int64_t grid = per_n * prm.n_tiles;
  return launch_ex(kern, dim3((unsigned)grid),
                   dim3(Layout<BN, kChunk, kResidentB, kStages>::kThreads), smem, st,
                   /*pdl=*/true, prm, tmap, tmap_a);
}

// TMA-fed layers keep up to eight activation stages in flight when shared
// memory allows: a stage's load latency is then covered by the MMAs of the
// stages ahead of it.
template <int BN, int kChunk, bool kResidentB, bool kGap = false>
bool launch_staged(const FusedParams& prm, const CUtensorMap& tmap, const CUtensorMap& tmap_a,
                   cudaStream_t st) {
  if constexpr (kChunk <= 1) {
    if (smem_bytes<BN, kChunk, kResidentB, 8>(prm.num_kb, prm.pad_classes) <= kSmemCap)
      return launch_persistent<BN, kChunk, kResidentB, 8, kGap>(prm, tmap, tmap_a, st);
    if (smem_bytes<BN, kChunk, kResidentB, 6>(prm.num_kb, prm.pad_classes) <= kSmemCap)
      return launch_persistent<BN, kChunk, kResidentB, 6, kGap>(prm, tmap, tmap_a, st);
  }
  return launch_persistent<BN, kChunk, kResidentB, kStagesFused, kGap>(prm, tmap, tmap_a, st);
}

template <int BN, int kChunk, bool kGap = false>
bool launch_bn(const FusedParams& prm, const CUtensorMap& tmap, const CUtensorMap& tmap_a,
               cudaStream_t st) {
  if (smem_bytes<BN, kChunk, true, kStagesFused>(prm.num_kb, prm.pad_classes) <= kSmemCap)
    return launch_staged<BN, kChunk, true, kGap>(prm, tmap, tmap_a, st);
  return launch_staged<BN, kChunk, false, kGap>(prm, tmap, tmap_a, st);
}

using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const int*, const int*,
                                    cuuint32_t, cuuint32_t, const cuuint32_t*,
                                    CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeIm2colFn im2col_encoder() {
  static EncodeIm2colFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeIm2colFn>(ptr);
  });
  return fn;
}

// The thread gather stays in use when QA_FUSED_GATHER=threads.
bool tma_gather_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("QA_FUSED_GATHER");
    return !(v && std::strcmp(v, "threads") == 0);
  }();
  return on;
}

// Im2col tensor map of the layer's input for the TMA gather: 4-D {C, W, H, N}
// uint8 over the (possibly channel-sliced) NHWC view, 16 channels x 128
// output pixels per load.  The bounding box holds exactly the output
// lattice (lower corner -pad, upper corner at the last output position), so
// every tile's first pixel is a start inside it; the traversal strides are
// the convolution strides and the taps are the load's offsets.  Returns
// false (no error recorded) for layers the map cannot describe.
// Channel bytes per im2col load: whole 128- or 64-byte runs of a pixel's
// channels when C allows (one load moves 4-8x the bytes of a 16-byte one).
int im2col_slice(const qa_fused_conv_desc& d) {
  return d.C % 128 == 0 ? 128 : d.C % 64 == 0 ? 64 : 16;
}

bool make_im2col_tmap(CUtensorMap* map, const qa_fused_conv_desc& d, int slice) {
  if (!tma_gather_enabled()) return false;
  EncodeIm2colFn fn = im2col_encoder();
  if (!fn) return false;
  // out-of-image taps read zero: exact only for a zero point of 0 (or no
  // out-of-image taps at all)
  const bool no_oob = d.PH == 0 && d.PW == 0 && (d.OH - 1) * d.SH + (d.KH - 1) * d.DH < d.H &&
                      (d.OW - 1) * d.SW + (d.KW - 1) * d.DW < d.W;
  if ((d.x_zp & 0xFF) != 0 && !no_oob && !d.pad_corr) return false;
  if (d.C % 16 || d.x_pix_stride % 16 || (reinterpret_cast<uintptr_t>(d.x) & 15)) return false;
  if (d.SH > 8 || d.SW > 8 || (d.KH - 1) * d.DH > 64 || (d.KW - 1) * d.DW > 64) return false;
  const int64_t up_w = (d.OW - 1) * d.SW - d.PW - d.W + 1;
  const int64_t up_h = (d.OH - 1) * d.SH - d.PH - d.H + 1;
  if (d.PW > 128 || d.PH > 128 || up_w < -128 || up_w > 127 || up_h < -128 || up_h > 127)
    return false;
  if (d.W > (int64_t(1) << 31) || d.H > (int64_t(1) << 31) || d.N > (int64_t(1) << 31))
    return false;
  cuuint64_t dims[4] = {(cuuint64_t)d.C, (cuuint64_t)d.W, (cuuint64_t)d.H, (cuuint64_t)d.N};
  cuuint64_t strides[3] = {(cuuint64_t)d.x_pix_stride, (cuuint64_t)(d.x_pix_stride * d.W),
                           (cuuint64_t)(d.x_pix_stride * d.W * d.H)};
  if (strides[2] >= (cuuint64_t(1) << 40)) return false;
  const int lower[2] = {(int)-d.PW, (int)-d.PH};  // {W, H}
  const int upper[2] = {(int)up_w, (int)up_h};
  cuuint32_t estr[4] = {1u, (cuuint32_t)d.SW, (cuuint32_t)d.SH, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(d.x), dims, strides, lower,
            upper, (cuuint32_t)slice, kBM, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            slice == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
            : slice == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool fits_int32_mult(int64_t m) { return m > -(int64_t(1) << 31) && m < (int64_t(1) << 31); }

// Is the 64-bit rescale ((v - z) * m + 2^(ts-1)) >> ts exact for every
// 8-bit v?  |v - z| <= 2^9 + |z|.
bool small_rescale_fast(int64_t z, int64_t m, int64_t s) {
  const int64_t ts = 31 + s;
  if (ts < 1 || ts > 62 || !fits_int32_mult(m)) return false;
  const int64_t vmax = 512 + (z < 0 ? -z : z);
  if (vmax >= (int64_t(1) << 31)) return false;
  const double bound = (double)vmax * (double)(m < 0 ? -m : m) + std::ldexp(1.0, (int)ts - 1);
  return bound < std::ldexp(1.0, 61);
}

// Is |mbqm(v - z, m, s)| < 2^29 for every 8-bit v (so that two such terms
// and a zero point add up exactly in int32)?
bool table_term_small(int64_t z, int64_t m, int64_t s) {
  const double vmax = 383.0 + std::fabs((double)z);
  const double t = vmax * std::fabs((double)m) * std::ldexp(1.0, -(int)(31 + s)) + 2.0;
  return s > -64 && s < 64 && t < std::ldexp(1.0, 29);
}

bool byte_range(int64_t lo, int64_t hi) { return lo >= -128 && hi <= 255 && lo <= hi; }

}  // namespace

bool fused_conv_v2(const qa_fused_conv_desc& d, cudaStream_t st) {
  if (d.N < 0 || d.H <= 0 || d.W <= 0 || d.C <= 0 || d.Cout <= 0 || d.KH <= 0 || d.KW <= 0 ||
      d.SH <= 0 || d.SW <= 0 || d.DH <= 0 || d.DW <= 0 || d.OH <= 0 || d.OW <= 0 || d.PH < 0 ||
      d.PW < 0 || d.groups < 1) {
    set_error(kBadArgument, "qa_conv_fused_dev: invalid geometry");
    return false;
  }
  // every value the epilogue passes between its steps is stored as a byte
  if (!byte_range(d.qmin, d.qmax) || (d.res && !byte_range(d.add_qmin, d.add_qmax)) ||
      (d.out2 && !byte_range(d.r_qmin, d.r_qmax))) {
    set_error(kUnsupported, "qa_conv_fused_dev: output ranges must be 8-bit");
    return false;
  }
  if (d.groups > 1) {
    if (d.gap_sum) {
      set_error(kUnsupported, "qa_conv_fused_dev: no fused GlobalAveragePool on grouped layers");
      return false;
    }
    return fused_conv_grouped(d, st);
  }
  const int chunk = (d.C % 16 == 0 && d.x_pix_stride % 16 == 0) ? 16
                    : (d.C % 4 == 0 && d.x_pix_stride % 4 == 0) ? 4 : 0;
  if (!chunk || (reinterpret_cast<uintptr_t>(d.x) & (chunk - 1)) || !d.w || !d.mult ||
      !d.shift) {
    set_error(kBadArgument, "qa_conv_fused_dev: misaligned or missing operand");
    return false;
  }
  int bn = (int)d.block_n;
  if (bn == 0) bn = d.Cout <= 16 ? 16 : d.Cout <= 32 ? 32 : d.Cout <= 64 ? 64
                   : d.Cout <= 128 ? 128 : 256;
  if (chunk == 4 && bn > 64) bn = 64;
  const int64_t n_tiles = (d.Cout + bn - 1) / bn;
  const int64_t K = d.KH * d.KW * d.C;
  if (d.w_kp % 16 || d.w_kp < K || d.w_rows < n_tiles * bn) {
    set_error(kBadArgument, "qa_conv_fused_dev: packed weight shape does not cover the layer");
    return false;
  }
  if (d.N == 0) return true;
  const int64_t M = d.N * d.OH * d.OW;
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  // 32-bit row / tap arithmetic: rows, taps and one image's bytes fit int32
  const int64_t tap_span = ((d.KH - 1) * d.DH * d.W + (d.KW - 1) * d.DW) * d.x_pix_stride + d.C;
  if (M + kBM > 0x7FFFFFFF || K > (1 << 16) || tap_span > 0x7FFFFFFF ||
      (d.KH - 1) * d.DH > 32767 || (d.KW - 1) * d.DW > 32767 || d.H * d.W > 0x7FFFFFFF) {
    set_error(kUnsupported, "qa_conv_fused_dev: layer too large for the fused kernel");
    return false;
  }
  CUtensorMap tmap;
  if (!make_weight_tmap(&tmap, d.w, d.w_rows, d.w_kp, bn)) return false;
  CUtensorMap tmap_a;
  std::memset(&tmap_a, 0, sizeof(tmap_a));
  // pointwise layers (1x1, stride 1, no padding) read their input pixels
  // as a plain row matrix: one 2-D TMA load per 16 KB K-block
  const bool tile_a = chunk == 16 && tma_gather_enabled() && d.KH == 1 && d.KW == 1 &&
                      d.SH == 1 && d.SW == 1 && d.PH == 0 && d.PW == 0 && d.OH == d.H &&
                      d.OW == d.W &&
                      make_rows_tmap(&tmap_a, d.x, d.N * d.H * d.W, d.C, d.x_pix_stride, kBM);
  if (!tile_a) clear_error();
  if (d.pad_corr && !(d.pad_row_class && d.pad_col_class && d.pad_classes >= 1 &&
                      d.pad_classes <= 16 && d.pad_col_classes >= 1 &&
                      d.pad_classes % d.pad_col_classes == 0)) {
    set_error(kBadArgument, "qa_conv_fused_dev: inconsistent border correction tables");
    return false;
  }
  const int slice = im2col_slice(d);
  const bool tma_a = !tile_a && chunk == 16 && make_im2col_tmap(&tmap_a, d, slice);

  FusedParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.a = static_cast<const uint8_t*>(d.x);
  prm.pix_stride = d.x_pix_stride;
  prm.pad_word = (uint32_t)(d.x_zp & 0xFF) * 0x01010101u;
  prm.a_signed = d.x_signed ? 1 : 0;
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
  prm.num_kb = (int32_t)((K + kBK - 1) / kBK);
  prm.slice = tma_a ? slice : 16;
  prm.n_tap = prm.num_kb * (kBK / (tma_a ? slice : chunk));
  prm.n_valid = (int32_t)d.Cout;
  prm.m_tiles = (int32_t)m_tiles;
  prm.n_tiles = (int32_t)n_tiles;
  auto al16 = [](const void* ptr, int64_t stride) {
    return ptr == nullptr || ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && stride % 16 == 0);
  };
  // the border corrections apply to the TMA gather only (the thread gather
  // writes the zero point into out-of-image taps itself)
  if (tma_a && d.pad_corr && (d.x_zp & 0xFF) != 0) {
    prm.pad_corr = d.pad_corr;
    prm.pad_row_class = d.pad_row_class;
    prm.pad_col_class = d.pad_col_class;
    prm.pad_ncol = (int32_t)d.pad_col_classes;
    prm.pad_classes = (int32_t)d.pad_classes;
  }
  prm.vec_ok = al16(d.out, d.out_pix_stride) && al16(d.out2, d.out2_pix_stride) &&
               al16(d.res, d.res_pix_stride);
  prm.status = device_status_word();
  prm.fast.requant = d.fast ? 1 : 0;
  prm.fast.add64 = d.res ? (small_rescale_fast(d.za, d.ma, d.sa) &&
                            small_rescale_fast(d.zb, d.mb, d.sb))
                         : 0;
  prm.fast.add_tab = d.res ? (table_term_small(d.za, d.ma, d.sa) &&
                              table_term_small(d.zb, d.mb, d.sb) && (d.sign == 1 || d.sign == -1) &&
                              d.add_zo > -(1 << 20) && d.add_zo < (1 << 20))
                           : 0;
  prm.fast.r64 = d.out2 ? small_rescale_fast(d.r_zp_in, d.r_m, d.r_s) : 0;
  fill_fused_epilogue(prm.epi, d);
  if (d.gap_sum) {
    // GlobalAveragePool fused into a pointwise layer's epilogue: the rows of
    // one warp span at most two images, every pooled sum fits int32
    const int64_t hw = d.OH * d.OW;
    if (!tile_a || (bn != 128 && bn != 256) || !d.gap_cnt || !d.gap_out || hw < 32 ||
        hw * 255 >= (int64_t(1) << 31) || d.gap_zp_in < -128 || d.gap_zp_in > 255 ||
        d.gap_qmin < -128 || d.gap_qmax > 255) {
      set_error(kUnsupported, "qa_conv_fused_dev: fused GlobalAveragePool needs a pointwise "
                              "layer, a 128 or 256 column tile and at least 32 pixels per "
                              "image");
      return false;
    }
    prm.gap_sum = d.gap_sum;
    prm.gap_cnt = d.gap_cnt;
    prm.gap_out = static_cast<uint8_t*>(d.gap_out);
    prm.gap_out_stride = d.gap_out_stride;
    prm.gap_hw = (int32_t)hw;
    prm.gap_zp_in = (int32_t)d.gap_zp_in;
    prm.gap_mult = d.gap_mult;
    prm.gap_shift = d.gap_shift;
    prm.gap_zp_out = d.gap_zp_out;
    prm.gap_qmin = d.gap_qmin;
    prm.gap_qmax = d.gap_qmax;
    {
      // |sum| <= hw * 255 (int8 / uint8 input against its zero point)
      const int64_t ts = 31 + d.gap_shift;
      const double bound = (double)hw * 255.0 * std::fabs((double)d.gap_mult) +
                           std::ldexp(1.0, (int)std::min<int64_t>(std::max<int64_t>(ts, 1), 62));
      prm.gap_fast = ts >= 1 && ts <= 62 && bound < std::ldexp(1.0, 62) ? 1 : 0;
    }
    return bn == 128 ? launch_bn<128, 1, true>(prm, tmap, tmap_a, st)
                     : launch_bn<256, 1, true>(prm, tmap, tmap_a, st);
  }
  if (tile_a) {
    switch (bn) {
      case 16: return launch_bn<16, 1>(prm, tmap, tmap_a, st);
      case 32: return launch_bn<32, 1>(prm, tmap, tmap_a, st);
      case 64: return launch_bn<64, 1>(prm, tmap, tmap_a, st);
      case 128: return launch_bn<128, 1>(prm, tmap, tmap_a, st);
      case 256: return launch_bn<256, 1>(prm, tmap, tmap_a, st);
    }
  }
  if (tma_a) {
    switch (bn) {
      case 16: return launch_bn<16, 0>(prm, tmap, tmap_a, st);
      case 32: return launch_bn<32, 0>(prm, tmap, tmap_a, st);
      case 64: return launch_bn<64, 0>(prm, tmap, tmap_a, st);
      case 128: return launch_bn<128, 0>(prm, tmap, tmap_a, st);
      case 256: return launch_bn<256, 0>(prm, tmap, tmap_a, st);
    }
  } else if (chunk == 16) {
    switch (bn) {
      case 16: return launch_bn<16, 16>(prm, tmap, tmap_a, st);
      case 32: return launch_bn<32, 16>(prm, tmap, tmap_a, st);
      case 64: return launch_bn<64, 16>(prm, tmap, tmap_a, st);
      case 128: return launch_bn<128, 16>(prm, tmap, tmap_a, st);
      case 256: return launch_bn<256, 16>(prm, tmap, tmap_a, st);
    }
  } else {
    switch (bn) {
      case 16: return launch_bn<16, 4>(prm, tmap, tmap_a, st);
      case 32: return launch_bn<32, 4>(prm, tmap, tmap_a, st);
      case 64: return launch_bn<64, 4>(prm, tmap, tmap_a, st);
    }
  }
  set_error(kBadArgument, "qa_conv_fused_dev: unsupported column tile");
  return false;
}

}  // namespace qa

QA_API int qa_conv_fused_dev(const qa_fused_conv_desc* desc, void* stream) {
  qa::clear_error();
  if (!desc) {
    qa::set_error(qa::kBadArgument, "qa_conv_fused_dev: null descriptor");
    return qa::last_status();
  }
  return qa::fused_conv_v2(*desc, (cudaStream_t)stream) ? 0 : qa::last_status();
}
