/*
 * CPU ORACLE -- test infrastructure only, never shipped or timed as product.
 *
 * A plain-C restatement of the integer semantics of QuantAnything's native
 * kernels (quantization/kernels/qa_kernels.cpp in the reference project).
 * It exports the same 17 C symbols with the same signatures so the parity
 * tests can drive it through exactly the ctypes wrapper that drives the CUDA
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load it.
 *
 * The code is written for clarity, not speed: direct (not im2col) loops,
 * one thread, and explicitly wrapping unsigned arithmetic wherever the
 * reference relies on two's-complement wrap-around of signed types.
 *
 * Parity is pinned by tests/test_oracle_golden.py against vectors produced by
 * the reference's own C++ library (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#define QAO_API __attribute__((visibility("default")))

typedef __int128 i128;
typedef unsigned __int128 u128;

/* ------------------------------------------------------------ threading ---
 * qa_kernels.cpp:233-249: thread-count introspection.  The oracle is serial. */
QAO_API int qa_num_threads(void) { return 1; }
QAO_API void qa_set_num_threads(int n) { (void)n; }
QAO_API int qa_has_openmp(void) { return 0; }

/* ----------------------------------------------------------------- GEMM ---
 * qa_kernels.cpp:59-105 (gemm_tile / gemm_parallel): C[M,N] = A[M,K]·B[K,N],
 * row-major, every operand promoted to the accumulator type before the
 * multiply.  The int32 accumulator wraps modulo 2^32 (the reference's signed
 * int32 '+=' compiles to wrapping adds); we use uint32 to make that defined.
 * The reference skips a==0 terms (:73); adding zero changes nothing, so the
 * result is the plain sum in any order. */
QAO_API void qa_gemm_f32(int64_t M, int64_t N, int64_t K, const float* A,
                         const float* B, float* C) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      float s = 0.0f;
      for (int64_t k = 0; k < K; ++k) s += A[i * K + k] * B[k * N + j];
      C[i * N + j] = s;
    }
}

QAO_API void qa_gemm_i16_i32(int64_t M, int64_t N, int64_t K, const int16_t* A,
                             const int16_t* B, int32_t* C) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      uint32_t s = 0;
      for (int64_t k = 0; k < K; ++k)
        s += (uint32_t)((int32_t)A[i * K + k] * (int32_t)B[k * N + j]);
      C[i * N + j] = (int32_t)s;
    }
}

QAO_API void qa_gemm_i32_i64(int64_t M, int64_t N, int64_t K, const int32_t* A,
                             const int32_t* B, int64_t* C) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      uint64_t s = 0;
      for (int64_t k = 0; k < K; ++k)
        s += (uint64_t)((int64_t)A[i * K + k] * (int64_t)B[k * N + j]);
      C[i * N + j] = (int64_t)s;
    }
}

/* ----------------------------------------------------------------- conv ---
 * qa_kernels.cpp:108-185 (ConvShape / im2col / conv_nchw): NCHW input, OIHW
 * weights, `G` groups, stride (SH,SW), dilation (DH,DW), top/left padding
 * (PH,PW); the bottom/right padding is implied by the caller's OH/OW.  Taps
 * that fall outside the image contribute zero (the im2col buffer is zero
 * filled there, :124-133).  On the narrow path the int32 input is cast to the
 * int16 operand type before the multiply (im2col's static_cast<TA>, :131-133,
 * and the pointwise copy, :163-164), so that cast is reproduced here. */
#define CONV_ARGS                                                           \
  int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cout, int64_t KH,     \
      int64_t KW, int64_t SH, int64_t SW, int64_t PH, int64_t PW, int64_t DH, \
      int64_t DW, int64_t G, int64_t OH, int64_t OW

QAO_API void qa_conv_f32(const float* x, const float* w, float* y, CONV_ARGS) {
  const int64_t Cg = C / G, Cog = Cout / G;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t co = 0; co < Cout; ++co) {
      const int64_t g = co / Cog;
      for (int64_t oy = 0; oy < OH; ++oy)
        for (int64_t ox = 0; ox < OW; ++ox) {
          float s = 0.0f;
          for (int64_t ci = 0; ci < Cg; ++ci)
            for (int64_t ky = 0; ky < KH; ++ky) {
              const int64_t iy = oy * SH - PH + ky * DH;
              if (iy < 0 || iy >= H) continue;
              for (int64_t kx = 0; kx < KW; ++kx) {
                const int64_t ix = ox * SW - PW + kx * DW;
                if (ix < 0 || ix >= W) continue;
                s += x[((n * C + g * Cg + ci) * H + iy) * W + ix] *
                     w[((co * Cg + ci) * KH + ky) * KW + kx];
              }
            }
          y[((n * Cout + co) * OH + oy) * OW + ox] = s;
        }
    }
}

QAO_API void qa_conv_i32_i16_i32(const int32_t* x, const int16_t* w,
                                 int32_t* y, CONV_ARGS) {
  const int64_t Cg = C / G, Cog = Cout / G;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t co = 0; co < Cout; ++co) {
      const int64_t g = co / Cog;
      for (int64_t oy = 0; oy < OH; ++oy)
        for (int64_t ox = 0; ox < OW; ++ox) {
          uint32_t s = 0;
          for (int64_t ci = 0; ci < Cg; ++ci)
            for (int64_t ky = 0; ky < KH; ++ky) {
              const int64_t iy = oy * SH - PH + ky * DH;
              if (iy < 0 || iy >= H) continue;
              for (int64_t kx = 0; kx < KW; ++kx) {
                const int64_t ix = ox * SW - PW + kx * DW;
                if (ix < 0 || ix >= W) continue;
                const int16_t xv =
                    (int16_t)x[((n * C + g * Cg + ci) * H + iy) * W + ix];
                s += (uint32_t)((int32_t)xv *
                                (int32_t)w[((co * Cg + ci) * KH + ky) * KW + kx]);
              }
            }
          y[((n * Cout + co) * OH + oy) * OW + ox] = (int32_t)s;
        }
    }
}

QAO_API void qa_conv_i32_i32_i64(const int32_t* x, const int32_t* w,
                                 int64_t* y, CONV_ARGS) {
  const int64_t Cg = C / G, Cog = Cout / G;
  for (int64_t n = 0; n < N; ++n)
    for (int64_t co = 0; co < Cout; ++co) {
      const int64_t g = co / Cog;
      for (int64_t oy = 0; oy < OH; ++oy)
        for (int64_t ox = 0; ox < OW; ++ox) {
          uint64_t s = 0;
          for (int64_t ci = 0; ci < Cg; ++ci)
            for (int64_t ky = 0; ky < KH; ++ky) {
              const int64_t iy = oy * SH - PH + ky * DH;
              if (iy < 0 || iy >= H) continue;
              for (int64_t kx = 0; kx < KW; ++kx) {
                const int64_t ix = ox * SW - PW + kx * DW;
                if (ix < 0 || ix >= W) continue;
                s += (uint64_t)(
                    (int64_t)x[((n * C + g * Cg + ci) * H + iy) * W + ix] *
                    (int64_t)w[((co * Cg + ci) * KH + ky) * KW + kx]);
              }
            }
          y[((n * Cout + co) * OH + oy) * OW + ox] = (int64_t)s;
        }
    }
}

/* -------------------------------------------------- fixed-point multiply ---
 * qa_kernels.cpp:194-205 (mbqm): round(x·mult·2^-(31+shift)) on a 128-bit
 * product.  With ts = 31 + shift: ts > 0 rounds half up and shifts right
 * arithmetically (ts capped at 120); ts <= 0 multiplies by 2^-ts (capped at
 * 2^60), wrapping modulo 2^128 like the reference's i128 multiply. */
static i128 mbqm(int64_t x, int64_t mult, int64_t shift) {
  const i128 p = (i128)x * (i128)mult;
  int64_t ts = 31 + shift;
  if (ts > 0) {
    if (ts > 120) ts = 120;
    return (p + ((i128)1 << (ts - 1))) >> ts;
  }
  if (ts < -60) ts = -60;
  return (i128)((u128)p << (unsigned)(-ts));
}

/* qa_kernels.cpp:188-192 (clamp128). */
static int64_t clamp128(i128 v, int64_t lo, int64_t hi) {
  if (v < (i128)lo) return lo;
  if (v > (i128)hi) return hi;
  return (int64_t)v;
}

/* ------------------------------------------------------------ requantize ---
 * qa_kernels.cpp:207-228 and :287-302: accumulators viewed as
 * [outer, C, inner]; channel c maps acc to
 * clamp(mbqm(acc + pre[c], M0[c], shift[c]) + post[c] + zp, qmin, qmax). */
#define REQUANT_BODY(T)                                                      \
  for (int64_t o = 0; o < outer; ++o)                                        \
    for (int64_t c = 0; c < C; ++c) {                                        \
      const int64_t pb = pre_bias ? pre_bias[c] : 0;                         \
      const int64_t qb = (post_bias ? post_bias[c] : 0) + zp;                \
      for (int64_t i = 0; i < inner; ++i) {                                  \
        const int64_t idx = (o * C + c) * inner + i;                         \
        const i128 v = mbqm((int64_t)acc[idx] + pb, mult[c], shift[c]) + qb; \
        out[idx] = (int32_t)clamp128(v, qmin, qmax);                         \
      }                                                                      \
    }

QAO_API void qa_requantize_i32(const int32_t* acc, int32_t* out, int64_t outer,
                               int64_t C, int64_t inner, const int64_t* mult,
                               const int64_t* shift, const int64_t* pre_bias,
                               const int64_t* post_bias, int64_t zp,
                               int64_t qmin, int64_t qmax) {
  REQUANT_BODY(int32_t)
}

QAO_API void qa_requantize_i64(const int64_t* acc, int32_t* out, int64_t outer,
                               int64_t C, int64_t inner, const int64_t* mult,
                               const int64_t* shift, const int64_t* pre_bias,
                               const int64_t* post_bias, int64_t zp,
                               int64_t qmin, int64_t qmax) {
  REQUANT_BODY(int64_t)
}

/* --------------------------------------------------------- element-wise --- */

/* qa_kernels.cpp:307-316: out = clamp(mbqm(x - zp_in, m, s) + zp_out). */
QAO_API void qa_rescale(const int32_t* x, int32_t* out, int64_t n,
                        int64_t zp_in, int64_t m, int64_t s, int64_t zp_out,
                        int64_t qmin, int64_t qmax) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = (int32_t)clamp128(mbqm((int64_t)x[i] - zp_in, m, s) + zp_out,
                               qmin, qmax);
}

/* qa_kernels.cpp:319-331:
 * out = clamp(mbqm(a-za,ma,sa) + sign·mbqm(b-zb,mb,sb) + zp_out). */
QAO_API void qa_add(const int32_t* a, const int32_t* b, int32_t* out,
                    int64_t n, int64_t za, int64_t ma, int64_t sa, int64_t zb,
                    int64_t mb, int64_t sb, int64_t sign, int64_t zp_out,
                    int64_t qmin, int64_t qmax) {
  for (int64_t i = 0; i < n; ++i) {
    const i128 ta = mbqm((int64_t)a[i] - za, ma, sa);
    const i128 tb = mbqm((int64_t)b[i] - zb, mb, sb);
    const i128 v = (i128)((u128)ta + (u128)((i128)sign * tb)) + zp_out;
    out[i] = (int32_t)clamp128(v, qmin, qmax);
  }
}

/* qa_kernels.cpp:334-345: out = clamp(mbqm((a-za)(b-zb), m, s) + zp_out). */
QAO_API void qa_mul(const int32_t* a, const int32_t* b, int32_t* out,
                    int64_t n, int64_t za, int64_t zb, int64_t m, int64_t s,
                    int64_t zp_out, int64_t qmin, int64_t qmax) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t prod =
        (int64_t)((uint64_t)((int64_t)a[i] - za) * (uint64_t)((int64_t)b[i] - zb));
    out[i] = (int32_t)clamp128(mbqm(prod, m, s) + zp_out, qmin, qmax);
  }
}

/* qa_kernels.cpp:348-358: out = lut[clamp(x - offset, 0, lut_len - 1)]. */
QAO_API void qa_lut(const int32_t* x, int32_t* out, int64_t n, int64_t offset,
                    const int32_t* lut, int64_t lut_len) {
  for (int64_t i = 0; i < n; ++i) {
    int64_t idx = (int64_t)x[i] - offset;
    if (idx < 0) idx = 0;
    if (idx > lut_len - 1) idx = lut_len - 1;
    out[i] = lut[idx];
  }
}

/* ---------------------------------------------------- float <-> integer ---
 * qa_kernels.cpp:363-376: q = clamp(nearbyint((double)x / scale) + zp) with
 * the clamp done in double and the result truncated to int32.  x86's
 * truncating conversion turns NaN (and anything out of int32 range) into
 * INT32_MIN; that is made explicit here so the oracle does not depend on UB. */
static int32_t to_i32_like_x86(double v) {
  if (!(v >= -2147483648.0 && v < 2147483648.0)) return INT32_MIN;
  return (int32_t)v;
}

QAO_API void qa_quantize_f32(const float* x, int32_t* q, int64_t n,
                             double scale, int64_t zp, int64_t qmin,
                             int64_t qmax) {
  for (int64_t i = 0; i < n; ++i) {
    double v = nearbyint((double)x[i] / scale) + (double)zp;
    /* std::max<double>(v, qmin) then std::min<double>(., qmax): NaN passes
     * through both (the comparisons are false). */
    if (v < (double)qmin) v = (double)qmin;
    if ((double)qmax < v) v = (double)qmax;
    q[i] = to_i32_like_x86(v);
  }
}

/* qa_kernels.cpp:379-386: x = (float)((double)(q - zp) * scale). */
QAO_API void qa_dequantize_f32(const int32_t* q, float* x, int64_t n,
                               double scale, int64_t zp) {
  for (int64_t i = 0; i < n; ++i)
    x[i] = (float)((double)((int64_t)q[i] - zp) * scale);
}
