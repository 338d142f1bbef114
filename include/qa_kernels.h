/*
 * qa_kernels.h -- C ABI of the B200 (sm_100a) QuantAnything kernel library.
 *
 * libqa_kernels.so is a drop-in for the reference's CPU library: the first
 * block below is the exact symbol set and signature set that the reference's
 * ctypes loader declares (quantization/native.py:104-128 in the reference
 * project), so `QA_LIB=/path/to/libqa_kernels.so` swaps it in under the
 * reference's unchanged Python.  Those entry points take HOST pointers,
 * copy to the GPU, compute, copy back and return synchronously -- the same
 * contract as the CPU library (outputs valid on return, caller owns every
 * buffer, no pointer retained).
 *
 * The second block adds what the reference has no counterpart for: an error
 * channel, device selection, and DEVICE-pointer entry points (suffix _dev)
 * that enqueue on a caller-provided CUDA stream for the device-resident
 * executor.  Every signature uses only plain C types.
 *
 * Conventions shared with the reference (quantization/kernels/
 * qa_kernels.cpp:1-13): row-major contiguous buffers; activations cross the
 * boundary as int32 arrays holding values in [qmin, qmax]; the "narrow" path
 * has int16 operands and an int32 accumulator, the "wide" path int32 operands
 * and an int64 accumulator; requantization rounds half up on a 128-bit
 * product.
 */
#ifndef QA_KERNELS_H_
#define QA_KERNELS_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================================== *
 *  1. Reference ABI (host pointers, synchronous)                        *
 * ===================================================================== */

/* qa_kernels.cpp:233 -- number of GPUs visible to the library (the CPU
 * library returns its OpenMP thread count). */
int qa_num_threads(void);
/* qa_kernels.cpp:235 -- accepted and ignored (GPU work is not threaded by
 * the host). */
void qa_set_num_threads(int n);
/* qa_kernels.cpp:243 -- always 0: the GPU library has no OpenMP. */
int qa_has_openmp(void);

/* qa_kernels.cpp:252 -- C[M,N] = A[M,K]·B[K,N], float32. */
void qa_gemm_f32(int64_t M, int64_t N, int64_t K, const float* A,
                 const float* B, float* C);
/* qa_kernels.cpp:256 -- int16 operands, exact int32 accumulator (wraps
 * modulo 2^32 exactly like the CPU library if the caller's bound fails). */
void qa_gemm_i16_i32(int64_t M, int64_t N, int64_t K, const int16_t* A,
                     const int16_t* B, int32_t* C);
/* qa_kernels.cpp:260 -- int32 operands, exact int64 accumulator. */
void qa_gemm_i32_i64(int64_t M, int64_t N, int64_t K, const int32_t* A,
                     const int32_t* B, int64_t* C);

/* qa_kernels.cpp:273-284 -- NCHW convolution with OIHW weights, G groups,
 * strides (SH,SW), top/left padding (PH,PW), dilations (DH,DW); the
 * bottom/right padding is implied by OH/OW.  The narrow variant casts the
 * int32 input to int16 before multiplying, like the CPU library. */
void qa_conv_f32(const float* x, const float* w, float* y, int64_t N,
                 int64_t C, int64_t H, int64_t W, int64_t Cout, int64_t KH,
                 int64_t KW, int64_t SH, int64_t SW, int64_t PH, int64_t PW,
                 int64_t DH, int64_t DW, int64_t G, int64_t OH, int64_t OW);
void qa_conv_i32_i16_i32(const int32_t* x, const int16_t* w, int32_t* y,
                         int64_t N, int64_t C, int64_t H, int64_t W,
                         int64_t Cout, int64_t KH, int64_t KW, int64_t SH,
                         int64_t SW, int64_t PH, int64_t PW, int64_t DH,
                         int64_t DW, int64_t G, int64_t OH, int64_t OW);
void qa_conv_i32_i32_i64(const int32_t* x, const int32_t* w, int64_t* y,
                         int64_t N, int64_t C, int64_t H, int64_t W,
                         int64_t Cout, int64_t KH, int64_t KW, int64_t SH,
                         int64_t SW, int64_t PH, int64_t PW, int64_t DH,
                         int64_t DW, int64_t G, int64_t OH, int64_t OW);

/* qa_kernels.cpp:287-302 -- accumulators viewed as [outer, C, inner]:
 * out = clamp(mbqm(acc + pre[c], mult[c], shift[c]) + post[c] + zp).
 * pre_bias / post_bias may be NULL. */
void qa_requantize_i32(const int32_t* acc, int32_t* out, int64_t outer,
                       int64_t C, int64_t inner, const int64_t* mult,
                       const int64_t* shift, const int64_t* pre_bias,
                       const int64_t* post_bias, int64_t zp, int64_t qmin,
                       int64_t qmax);
void qa_requantize_i64(const int64_t* acc, int32_t* out, int64_t outer,
                       int64_t C, int64_t inner, const int64_t* mult,
                       const int64_t* shift, const int64_t* pre_bias,
                       const int64_t* post_bias, int64_t zp, int64_t qmin,
                       int64_t qmax);

/* qa_kernels.cpp:307 -- out = clamp(mbqm(x - zp_in, m, s) + zp_out). */
void qa_rescale(const int32_t* x, int32_t* out, int64_t n, int64_t zp_in,
                int64_t m, int64_t s, int64_t zp_out, int64_t qmin,
                int64_t qmax);
/* qa_kernels.cpp:319 -- out = clamp(mbqm(a-za,ma,sa) + sign·mbqm(b-zb,mb,sb)
 * + zp_out). */
void qa_add(const int32_t* a, const int32_t* b, int32_t* out, int64_t n,
            int64_t za, int64_t ma, int64_t sa, int64_t zb, int64_t mb,
            int64_t sb, int64_t sign, int64_t zp_out, int64_t qmin,
            int64_t qmax);
/* qa_kernels.cpp:334 -- out = clamp(mbqm((a-za)(b-zb), m, s) + zp_out). */
void qa_mul(const int32_t* a, const int32_t* b, int32_t* out, int64_t n,
            int64_t za, int64_t zb, int64_t m, int64_t s, int64_t zp_out,
            int64_t qmin, int64_t qmax);
/* qa_kernels.cpp:348 -- out = lut[clamp(x - offset, 0, lut_len - 1)]. */
void qa_lut(const int32_t* x, int32_t* out, int64_t n, int64_t offset,
            const int32_t* lut, int64_t lut_len);
/* qa_kernels.cpp:363 -- q = clamp(rint(x / scale) + zp), half to even, in
 * IEEE double. */
void qa_quantize_f32(const float* x, int32_t* q, int64_t n, double scale,
                     int64_t zp, int64_t qmin, int64_t qmax);
/* qa_kernels.cpp:379 -- x = (float)((q - zp) · scale) in IEEE double. */
void qa_dequantize_f32(const int32_t* q, float* x, int64_t n, double scale,
                       int64_t zp);

/* ===================================================================== *
 *  2. Extensions (no counterpart in the reference)                      *
 * ===================================================================== */

/* Error channel.  The reference's entry points return void and cannot fail
 * loudly; here every entry point records a status for the calling host
 * thread.  Mode 1 (the default, since the reference's loader cannot check a
 * status) prints the message and aborts the process on any failure; mode 0
 * only records it for qa_last_status()/qa_last_error().  QA_ON_ERROR=record
 * in the environment selects mode 0 at load time. */
int qa_last_status(void);          /* 0 = ok */
const char* qa_last_error(void);   /* "" when the last call succeeded */
void qa_clear_error(void);
void qa_set_error_mode(int abort_on_error);

/* Device selection for the calling host thread (default: $QA_DEVICE or 0). */
int qa_device_count(void);
int qa_set_device(int ordinal);
int qa_get_device(void);

/* ===================================================================== *
 *  3. Device-pointer entry points (no counterpart in the reference)     *
 *                                                                       *
 *  All pointers are device pointers; `stream` is a cudaStream_t (NULL = *
 *  the legacy default stream).  The calls only enqueue work and return  *
 *  0 on success or a status code (see qa_last_error()).                 *
 * ===================================================================== */

/* Requantization of device accumulators (same math as qa_requantize_*). */
int qa_requantize_i32_dev(const int32_t* acc, int32_t* out, int64_t outer, int64_t C,
                          int64_t inner, const int64_t* mult, const int64_t* shift,
                          const int64_t* pre_bias, const int64_t* post_bias, int64_t zp,
                          int64_t qmin, int64_t qmax, void* stream);
int qa_requantize_i64_dev(const int64_t* acc, int32_t* out, int64_t outer, int64_t C,
                          int64_t inner, const int64_t* mult, const int64_t* shift,
                          const int64_t* pre_bias, const int64_t* post_bias, int64_t zp,
                          int64_t qmin, int64_t qmax, void* stream);

/* One fused 8-bit convolution / GEMM layer of the device-resident executor:
 * tcgen05 implicit GEMM over NHWC int8/uint8 activations followed by the
 * reference's per-layer integer sequence (ConvQuantize/GemmQuantize
 * requantize, optional LUT activation, optional residual Add, optional
 * rescaled copy into a Concat slice -- quant_layers.py:320-560).
 *
 * Layout: activation pixel p of image n at x + ((n*H + y)*W + x)*x_pix_stride,
 * channel c at +c (so channel slices of a wider tensor are views).  Weights
 * are packed [w_rows][w_kp] int8, row = output channel, K ordered
 * (ky, kx, c) with C channels per tap, zero padded; w_kp % 16 == 0 and
 * w_rows a multiple of the column tile (16..256, chosen from Cout).  Every
 * field is 8 bytes so the struct has no padding. */
typedef struct qa_fused_conv_desc {
  const void* x;          /* activations (NHWC bytes) */
  int64_t x_pix_stride;   /* bytes between pixels; multiple of 16 (C%16==0) or 4 */
  int64_t x_signed;       /* 1: int8, 0: uint8 */
  int64_t x_zp;           /* raw zero point: value of out-of-image taps */
  int64_t N, H, W, C;     /* C: channels per tap, multiple of 16 (or 4) */
  int64_t KH, KW, SH, SW, PH, PW, DH, DW, OH, OW;
  int64_t Cout;
  int64_t groups;         /* >1: grouped / depthwise (C = channels per group) */
  const void* w;          /* packed weights (int8) */
  int64_t w_rows, w_kp;
  const int64_t* bias;    /* per channel, may be NULL; includes -x_zp*sum(w) */
  const int64_t* mult;
  const int64_t* shift;
  int64_t zp, qmin, qmax;
  int64_t fast;           /* 1: host proved the 64-bit requantize exact */
  const int32_t* lut;     /* optional activation table */
  int64_t lut_offset, lut_len;
  const void* res;        /* optional residual (NHWC bytes), channel 0 */
  int64_t res_pix_stride, res_signed;
  int64_t za, ma, sa, zb, mb, sb, sign, add_zo, add_qmin, add_qmax;
  void* out;              /* optional primary output (NHWC bytes), channel 0 */
  int64_t out_pix_stride;
  void* out2;             /* optional rescaled copy, channel 0 */
  int64_t out2_pix_stride;
  int64_t r_identity;
  int64_t r_zp_in, r_m, r_s, r_zp_out, r_qmin, r_qmax;
  int64_t block_n;        /* column tile: 0 = choose from Cout */
  /* Border corrections for a nonzero x_zp with out-of-image taps (NULL:
   * none; such a layer then gathers its input with plain loads): the TMA
   * gather reads those taps as 0, and pad_corr[cls * Cout + co] =
   * x_zp * (sum of channel co's weights over the taps outside the image)
   * restores them; cls = pad_row_class[oy] * pad_col_classes +
   * pad_col_class[ox], class 0 for interior pixels. */
  const int32_t* pad_corr;
  const int32_t* pad_row_class;  /* [OH] */
  const int32_t* pad_col_class;  /* [OW] */
  int64_t pad_col_classes, pad_classes;
  /* Optional GlobalAveragePool of this layer's (final 8-bit) output fused
   * into the epilogue (gap_sum NULL: none; the reference's
   * GlobalAveragePoolQuantize, quant_layers.py:563-590):
   * gap_out[n * gap_out_stride + c] = clamp(mbqm(sum over the image's OH*OW
   * pixels of (v - gap_zp_in), gap_mult, gap_shift) + gap_zp_out).
   * gap_sum (int32 [N][Cout]) and gap_cnt (int32 [N][ceil(Cout / block_n)])
   * must hold zeros on entry and hold zeros again on exit.  Pointwise layers
   * (1x1, stride 1, no padding, C % 16 == 0) with block_n 128 or 256 and
   * OH * OW >= 32 only; `out` may be NULL to skip the full-size store. */
  int32_t* gap_sum;
  int32_t* gap_cnt;
  void* gap_out;
  int64_t gap_out_stride, gap_zp_in, gap_mult, gap_shift, gap_zp_out, gap_qmin, gap_qmax;
} qa_fused_conv_desc;

int qa_conv_fused_dev(const qa_fused_conv_desc* desc, void* stream);

/* Graph input: float32 NCHW -> quantized bytes NHWC with `pix_stride`
 * channels per pixel (channels C.. hold zp), same rounding as
 * qa_quantize_f32. */
int qa_quantize_to_nhwc_dev(const float* x, void* y, int64_t N, int64_t C, int64_t H, int64_t W,
                            int64_t pix_stride, double scale, int64_t zp, int64_t qmin,
                            int64_t qmax, void* stream);

/* The same quantization written as the im2col rows of a P x P, stride-P
 * convolution (a patch embedding): row (n * H/P + py) * W/P + px holds the
 * patch's P * P pixels, (ky * P + kx) * 4 bytes in, 4 channel bytes each
 * (channels C.. hold zp).  C <= 4, P % 4 == 0, H and W multiples of P. */
int qa_quantize_to_patch_rows_dev(const float* x, void* y, int64_t N, int64_t C, int64_t H,
                                  int64_t W, int64_t P, double scale, int64_t zp, int64_t qmin,
                                  int64_t qmax, void* stream);

/* GlobalAveragePool (quant_layers.py:563-590): int64 sum of centred bytes
 * over HW pixels, requantized with the scalar (mult, shift). */
int qa_gap_dev(const void* x, int64_t x_pix_stride, int64_t x_signed, int64_t N, int64_t HW,
               int64_t C, int64_t zp_in, int64_t mult, int64_t shift, int64_t zp_out,
               int64_t qmin, int64_t qmax, void* y, int64_t y_pix_stride, void* stream);

/* Softmax float fallback over rows of C bytes (quant_layers.py:195-205):
 * dequantize, float64 softmax, quantize; writes the int32 result (q_out) and
 * / or its float32 dequantization on the (y_scale, y_zp) grid (y_out). */
int qa_softmax_dev(const void* x, int64_t x_pix_stride, int64_t x_signed, int64_t N, int64_t C,
                   double in_scale, int64_t in_zp, double out_scale, int64_t out_zp,
                   int64_t qmin, int64_t qmax, int32_t* q_out, float* y_out, double y_scale,
                   int64_t y_zp, void* stream);

/* Standalone byte-tensor layers over [rows, C] views (row = pixel). */
int qa_lut_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                     int64_t y_stride, int64_t rows, int64_t C, int64_t offset,
                     const int32_t* lut, int64_t lut_len, void* stream);
int qa_add_bytes_dev(const void* a, int64_t a_stride, int64_t a_signed, const void* b,
                     int64_t b_stride, int64_t b_signed, void* y, int64_t y_stride,
                     int64_t rows, int64_t C, int64_t za, int64_t ma, int64_t sa, int64_t zb,
                     int64_t mb, int64_t sb, int64_t sign, int64_t zo, int64_t qmin,
                     int64_t qmax, void* stream);
/* Integer Mul of two activations (qa_kernels.cpp:334-345):
 * out = clamp(mbqm((a - za)(b - zb), m, s) + zo). */
int qa_mul_bytes_dev(const void* a, int64_t a_stride, int64_t a_signed, const void* b,
                     int64_t b_stride, int64_t b_signed, void* y, int64_t y_stride,
                     int64_t rows, int64_t C, int64_t za, int64_t zb, int64_t m, int64_t s,
                     int64_t zo, int64_t qmin, int64_t qmax, void* stream);
/* Inference BatchNorm (quant_layers.py:405-441, qa_kernels.cpp:207-228 with
 * a post-bias): out = clamp(mbqm(x - zp_in, mult[c], shift[c]) + post[c] +
 * zp_out), per-channel int64 device arrays. */
int qa_bn_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                    int64_t y_stride, int64_t rows, int64_t C, int64_t zp_in,
                    const int64_t* mult, const int64_t* shift, const int64_t* post,
                    int64_t zp_out, int64_t qmin, int64_t qmax, void* stream);
int qa_rescale_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                         int64_t y_stride, int64_t rows, int64_t C, int64_t identity,
                         int64_t zp_in, int64_t m, int64_t s, int64_t zp_out, int64_t qmin,
                         int64_t qmax, void* stream);
int qa_maxpool_bytes_dev(const void* x, int64_t x_stride, int64_t x_signed, void* y,
                         int64_t y_stride, int64_t N, int64_t H, int64_t W, int64_t C,
                         int64_t KH, int64_t KW, int64_t SH, int64_t SW, int64_t PH, int64_t PW,
                         int64_t DH, int64_t DW, int64_t OH, int64_t OW, int64_t pad_value,
                         void* stream);

/* Pad / Slice / Transpose of an NHWC byte tensor (quant_layers.py:593-650:
 * scale-preserving, Pad fills with the input zero point): output element
 * (n, c, y, x) of the [ON, OC, OH, OW] result (NHWC bytes, y_pix_stride per
 * pixel) reads x + sum_a (start[a] + i[a] * step[a]) * stride[a] (host
 * arrays of four, NCHW axis order; stride[a] in bytes of the source axis
 * output axis a reads), or `fill` where a coordinate leaves [0, dim[a]). */
int qa_window_copy_bytes_dev(const void* x, void* y, int64_t y_pix_stride, int64_t ON,
                             int64_t OC, int64_t OH, int64_t OW, const int64_t* start,
                             const int64_t* step, const int64_t* dim, const int64_t* stride,
                             int64_t fill, void* stream);

/* Layout conversion between NHWC byte views and NCHW int32 tensors. */
int qa_bytes_to_i32_dev(const void* x, int64_t x_stride, int64_t x_signed, int32_t* y,
                        int64_t N, int64_t HW, int64_t C, void* stream);
int qa_i32_to_bytes_dev(const int32_t* x, void* y, int64_t y_stride, int64_t N, int64_t HW,
                        int64_t C, void* stream);

/* Synchronizes `stream` and reports (then clears) a bounded-wait timeout
 * recorded by any kernel on this device. */
int qa_device_status_dev(void* stream);

/* Self-test of the bounded-wait error channel (no counterpart in the
 * reference, which has no device code): one thread waits, for at most
 * `budget_cycles` SM cycles (<= 2^32), on an mbarrier that it releases
 * itself only when `arrive` is nonzero.  A wait that runs out records a
 * timeout that the next qa_device_status_dev reports as kDeviceTimeout;
 * the context stays usable. */
int qa_wait_probe_dev(int64_t budget_cycles, int arrive, void* stream);

/* Fused network-input layer: float32 NCHW images with c_in <= 4 channels
 * are quantized with (scale, desc->x_zp, qmin, qmax) exactly like
 * qa_quantize_f32, convolved with the packed int8 weights of `desc`
 * (desc->C = 4: taps packed 4 channels wide, unused channels zero) on CUDA
 * cores, and passed through the layer epilogue of `desc` (requantize,
 * optional LUT; no residual / concat copy).  desc->x is ignored. */
int qa_conv_input_fused_dev(const qa_fused_conv_desc* desc, const float* x, int64_t c_in,
                            double scale, int64_t qmin, int64_t qmax, void* stream);

/* Transformer (ViT) graphs, activations as byte rows [rows, features].
 *
 * Token embedding: out[n, 0, :] = cls_row, out[n, t, d] =
 * clamp(ta[x[n, t-1, d] + 128] + pos[t * D + d], qmin, qmax) for t >= 1: the
 * Concat of the class token with the patch tokens followed by the
 * positional-embedding Add (quant_layers.py:486-513, 543-560), as exact
 * integer tables (ta: 384 entries over byte values -128..255). */
int qa_vit_embed_dev(const void* x, int64_t x_stride, int32_t x_signed, const int32_t* ta,
                     const int32_t* pos, const void* cls_row, int64_t qmin, int64_t qmax,
                     void* out, int64_t out_stride, int64_t B, int64_t T, int64_t D,
                     void* stream);

/* LayerNormalization over the last axis as the reference's float fallback
 * (float_ops.py:336-347 between qa_dequantize_f32 and qa_quantize_f32);
 * beta may be NULL. */
int qa_layernorm_bytes_dev(const void* x, int64_t x_stride, int32_t x_signed, int64_t zp_in,
                           double scale_in, const float* gamma, const float* beta, double eps,
                           double scale_out, int64_t zp_out, int64_t qmin, int64_t qmax,
                           void* out, int64_t out_stride, int64_t rows, int64_t D,
                           void* stream);

/* Multi-head self-attention of one block, fused: scores MatMul, the Mul by
 * 1/sqrt(head_dim) (mul_table: 384 entries), Softmax over the keys and the
 * MatMul with V, each quantized like the reference's float fallbacks
 * (quant_layers.py:195-205), written in the head-merged [B*T, H*hd] layout.
 * qkv rows hold q | k | v (H*hd bytes each).  s_params: scales of
 * {scores, Mul output, softmax output, attention output}; z_params:
 * {scores zp, qmin, qmax, softmax zp, qmin, qmax, output zp, qmin, qmax,
 * Mul output zp} (host arrays, read at the call).  T <= 256, head_dim <= 128
 * and a multiple of 4. */
int qa_attention_bytes_dev(const void* qkv, int64_t qkv_stride, int32_t qkv_signed,
                           int64_t z_qkv, double s_qkv, int64_t B, int64_t T, int64_t H,
                           int64_t hd, const double* s_params, const int64_t* z_params,
                           const int32_t* mul_table, int32_t p_signed, void* out,
                           int64_t out_stride, void* stream);

/* out[r, :] = table[x[r * every + first, :] + 128]: a Gather of one token per
 * image through its requantization (table: 384 entries). */
int qa_gather_table_dev(const void* x, int64_t x_stride, int32_t x_signed, int64_t every,
                        int64_t first, const int32_t* table, void* out, int64_t out_stride,
                        int64_t rows, int64_t D, void* stream);

/* MatMul of two activations (the reference's float fallback,
 * quant_layers.py:195-205 with the float MatMul of float_ops.py):
 * Y[b, m, n] = clamp(rint(sa * sb * sum_k (A[b,m,k] - za)(B[b,k,n] - zb) / so)
 * + zo, qmin, qmax), the integer sum exact (K * max|a - za| * max|b - zb| <
 * 2^31, else kUnsupported).  A element (b, m, k) is the byte at
 * a + b * a_sb + m * a_sm + k * a_sk, B element (b, k, n) at
 * b + b * b_sb + k * b_sk + n * b_sn (a transposed operand swaps strides);
 * Y element (b, m, n) at y + (b * M + m) * y_stride + n.  Agrees with the
 * reference within one output step (its float32 sum rounds differently). */
int qa_matmul_act_bytes_dev(const void* a, int32_t a_signed, int64_t a_sb, int64_t a_sm,
                            int64_t a_sk, int64_t za, double sa, const void* b, int32_t b_signed,
                            int64_t b_sb, int64_t b_sk, int64_t b_sn, int64_t zb, double sb,
                            void* y, int64_t y_stride, int64_t batch, int64_t M, int64_t N,
                            int64_t K, double so, int64_t zo, int64_t qmin, int64_t qmax,
                            void* stream);

/* Byte rows to int32 and/or float32 (qa_dequantize_f32 semantics). */
int qa_dequantize_rows_dev(const void* x, int64_t x_stride, int32_t x_signed, int64_t zp,
                           double scale, int32_t* q_out, float* f_out, int64_t rows, int64_t C,
                           void* stream);

/* 16-bit transformer layers (int16 ViT graphs), on two-plane int16 tensors
 * (see the 16-bit block below for the plane layout): the token embedding
 * (ta: 65536-entry table indexed by value + 32768, cls_row int32 values),
 * LayerNorm, the attention core (s_params: scales of scores, Mul output,
 * softmax output, attention output; z_params: {zp, qmin, qmax} of each;
 * mul_params: {constant, its zp, scores zp, mult, shift} of the integer
 * scale Mul), the class-token Gather (65536-entry table) and the output
 * dequantize -- the 8-bit route's float-fallback arithmetic
 * (quant_layers.py:195-205), integer products exact. */
int qa_vit_embed16_dev(const void* x, int64_t x_plane, int64_t x_stride, const int32_t* ta,
                       const int32_t* pos, const int32_t* cls_row, int64_t qmin, int64_t qmax,
                       void* out, int64_t out_plane, int64_t out_stride, int64_t B, int64_t T,
                       int64_t D, void* stream);
int qa_layernorm16_dev(const void* x, int64_t x_plane, int64_t x_stride, int64_t zp_in,
                       double s_in, const float* gamma, const float* beta, double eps,
                       double s_out, int64_t zp_out, int64_t qmin, int64_t qmax, void* out,
                       int64_t out_plane, int64_t out_stride, int64_t rows, int64_t D,
                       void* stream);
int qa_attention16_dev(const void* qkv, int64_t qkv_plane, int64_t qkv_stride, int64_t z_qkv,
                       double s_qkv, int64_t B, int64_t T, int64_t H, int64_t hd,
                       const double* s_params, const int64_t* z_params,
                       const int64_t* mul_params, void* out, int64_t out_plane,
                       int64_t out_stride, void* stream);
int qa_gather16_dev(const void* x, int64_t x_plane, int64_t x_stride, int64_t every,
                    int64_t first, const int32_t* table, void* out, int64_t out_plane,
                    int64_t out_stride, int64_t rows, int64_t D, void* stream);
int qa_dequantize_rows16_dev(const void* x, int64_t x_plane, int64_t x_stride, int64_t zp,
                             double scale, int32_t* q_out, float* f_out, int64_t rows, int64_t C,
                             void* stream);

/* 16-bit device-resident layers (int16 graphs: quant_type "int16").
 *
 * An int16 activation tensor is two NHWC byte planes of the same geometry:
 * the low plane holds v & 0xFF, the high plane (`plane` bytes further on)
 * holds v >> 8, so v = lo + 256 * (int8)hi.  Every pointer below names the
 * LOW plane of channel 0 of its view; `*_plane` is the distance in bytes to
 * the high plane.
 *
 * Fused 16-bit Conv / Gemm (ConvQuantize / GemmQuantize with the wide
 * accumulator, quant_layers.py:320-341, 384-401, native.py:363-373 route
 * them to qa_conv_i32_i32_i64 / qa_gemm_i32_i64, qa_kernels.cpp:260-263,
 * 281-284): base.w holds the packed int16 weights as two byte planes
 * [2][base.w_rows][base.w_kp] (low plane rows first), K ordered (ky, kx, c).
 * Dense layers run on the tensor cores as four 8-bit products (lo*lo,
 * lo*hi, hi*lo, hi*hi) in three int32 TMEM accumulators that the epilogue
 * combines exactly in int64 (exact while K * 255 * 255 < 2^31, checked);
 * grouped / depthwise layers run on CUDA cores.  The epilogue is the 8-bit
 * one's layer sequence (requantize with the exact 128-bit mbqm, activation
 * LUT of 65536 entries, residual Add, rescaled Concat copy) on int16 values.
 * base.x_signed, res_signed must be 1; base.fast = 1 asserts that every
 * channel has 0 <= mult < 2^31 and 32 <= 31 + shift <= 94 (the requantize
 * then skips its per-channel check); the pad_corr fields are ignored
 * (out-of-image taps read the raw zero point). */
typedef struct qa_fused_conv16_desc {
  qa_fused_conv_desc base;
  int64_t x_plane, res_plane, out_plane, out2_plane;
  /* optional: base.lut's entries as int16 (every entry in int16 range,
   * base.lut_len <= 65536); dense layers then keep the table in shared
   * memory */
  const int16_t* lut16;
  /* weight byte planes at base.w, each base.w_rows x base.w_kp: 2 (or 0)
   * for int16 weights (v & 0xFF, v >> 8); 3 for the 17-bit centred weights
   * of uint16 graphs (v & 0xFF, (v >> 8) & 0xFF, v >> 16 as a signed byte) */
  int64_t w_planes;
} qa_fused_conv16_desc;

int qa_conv16_fused_dev(const qa_fused_conv16_desc* desc, void* stream);

/* Graph input: float32 NCHW -> int16 planes NHWC with `pix_stride` channels
 * per pixel (channels C.. hold zp), qa_quantize_f32's rounding. */
int qa_quantize_to_planes16_dev(const float* x, void* y, int64_t y_plane, int64_t N, int64_t C,
                                int64_t H, int64_t W, int64_t pix_stride, double scale,
                                int64_t zp, int64_t qmin, int64_t qmax, void* stream);

/* GlobalAveragePool, Softmax fallback and the standalone scale-matching
 * layers (LUT, Add, Concat rescale) of qa_gap_dev, qa_softmax_dev and
 * qa_*_bytes_dev on int16 planes. */
int qa_gap16_dev(const void* x, int64_t x_plane, int64_t x_pix_stride, int64_t N, int64_t HW,
                 int64_t C, int64_t zp_in, int64_t mult, int64_t shift, int64_t zp_out,
                 int64_t qmin, int64_t qmax, void* y, int64_t y_plane, int64_t y_pix_stride,
                 void* stream);
int qa_softmax16_dev(const void* x, int64_t x_plane, int64_t x_pix_stride, int64_t N, int64_t C,
                     double in_scale, int64_t in_zp, double out_scale, int64_t out_zp,
                     int64_t qmin, int64_t qmax, int32_t* q_out, float* y_out, double y_scale,
                     int64_t y_zp, void* stream);
int qa_lut16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y, int64_t y_plane,
                 int64_t y_stride, int64_t rows, int64_t C, int64_t offset, const int32_t* lut,
                 int64_t lut_len, void* stream);
int qa_add16_dev(const void* a, int64_t a_plane, int64_t a_stride, const void* b,
                 int64_t b_plane, int64_t b_stride, void* y, int64_t y_plane, int64_t y_stride,
                 int64_t rows, int64_t C, int64_t za, int64_t ma, int64_t sa, int64_t zb,
                 int64_t mb, int64_t sb, int64_t sign, int64_t zo, int64_t qmin, int64_t qmax,
                 void* stream);
int qa_rescale16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y, int64_t y_plane,
                     int64_t y_stride, int64_t rows, int64_t C, int64_t identity, int64_t zp_in,
                     int64_t m, int64_t s, int64_t zp_out, int64_t qmin, int64_t qmax,
                     void* stream);
int qa_bn16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y, int64_t y_plane,
                int64_t y_stride, int64_t rows, int64_t C, int64_t zp_in, const int64_t* mult,
                const int64_t* shift, const int64_t* post, int64_t zp_out, int64_t qmin,
                int64_t qmax, void* stream);
int qa_mul16_dev(const void* a, int64_t a_plane, int64_t a_stride, const void* b,
                 int64_t b_plane, int64_t b_stride, void* y, int64_t y_plane, int64_t y_stride,
                 int64_t rows, int64_t C, int64_t za, int64_t zb, int64_t m, int64_t s,
                 int64_t zo, int64_t qmin, int64_t qmax, void* stream);
/* MaxPool over int16 planes (out-of-image taps read pad_value: the
 * reference pads with qmin, quant_layers.py:647-648). */
int qa_maxpool16_dev(const void* x, int64_t x_plane, int64_t x_stride, void* y, int64_t y_plane,
                     int64_t y_stride, int64_t N, int64_t H, int64_t W, int64_t C, int64_t KH,
                     int64_t KW, int64_t SH, int64_t SW, int64_t PH, int64_t PW, int64_t DH,
                     int64_t DW, int64_t OH, int64_t OW, int64_t pad_value, void* stream);

/* Allocation-free narrow GEMM.  No counterpart in the reference: it exists
 * for callers that may not allocate GPU memory while they run (a service
 * that reserves all device memory up front and forbids allocation later, a
 * host runtime that passes only the input and output buffers it owns),
 * which the regular entry points cannot serve because they grow device
 * buffers with cudaMalloc on first use.
 *
 * C[M,N] = A[M,K]·B[K,N] (int16 operands, int32 results, bit-identical to
 * qa_gemm_i16_i32) on DEVICE pointers, enqueued on `stream`.  The operands
 * are packed into a fixed 16 MiB library-owned device array that every GPU
 * holds from library load until process exit (qa_noalloc_scratch_bytes());
 * requests needing more (about 2*M*K + 2*N*K bytes) are rejected with an
 * error.  The first call on each device looks up the array's address, so
 * make it before any stream capture.  Calls share the array: calls that
 * overlap on the GPU (different streams, or another thread) race.
 *
 * qa_noalloc_status_dev(stream): after the calls' stream work, reads and
 * clears this entry point's own bounded-wait status word (one device-to-host
 * word copy and a synchronize of `stream`; call it outside any stream
 * capture).  Returns 0, or kDeviceTimeout (3) when a kernel of an earlier
 * call gave up a wait and left that call's C incomplete. */
int64_t qa_noalloc_scratch_bytes(void);
int qa_gemm_i16_i32_noalloc_dev(const int16_t* A, const int16_t* B, int32_t* C, int64_t M,
                                int64_t N, int64_t K, void* stream);
int qa_noalloc_status_dev(void* stream);

/* Output dequantize fused with the multi-GPU output gather.  No reference
 * counterpart: the reference dequantizes each graph output on the host
 * (quant_container.py:186-193, x = (q - zp) * scale in float64, stored as
 * float32) and runs in one process.  Sharded by batch over one process per
 * GPU, each rank calls qa_dequantize_gather_peers_dev once per step: it
 * stores its float32 rows into EVERY rank's gather buffer over NVLink peer
 * memory (plain stores) and waits for the other ranks' rows to land in its
 * own, so no separate collective follows.
 *
 * qa_peer_buffer_create(bytes, &ptr, handle): cudaMalloc's `bytes` (at least
 * qa_peer_buffer_header_bytes()) on the calling thread's device, zeroes the
 * header and writes the buffer's 64-byte CUDA IPC handle to `handle`.
 * qa_peer_buffer_open(handle, &ptr) maps another process's buffer;
 * qa_peer_buffer_close unmaps it; qa_peer_buffer_destroy frees this
 * process's own (after every peer has closed it).
 *
 * Buffer layout: a header of qa_peer_buffer_header_bytes() (4096) bytes --
 * int64 consumed[8] at 0 and ready[8] at 128, written by the ranks, and a
 * CTA counter at 256 -- then two slots of world * rows * cols float32.
 * Epoch e (1, 2, ... per call, the same on every rank) fills slot e & 1 of
 * every rank at rows [rank * rows, (rank + 1) * rows).
 *
 * qa_dequantize_gather_peers_dev(q, q_stride, zp, scale, rows, cols, bases,
 * world, rank, epoch, budget_ns, stream): q is this rank's int32 output
 * [rows, cols] (row stride q_stride elements); bases[r] is rank r's buffer
 * as mapped in this process (bases[rank] = its own), world <= 8.  The launch
 * first tells every rank that this one has consumed epoch - 1 (everything
 * earlier on `stream` has finished), waits until every rank has consumed
 * epoch - 2 before overwriting that slot, stores its rows and then waits
 * until every rank's rows of this epoch have arrived.  Waits give up after
 * budget_ns nanoseconds and set the device status word to kDeviceTimeout
 * (3; read it with qa_device_status_dev). */
int64_t qa_peer_buffer_header_bytes(void);
int qa_peer_buffer_create(int64_t bytes, void** ptr, void* handle);
int qa_peer_buffer_open(const void* handle, void** ptr);
int qa_peer_buffer_close(void* ptr);
int qa_peer_buffer_destroy(void* ptr);
int qa_dequantize_gather_peers_dev(const void* q, int64_t q_stride, int64_t zp, double scale,
                                   int64_t rows, int64_t cols, const void* const* bases,
                                   int32_t world, int32_t rank, int64_t epoch, int64_t budget_ns,
                                   void* stream);

/* Device float pass of calibration (QuantContainer.calibrate(...,
 * device=True)).  The reference runs the float graph on host arrays
 * (float_ops.py, with qa_conv_f32 / qa_gemm_f32) and reduces min / max of
 * every layer output (quant_layers.py:130-137) and graph input
 * (quant_container.py:141-149) with NumPy; these entry points keep the
 * float tensors in device memory and fold the values each kernel writes
 * into that tensor's range slot.  No reference counterpart for the
 * individual symbols.
 *
 * A range slot is two uint32 words {min key, max key}, initialized to
 * {0xFFFFFFFF, 0}, where key(f) = bits(f) ^ (sign ? 0xFFFFFFFF : 0x80000000)
 * orders floats like their values (NaN above +inf).  `range` may be NULL (no
 * reduction).  Float tensors are float32; strides and shapes are in
 * elements, at most 6 dimensions (pass host arrays of `rank` int64).  Every
 * call enqueues on `stream` and returns 0 or an error status.
 *
 * qa_f32_map_dev: y[i] = f(x[i]) for op 0 copy, 1 Sigmoid, 2 Relu,
 *   3 LeakyRelu(p0), 4 Tanh, 5 HardSigmoid(p0, p1), 6 HardSwish, 7 Elu(p0),
 *   8 Softplus, 9 Abs, 10 Neg, 11 Sqrt, 12 Exp, 13 Erf, 14 Gelu (erf),
 *   15 Gelu (tanh), 16 Clip(p0, p1); float64 where float_ops widens.
 * qa_f32_binary_dev: dense y over `shape` = a op b, a and b read through
 *   broadcast strides; op 0 Add, 1 Sub, 2 Mul, 3 Div, 4 Max, 5 Min, 6 Pow.
 * qa_f32_copy_dev: y[sum c * y_strides] = x[sum c * x_strides] over `shape`
 *   (Transpose, Slice, Split, Concat, Pad interior, Expand, Gather).
 * qa_f32_fill_dev: y[0, n) = value (Pad borders).
 * qa_f32_range_dev: folds x[0, n) into the slot (graph inputs, views).
 * qa_f32_range_decode_dev: `count` slots -> float32 pairs (lo, -hi); a
 *   slot never folded gives (+inf, +inf).  One MIN all-reduce of the pairs
 *   combines the tables of several ranks.
 * qa_f32_gemm_dev: C[z] (dense [M, N]) = alpha * A[z] . B[z] for z < batch,
 *   A[z][m][k] at A + z*a_batch + m*a_m + k*a_k, B alike; float32 sums.
 * qa_f32_conv_dev: the qa_conv_f32 convolution on device pointers (same
 *   kernel, same sums); no range (the bias Add that follows folds it).
 * qa_f32_softmax_dev: last-axis softmax of [rows, cols], float64.
 * qa_f32_layernorm_dev: [rows, D] normalized in float64, * gamma (+ beta).
 * qa_f32_maxpool_dev: NCHW max pool, padding reads -inf.
 * qa_f32_plane_mean_dev: y[p] = mean of x[p * HW, (p + 1) * HW). */
int qa_f32_map_dev(const float* x, float* y, int64_t n, int32_t op, float p0, float p1,
                   uint32_t* range, void* stream);
int qa_f32_binary_dev(const float* a, const float* b, float* y, int32_t rank,
                      const int64_t* shape, const int64_t* a_strides, const int64_t* b_strides,
                      int32_t op, uint32_t* range, void* stream);
int qa_f32_copy_dev(const float* x, float* y, int32_t rank, const int64_t* shape,
                    const int64_t* x_strides, const int64_t* y_strides, uint32_t* range,
                    void* stream);
int qa_f32_fill_dev(float* y, int64_t n, float value, uint32_t* range, void* stream);
int qa_f32_range_dev(const float* x, int64_t n, uint32_t* range, void* stream);
int qa_f32_range_decode_dev(const uint32_t* range, float* out, int64_t count, void* stream);
int qa_f32_gemm_dev(const float* A, const float* B, float* C, int64_t batch, int64_t M,
                    int64_t N, int64_t K, int64_t a_batch, int64_t a_m, int64_t a_k,
                    int64_t b_batch, int64_t b_k, int64_t b_n, float alpha, uint32_t* range,
                    void* stream);
int qa_f32_conv_dev(const float* x, const float* w, float* y, int64_t N, int64_t C, int64_t H,
                    int64_t W, int64_t Cout, int64_t KH, int64_t KW, int64_t SH, int64_t SW,
                    int64_t PH, int64_t PW, int64_t DH, int64_t DW, int64_t G, int64_t OH,
                    int64_t OW, void* stream);
int qa_f32_softmax_dev(const float* x, float* y, int64_t rows, int64_t cols, uint32_t* range,
                       void* stream);
int qa_f32_layernorm_dev(const float* x, const float* gamma, const float* beta, float* y,
                         int64_t rows, int64_t D, double eps, uint32_t* range, void* stream);
int qa_f32_maxpool_dev(const float* x, float* y, int64_t NC, int64_t H, int64_t W, int64_t kh,
                       int64_t kw, int64_t sh, int64_t sw, int64_t pt, int64_t pl, int64_t dh,
                       int64_t dw, int64_t OH, int64_t OW, uint32_t* range, void* stream);
int qa_f32_plane_mean_dev(const float* x, float* y, int64_t NC, int64_t HW, uint32_t* range,
                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QA_KERNELS_H_ */
