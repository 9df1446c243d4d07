/*
 * ks_oracle.c -- CPU oracle for the quantized GEMV path (TEST INFRASTRUCTURE).
 *
 * This file is the checker, never the product.  Only tests/, the smoke entry
 * point and the CPU-baseline leg of bench.py load it.  The B200 library
 * (libkernelsmith) does not link it and has no CPU fallback.
 *
 * Every function restates, in plain C99, the arithmetic of the reference
 * libkernelsmith (pkp124/ulir-kernels) for the same inputs:
 *
 *   kso_dot_i8        <- lib/kernelsmith/ks_quantized.c:44-65
 *   kso_matvec_i8     <- lib/kernelsmith/ks_quantized.c:67-91
 *   kso_dot_w4a8      <- lib/kernelsmith/ks_quantized.c:94-127
 *   kso_matvec_w4a8   <- lib/kernelsmith/ks_quantized.c:129-159
 *   kso_unpack_i4     <- lib/kernelsmith/ks_quantized.c:28-33
 *   layout helpers    <- lib/kernelsmith/ks_quantized.c:177-185
 *   kso_rms_norm_f32  <- lib/kernelsmith/ks_normalization.c:13-36
 *   kso_silu_f32      <- lib/kernelsmith/ks_activations.c:39-49
 *   kso_mul_f32       <- lib/kernelsmith/ks_elementwise.c:22-30
 *
 * and composes them for the B200 extensions that have no reference function
 * (per-channel dequant epilogue, f16 group scales, skinny INT8 GEMM with
 * requantisation, per-token activation quantisation, a W4A8 decode layer).
 * The compositions fix the floating-point evaluation order written next to
 * each one; the GPU kernels follow the same order, so their epilogues are
 * bit-exact against this file.
 *
 * Build with -ffp-contract=off: the reference's generic profile is built for
 * baseline x86-64, which has no FMA, so a fused multiply-add would change the
 * rounding of the W4A8 per-element chain.
 *
 * Integer accumulators use uint32_t arithmetic: the reference accumulates in
 * int32_t, and two's-complement wrap-around is what its compiled code does on
 * overflow; uint32_t makes that wrap defined here.
 */

#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define KSO_OK 0
#define KSO_ERR_INVALID_ARG (-1)

static int kso_i8_zp_ok(int32_t zp) { return zp >= -128 && zp <= 127; }
static int kso_i4_zp_ok(int32_t zp) { return zp >= -8 && zp <= 7; }
static int kso_pos_finite(float v) { return v > 0.0f && isfinite(v); }

/* Signed int4 at logical index `index` of a packed byte: even index in bits
 * 0..3, odd index in bits 4..7, two's complement. */
static int32_t kso_unpack_i4(uint8_t byte, size_t index) {
  int32_t nib = (index & 1u) ? (byte >> 4) : (byte & 0x0f);
  return nib >= 8 ? nib - 16 : nib;
}

size_t kso_w4a8_packed_row_bytes(size_t cols) { return cols / 2u + (cols & 1u); }

size_t kso_w4a8_scale_groups(size_t cols, size_t group_size) {
  if (group_size == 0)
    return 0;
  return cols / group_size + (cols % group_size != 0);
}

/* IEEE binary16 bits -> binary32, exact (every half is a float). */
float kso_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0x1f) {
    bits = sign | 0x7f800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {
    /* subnormal half: value = man * 2^-24, exactly representable */
    float v = (float)man * 5.9604644775390625e-08f;
    memcpy(&bits, &v, 4);
    bits |= sign;
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

/* ---------------------------------------------------------------- INT8 --- */

int kso_dot_i8(const int8_t *x, const int8_t *w, size_t k, int32_t zx,
               int32_t zw, int32_t *out) {
  if (!x || !w || !out)
    return KSO_ERR_INVALID_ARG;
  if (!kso_i8_zp_ok(zx) || !kso_i8_zp_ok(zw))
    return KSO_ERR_INVALID_ARG;
  uint32_t acc = 0;
  for (size_t i = 0; i < k; ++i)
    acc += (uint32_t)(((int32_t)x[i] - zx) * ((int32_t)w[i] - zw));
  *out = (int32_t)acc;
  return KSO_OK;
}

int kso_matvec_i8(const int8_t *x, const int8_t *w, size_t stride,
                  int32_t *out, size_t rows, size_t cols, int32_t zx,
                  int32_t zw) {
  if (!x || !w || !out)
    return KSO_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0 || stride < cols)
    return KSO_ERR_INVALID_ARG;
  if (!kso_i8_zp_ok(zx) || !kso_i8_zp_ok(zw))
    return KSO_ERR_INVALID_ARG;
  for (size_t r = 0; r < rows; ++r) {
    int rc = kso_dot_i8(x, w + r * stride, cols, zx, zw, &out[r]);
    if (rc != KSO_OK)
      return rc;
  }
  return KSO_OK;
}

/* Extension: INT8 GEMV with a per-output-channel f32 dequant epilogue.
 * out[r] = (f32(acc[r]) * w_scale[r]) * a_scale, each product rounded to
 * nearest (no FMA). */
int kso_matvec_i8_dequant(const int8_t *x, const int8_t *w, size_t stride,
                          const float *w_scale, float a_scale, float *out,
                          size_t rows, size_t cols, int32_t zx, int32_t zw) {
  if (!w_scale || !out)
    return KSO_ERR_INVALID_ARG;
  for (size_t r = 0; r < rows; ++r) {
    int32_t acc;
    int rc = kso_dot_i8(x, w + r * stride, cols, zx, zw, &acc);
    if (rc != KSO_OK)
      return rc;
    float t = (float)acc * w_scale[r];
    out[r] = t * a_scale;
  }
  return KSO_OK;
}

/* ---------------------------------------------------------------- W4A8 --- */

int kso_dot_w4a8(const int8_t *x, const uint8_t *pw, const float *scales,
                 size_t k, size_t group, float sx, int32_t zx, int32_t zw,
                 float *out) {
  if (!x || !pw || !scales || !out)
    return KSO_ERR_INVALID_ARG;
  if (group == 0)
    return KSO_ERR_INVALID_ARG;
  if (!kso_pos_finite(sx))
    return KSO_ERR_INVALID_ARG;
  if (!kso_i8_zp_ok(zx) || !kso_i4_zp_ok(zw))
    return KSO_ERR_INVALID_ARG;
  size_t groups = kso_w4a8_scale_groups(k, group);
  for (size_t g = 0; g < groups; ++g)
    if (!kso_pos_finite(scales[g]))
      return KSO_ERR_INVALID_ARG;
  /* One f32 chain in k order: acc += (x' * sx) * (w' * s[k / group]). */
  float acc = 0.0f;
  for (size_t i = 0; i < k; ++i) {
    int32_t xv = (int32_t)x[i] - zx;
    int32_t wv = kso_unpack_i4(pw[i / 2], i) - zw;
    float a = (float)xv * sx;
    float b = (float)wv * scales[i / group];
    acc += a * b;
  }
  *out = acc;
  return KSO_OK;
}

int kso_matvec_w4a8(const int8_t *x, const uint8_t *pw, size_t pstride,
                    const float *scales, size_t sstride, float *out,
                    size_t rows, size_t cols, size_t group, float sx,
                    int32_t zx, int32_t zw) {
  if (!x || !pw || !scales || !out)
    return KSO_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0 || group == 0)
    return KSO_ERR_INVALID_ARG;
  if (pstride < kso_w4a8_packed_row_bytes(cols) ||
      sstride < kso_w4a8_scale_groups(cols, group))
    return KSO_ERR_INVALID_ARG;
  /* Rows are written in order; a bad scale row stops the loop, leaving the
   * rows before it written and the rest untouched (reference :148-156). */
  for (size_t r = 0; r < rows; ++r) {
    int rc = kso_dot_w4a8(x, pw + r * pstride, scales + r * sstride, cols,
                          group, sx, zx, zw, &out[r]);
    if (rc != KSO_OK)
      return rc;
  }
  return KSO_OK;
}

/* Extension: the same GEMV with IEEE half scales.  Each half widens exactly
 * to f32, after which the arithmetic is kso_dot_w4a8's, row by row.  A bad
 * scale (<= 0, inf, nan) rejects its row as in the f32 form. */
int kso_matvec_w4a8_f16(const int8_t *x, const uint8_t *pw, size_t pstride,
                        const uint16_t *scales, size_t sstride, float *out,
                        size_t rows, size_t cols, size_t group, float sx,
                        int32_t zx, int32_t zw, float *row_scratch) {
  if (!x || !pw || !scales || !out || !row_scratch)
    return KSO_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0 || group == 0)
    return KSO_ERR_INVALID_ARG;
  size_t groups = kso_w4a8_scale_groups(cols, group);
  if (pstride < kso_w4a8_packed_row_bytes(cols) || sstride < groups)
    return KSO_ERR_INVALID_ARG;
  for (size_t r = 0; r < rows; ++r) {
    for (size_t g = 0; g < groups; ++g)
      row_scratch[g] = kso_f16_to_f32(scales[r * sstride + g]);
    int rc = kso_dot_w4a8(x, pw + r * pstride, row_scratch, cols, group, sx,
                          zx, zw, &out[r]);
    if (rc != KSO_OK)
      return rc;
  }
  return KSO_OK;
}

/* ------------------------------------------------ skinny INT8 GEMM (ext) --- */

/* Round to nearest, ties to even, on an f32 that is already finite. */
static float kso_rne(float v) { return nearbyintf(v); }

static int8_t kso_sat_i8(float r) {
  if (r >= 127.0f)
    return 127;
  if (r <= -128.0f)
    return -128;
  return (int8_t)r;
}

/*
 * out[m, n] = sat_i8(rne(((f32(acc[m, n]) * a_scale[m]) * w_scale[n]) / out_scale))
 * acc[m, n] = sum_k A[m, k] * W[n, k]   (int32, zero points 0)
 * A is [M, K] with row stride lda, W is [N, K] with row stride ldw (the GEMV
 * weight layout), out is [M, N] with row stride ldo.  Each rounding step is
 * one IEEE operation in the order written.
 */
int kso_gemm_i8_requant(const int8_t *a, size_t lda, const float *a_scale,
                        const int8_t *w, size_t ldw, const float *w_scale,
                        float out_scale, int8_t *out, size_t ldo, size_t m,
                        size_t n, size_t k, int32_t *acc_out) {
  if (!a || !a_scale || !w || !w_scale || !out)
    return KSO_ERR_INVALID_ARG;
  if (m == 0 || n == 0 || k == 0 || lda < k || ldw < k || ldo < n)
    return KSO_ERR_INVALID_ARG;
  if (!kso_pos_finite(out_scale))
    return KSO_ERR_INVALID_ARG;
  for (size_t i = 0; i < m; ++i) {
    for (size_t j = 0; j < n; ++j) {
      int32_t acc;
      kso_dot_i8(a + i * lda, w + j * ldw, k, 0, 0, &acc);
      if (acc_out)
        acc_out[i * n + j] = acc;
      float t = (float)acc * a_scale[i];
      t = t * w_scale[j];
      t = t / out_scale;
      out[i * ldo + j] = kso_sat_i8(kso_rne(t));
    }
  }
  return KSO_OK;
}

/* --------------------------------------------- decode-layer helpers (ext) --- */

int kso_rms_norm_f32(const float *in, const float *w, float *out, size_t outer,
                     size_t inner, float eps) {
  if (!in || !w || !out || inner == 0 || eps <= 0.0f || !isfinite(eps))
    return KSO_ERR_INVALID_ARG;
  for (size_t r = 0; r < outer; ++r) {
    const float *row = in + r * inner;
    float ss = 0.0f;
    for (size_t c = 0; c < inner; ++c)
      ss += row[c] * row[c];
    float ms = ss / (float)inner;
    float scale = 1.0f / sqrtf(ms + eps);
    for (size_t c = 0; c < inner; ++c)
      out[r * inner + c] = row[c] * scale * w[c];
  }
  return KSO_OK;
}

int kso_silu_f32(const float *in, float *out, size_t n) {
  if (!in || !out)
    return KSO_ERR_INVALID_ARG;
  for (size_t i = 0; i < n; ++i)
    out[i] = in[i] / (1.0f + expf(-in[i]));
  return KSO_OK;
}

int kso_mul_f32(const float *a, const float *b, float *out, size_t n) {
  if (!a || !b || !out)
    return KSO_ERR_INVALID_ARG;
  for (size_t i = 0; i < n; ++i)
    out[i] = a[i] * b[i];
  return KSO_OK;
}

/*
 * Per-token symmetric activation quantisation (zero point 0):
 *   amax  = max_i |x[i]|            (exact: max is order-free)
 *   scale = amax / 127              (one IEEE division; 1.0 if amax == 0)
 *   q[i]  = sat_i8(rne(x[i] / scale))
 * The reference fixes the rounding (math.roundeven, quantization spec
 * "Lowering Strategy") but not the scale choice; this max-abs rule is the
 * one the B200 decode kernels use.
 */
int kso_quantize_per_token(const float *x, size_t n, int8_t *q, float *scale) {
  if (!x || !q || !scale || n == 0)
    return KSO_ERR_INVALID_ARG;
  float amax = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float a = fabsf(x[i]);
    if (a > amax)
      amax = a;
  }
  float s = amax > 0.0f ? amax / 127.0f : 1.0f;
  for (size_t i = 0; i < n; ++i)
    q[i] = kso_sat_i8(kso_rne(x[i] / s));
  *scale = s;
  return KSO_OK;
}
