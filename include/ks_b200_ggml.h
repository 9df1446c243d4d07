/*
 * ks_b200_ggml.h -- the llama.cpp / GGML operation adapter of libkernelsmith
 * for NVIDIA B200.
 *
 * The reference's integration design routes one selected operation of a
 * pinned llama.cpp build through the public KernelSmith C API behind an
 * opt-in build flag, reports a non-zero invocation count, and converts GGML
 * quantized weights by decoding them to a numerical reference and
 * requantizing to the native layout
 * (docs/design/DES-016-known-runtime-first-transformer-integration.md:60-160,
 * docs/design/DES-015-quantized-layout-abi-and-integration-conversion-paths.md:148-179).
 * The seam here is the decode-oriented one that design names first: GGML's
 * MUL_MAT with a Q4_0 src0 (weights, rows x cols) and an f32 src1
 * (activations, n_tokens x cols), giving an f32 dst (n_tokens x rows).
 *
 * Everything declared here is written on the public ks_b200_* functions of
 * ks_b200.h only, so the same code can live in the runtime's tree; it is
 * compiled into this library for convenience.
 *
 *   weights  ks_b200_ggml_q4_0_create converts a Q4_0 tensor once
 *            (ks_b200_import_ggml_q4_0_async: native group 32, f16 scales)
 *            and keeps the native copy resident on the current device.
 *   MUL_MAT  dst[t, r] = sum_k W[r, k] * x[t, k]: each token's activations
 *            are quantised to int8 (s = max|x| / 127, round half to even) and
 *            multiplied with the W4A8 kernels -- one token: the f32-input
 *            GEMV (ks_b200_matvec_w4a8_f32in_async); more: per-token
 *            quantisation and the tensor-core W4A8 GEMM, up to 64 tokens per
 *            launch.  The results are the W4A8 path's, not GGML's Q4_0 x Q8_0
 *            arithmetic (the design rules out claiming bit-exact Q4_0
 *            compatibility).
 *   report   counters of conversions, MUL_MAT calls, tokens and launches
 *            (the design's invocation counter).
 *
 * Return codes are ks_common.h's (KS_OK, KS_ERR_INVALID_ARG,
 * KS_ERR_UNSUPPORTED) and ks_b200.h's KS_ERR_DEVICE.
 */
#ifndef KS_B200_GGML_H
#define KS_B200_GGML_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A Q4_0 weight tensor converted to the native W4A8 layout, device-resident. */
typedef struct ks_b200_ggml_q4_0 ks_b200_ggml_q4_0;

/*
 * blocks: rows x (cols / 32) Q4_0 blocks of 18 bytes (GGML's block_q4_0),
 * row stride block_row_stride bytes (even), host or device memory, 2-byte
 * aligned.  cols must be a multiple of 256 (the streaming kernels stage whole
 * 16-byte scale rows: cols / 32 f16 scales).  Converts on `stream` and
 * returns after the conversion has finished; *weight receives the handle.
 */
int ks_b200_ggml_q4_0_create(const void *blocks, size_t block_row_stride,
                             size_t rows, size_t cols, void *stream,
                             ks_b200_ggml_q4_0 **weight);

/* Frees the native copy (after the work queued on it has finished). */
int ks_b200_ggml_q4_0_destroy(ks_b200_ggml_q4_0 *weight);

/*
 * The native copy, for diagnostics and tests: packed int4 rows
 * (row stride cols / 2 bytes) and f16 group-32 scales (row stride cols / 32
 * elements), device pointers owned by the handle.
 */
int ks_b200_ggml_q4_0_native(const ks_b200_ggml_q4_0 *weight,
                             const uint8_t **packed, const uint16_t **scales_f16,
                             size_t *rows, size_t *cols);

/*
 * MUL_MAT(src0 = weight, src1) on `stream`: src1 f32 [n_tokens x cols] (row
 * stride src1_stride elements, 16-byte aligned rows), dst f32
 * [n_tokens x rows] (row stride dst_stride elements), device pointers.  The
 * handle's scratch is used for n_tokens > 1, so calls on one handle are
 * ordered by the caller (one stream).  status: KS_B200_STATUS_WORDS device
 * words as for the other asynchronous calls, or NULL (then the handle's own).
 */
int ks_b200_ggml_mul_mat_q4_0_async(const ks_b200_ggml_q4_0 *weight,
                                    const float *src1, size_t src1_stride,
                                    float *dst, size_t dst_stride,
                                    size_t n_tokens, uint32_t *status, void *stream);

/* Invocation report, counted since the library was loaded or last reset. */
typedef struct ks_b200_ggml_report {
  uint64_t conversions;    /* ks_b200_ggml_q4_0_create calls that converted */
  uint64_t mul_mat_calls;  /* ks_b200_ggml_mul_mat_q4_0_async calls queued */
  uint64_t tokens;         /* activation rows multiplied */
  uint64_t gemv_launches;  /* f32-input W4A8 GEMV launches */
  uint64_t gemm_launches;  /* W4A8 GEMM launches (each after a quantisation) */
} ks_b200_ggml_report;

void ks_b200_ggml_report_get(ks_b200_ggml_report *report);
void ks_b200_ggml_report_reset(void);

#ifdef __cplusplus
}
#endif

#endif /* KS_B200_GGML_H */
