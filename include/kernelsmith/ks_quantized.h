/*
 * kernelsmith/ks_quantized.h -- quantized dot / GEMV C API (B200 build).
 *
 * Drop-in for the reference header of the same name
 * (pkp124/ulir-kernels include/kernelsmith/ks_quantized.h): the same
 * functions with the same signatures, argument meaning, validation order and
 * return codes.  Only the implementation differs: every call runs on an
 * NVIDIA B200 (sm_100a) through hand-written CUDA kernels.
 *
 * Data layout (unchanged from the reference):
 *   INT8 weights  row-major int8, rows x cols, weight_stride elements apart.
 *   W4A8 weights  two's-complement int4, two per byte; for logical index k,
 *                 byte k/2 holds it in bits 0..3 if k is even, bits 4..7 if
 *                 odd.  Rows are packed_stride_bytes apart and hold at least
 *                 ceil(cols/2) bytes.
 *   W4A8 scales   f32, row-major, one per group of group_size columns:
 *                 element k of a row uses scale k / group_size.  Rows are
 *                 scale_stride elements apart.
 *
 * Memory: pointers may be device, managed or host memory.  Device and managed
 * memory is used in place; host memory is staged through device buffers the
 * library owns (correct, but bound by the host link).
 *
 * Synchronisation: each call is synchronous.  Its kernels run on the
 * device's legacy default stream, so they see all work previously queued on
 * blocking streams, and the call returns after the results are in `output`.
 *
 * Threads: calls may be made from several host threads at once.  The library
 * keeps per-thread staging buffers; it has no state that one call leaves for
 * the next to read.
 *
 * Workspace: no function needs caller workspace; every *_workspace query
 * returns 0 and the workspace arguments are ignored, as in the reference.
 *
 * Errors: KS_ERR_INVALID_ARG for any argument the reference rejects,
 * including a weight scale <= 0, inf or nan (found on the device while the
 * rows are computed).  On a bad scale the rows before the first bad row hold
 * their results, as in the reference; later rows are unspecified.  Device
 * failures return KS_ERR_DEVICE (ks_b200.h).
 */

#ifndef KERNELSMITH_QUANTIZED_H
#define KERNELSMITH_QUANTIZED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* output = sum_k (input[k] - input_zero_point) * (weight[k] - weight_zero_point)
 * in int32.  Both zero points must lie in [-128, 127].  k == 0 gives 0.
 * Replaces reference ks_quantized.h:35-37 (ks_quantized.c:44-65). */
int ks_dot_i8(const int8_t *input, const int8_t *weight, size_t k,
              int32_t input_zero_point, int32_t weight_zero_point,
              int32_t *output, void *workspace, size_t ws_size);

/* One int32 dot per weight row: output[r] = ks_dot_i8(input, weights + r *
 * weight_stride, cols, ...).  rows, cols > 0 and weight_stride >= cols.
 * Replaces reference ks_quantized.h:45-48 (ks_quantized.c:67-91). */
int ks_matvec_i8(const int8_t *input, const int8_t *weights,
                 size_t weight_stride, int32_t *output, size_t rows,
                 size_t cols, int32_t input_zero_point,
                 int32_t weight_zero_point, void *workspace, size_t ws_size);

/* output = sum_k ((input[k] - input_zero_point) * input_scale) *
 *                ((int4(weight, k) - weight_zero_point) * weight_scales[k / group_size])
 * in f32.  group_size > 0, input_scale > 0 and finite, input_zero_point in
 * [-128, 127], weight_zero_point in [-8, 7], every one of the
 * ceil(k / group_size) scales > 0 and finite.
 * Replaces reference ks_quantized.h:68-72 (ks_quantized.c:94-127). */
int ks_dot_w4a8(const int8_t *input, const uint8_t *packed_weight,
                const float *weight_scales, size_t k, size_t group_size,
                float input_scale, int32_t input_zero_point,
                int32_t weight_zero_point, float *output, void *workspace,
                size_t ws_size);

/* One W4A8 dot per packed weight row.  rows, cols, group_size > 0,
 * packed_stride_bytes >= ceil(cols / 2), scale_stride >= ceil(cols /
 * group_size).  Replaces reference ks_quantized.h:83-88
 * (ks_quantized.c:129-159). */
int ks_matvec_w4a8(const int8_t *input, const uint8_t *packed_weights,
                   size_t packed_stride_bytes, const float *weight_scales,
                   size_t scale_stride, float *output, size_t rows,
                   size_t cols, size_t group_size, float input_scale,
                   int32_t input_zero_point, int32_t weight_zero_point,
                   void *workspace, size_t ws_size);

/* Workspace queries: all 0 (reference ks_quantized.h:90-93). */
size_t ks_dot_i8_workspace(size_t k);
size_t ks_matvec_i8_workspace(size_t rows, size_t cols);
size_t ks_dot_w4a8_workspace(size_t k, size_t group_size);
size_t ks_matvec_w4a8_workspace(size_t rows, size_t cols, size_t group_size);

/* Preferred buffer alignment in bytes: 16, one 128-bit load
 * (reference ks_quantized.h:94). */
size_t ks_quantized_alignment(void);

/* Layout helpers (reference ks_quantized.h:97-98): ceil(cols / 2), and
 * ceil(cols / group_size) or 0 when group_size == 0. */
size_t ks_w4a8_packed_row_bytes(size_t cols);
size_t ks_w4a8_scale_groups(size_t cols, size_t group_size);

#ifdef __cplusplus
}
#endif

#endif /* KERNELSMITH_QUANTIZED_H */
