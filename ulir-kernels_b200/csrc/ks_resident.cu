// ks_resident.cu -- resident W4A8 weights: upload a packed matrix (or a row
// slice of it, a rank's shard) to the GPU once and run GEMVs on it.
//
// The reference keeps weights in the caller's memory and reads them on every
// call; on a GPU the weights should stay in HBM between calls.  Registration
// copies the rows byte for byte in the ABI layout (signed int4, two per byte,
// low nibble first; group scales row-major), only the row strides may grow
// to a multiple of 16 bytes so the streaming kernel applies (the padding is
// zero and never read).  It checks the caller's quantized layout version
// against KS_QUANT_LAYOUT_VERSION, the version every kernel reads, so a
// converter written for another layout is refused instead of producing
// wrong numbers.

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <string>

#include "ks_b200.h"
#include "ks_internal.h"

struct ks_b200_w4a8_weights {
  uint8_t *packed;       // device, rows x packed_stride bytes
  void *scales;          // device, rows x scale_stride elements
  size_t packed_stride;  // bytes
  size_t scale_stride;   // elements
  size_t rows, cols, group, row_begin;
  int scale_type;
  int device;
};

namespace {

int fail(int code, const std::string &msg) {
  ksb::set_last_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  const std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
  cudaGetLastError();
  return fail(KS_ERR_DEVICE, msg);
}

size_t round16(size_t v) { return (v + 15) / 16 * 16; }

}  // namespace

extern "C" int ks_b200_w4a8_register(const uint8_t *packed_weights, size_t packed_stride_bytes,
                                     const void *weight_scales, int scale_type, size_t scale_stride, size_t rows,
                                     size_t cols, size_t group_size, size_t row_begin, size_t row_count,
                                     int layout_version, ks_b200_w4a8_weights **out) {
  if (!out) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  *out = nullptr;
  if (!packed_weights || !weight_scales) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || group_size == 0 || row_count == 0)
    return fail(KS_ERR_INVALID_ARG, "rows, cols, group_size and row_count must be > 0");
  const size_t row_bytes = cols / 2 + (cols & 1);
  const size_t groups = cols / group_size + (cols % group_size != 0);
  if (packed_stride_bytes < row_bytes || scale_stride < groups)
    return fail(KS_ERR_INVALID_ARG, "stride smaller than one row");
  if (scale_type != KS_B200_SCALE_F32 && scale_type != KS_B200_SCALE_F16)
    return fail(KS_ERR_INVALID_ARG, "scale_type must be KS_B200_SCALE_F32 or KS_B200_SCALE_F16");
  if (row_begin >= rows || row_count > rows - row_begin)
    return fail(KS_ERR_INVALID_ARG, "row_begin + row_count beyond rows");
  if (layout_version != KS_QUANT_LAYOUT_VERSION)
    return fail(KS_ERR_UNSUPPORTED, "quantized layout version " + std::to_string(layout_version) +
                                        "; this library reads version " + std::to_string(KS_QUANT_LAYOUT_VERSION));
  int devcount = 0;
  if (cudaGetDeviceCount(&devcount) != cudaSuccess || devcount == 0) {
    cudaGetLastError();
    return fail(KS_ERR_DEVICE, "no CUDA device available for the B200 kernels");
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const size_t ssize = scale_type == KS_B200_SCALE_F16 ? 2 : 4;
  auto *w = new ks_b200_w4a8_weights{};
  w->packed_stride = round16(row_bytes);
  w->scale_stride = round16(groups * ssize) / ssize;
  w->rows = row_count;
  w->cols = cols;
  w->group = group_size;
  w->row_begin = row_begin;
  w->scale_type = scale_type;
  w->device = dev;
  auto undo = [&](cudaError_t err, const char *what) {
    if (w->packed) cudaFree(w->packed);
    if (w->scales) cudaFree(w->scales);
    delete w;
    return cuda_fail(err, what);
  };
  if ((e = cudaMalloc(reinterpret_cast<void **>(&w->packed), row_count * w->packed_stride)) != cudaSuccess)
    return undo(e, "cudaMalloc(weights)");
  if ((e = cudaMalloc(&w->scales, row_count * w->scale_stride * ssize)) != cudaSuccess)
    return undo(e, "cudaMalloc(scales)");
  // zero the stride padding, then copy the rows (host or device source)
  if ((e = cudaMemset(w->packed, 0, row_count * w->packed_stride)) != cudaSuccess) return undo(e, "cudaMemset");
  if ((e = cudaMemset(w->scales, 0, row_count * w->scale_stride * ssize)) != cudaSuccess) return undo(e, "cudaMemset");
  e = cudaMemcpy2D(w->packed, w->packed_stride, packed_weights + row_begin * packed_stride_bytes, packed_stride_bytes,
                   row_bytes, row_count, cudaMemcpyDefault);
  if (e != cudaSuccess) return undo(e, "cudaMemcpy2D(weights)");
  e = cudaMemcpy2D(w->scales, w->scale_stride * ssize,
                   static_cast<const uint8_t *>(weight_scales) + row_begin * scale_stride * ssize,
                   scale_stride * ssize, groups * ssize, row_count, cudaMemcpyDefault);
  if (e != cudaSuccess) return undo(e, "cudaMemcpy2D(scales)");
  *out = w;
  return KS_OK;
}

extern "C" int ks_b200_w4a8_weights_info(const ks_b200_w4a8_weights *w, const uint8_t **packed_weights,
                                         size_t *packed_stride_bytes, const void **weight_scales,
                                         size_t *scale_stride, size_t *rows, size_t *row_begin) {
  if (!w) return fail(KS_ERR_INVALID_ARG, "NULL handle");
  if (packed_weights) *packed_weights = w->packed;
  if (packed_stride_bytes) *packed_stride_bytes = w->packed_stride;
  if (weight_scales) *weight_scales = w->scales;
  if (scale_stride) *scale_stride = w->scale_stride;
  if (rows) *rows = w->rows;
  if (row_begin) *row_begin = w->row_begin;
  return KS_OK;
}

extern "C" int ks_b200_w4a8_matvec_registered_async(const ks_b200_w4a8_weights *w, const int8_t *input,
                                                    float input_scale, int32_t input_zero_point,
                                                    int32_t weight_zero_point, float *output, uint32_t *status,
                                                    void *stream) {
  if (!w) return fail(KS_ERR_INVALID_ARG, "NULL handle");
  return ks_b200_matvec_w4a8_async(input, w->packed, w->packed_stride, w->scales, w->scale_type, w->scale_stride,
                                   output, w->rows, w->cols, w->group, input_scale, input_zero_point,
                                   weight_zero_point, status, stream);
}

extern "C" int ks_b200_w4a8_release(ks_b200_w4a8_weights *w) {
  if (!w) return KS_OK;
  int cur = -1;
  const bool had = cudaGetDevice(&cur) == cudaSuccess;
  cudaSetDevice(w->device);
  cudaFree(w->packed);
  cudaFree(w->scales);
  if (had) cudaSetDevice(cur);
  cudaGetLastError();
  delete w;
  return KS_OK;
}
