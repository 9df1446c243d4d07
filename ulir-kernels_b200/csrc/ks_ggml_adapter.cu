// ks_ggml_adapter.cu -- the GGML MUL_MAT(Q4_0, f32) operation adapter
// (include/ks_b200_ggml.h), written on the public ks_b200_* functions only.
//
// The reference plans this seam without implementing it: a llama.cpp build
// with an opt-in hook sends one selected operation through the KernelSmith C
// API and reports how often it ran
// (docs/design/DES-016-known-runtime-first-transformer-integration.md:60-160).
// Weight conversion follows DES-015:148-179 (decode Q4_0, requantise to the
// native layout with positive scales) through ks_b200_import_ggml_q4_0_async.
// Native group 32 with f16 scales: a Q4_0 block with d > 0 holds values in
// [-8d, 7d] and converts without loss (scale d, codes nibble - 8); with d < 0
// it reaches +8|d|, which becomes 7 * (8|d| / 7), within half a native step.

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <new>
#include <string>

#include "ks_b200.h"
#include "ks_b200_ggml.h"
#include "ks_internal.h"

struct ks_b200_ggml_q4_0 {
  size_t rows = 0, cols = 0;
  int device = -1;
  uint8_t *packed = nullptr;    // rows x cols/2
  uint16_t *scales = nullptr;   // rows x cols/32, f16 bits
  int8_t *xq = nullptr;         // scratch: kTokens x cols quantised activations
  float *xs = nullptr;          // scratch: kTokens scales
  uint32_t *status = nullptr;   // KS_B200_STATUS_WORDS words
};

namespace {

constexpr size_t kGroup = 32;
constexpr size_t kTokens = 64;  // tokens per W4A8 GEMM launch

std::atomic<uint64_t> g_conversions{0}, g_calls{0}, g_tokens{0}, g_gemv{0}, g_gemm{0};

int fail(int code, const char *msg) {
  ksb::set_last_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  cudaGetLastError();
  ksb::set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
  return KS_ERR_DEVICE;
}

void release(ks_b200_ggml_q4_0 *w) {
  cudaFree(w->packed);
  cudaFree(w->scales);
  cudaFree(w->xq);
  cudaFree(w->xs);
  cudaFree(w->status);
  delete w;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int ks_b200_ggml_q4_0_create(const void *blocks, size_t block_row_stride, size_t rows, size_t cols,
                                        void *stream, ks_b200_ggml_q4_0 **weight) {
  if (!blocks || !weight) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  *weight = nullptr;
  if (rows == 0 || cols == 0 || cols % 32)
    return fail(KS_ERR_INVALID_ARG, "rows must be > 0 and cols a positive multiple of 32 (the Q4_0 block)");
  if (cols % 256)
    return fail(KS_ERR_UNSUPPORTED, "cols must be a multiple of 256 (whole 16-byte rows of group-32 f16 scales)");
  if (block_row_stride < cols / 32 * 18 || (block_row_stride & 1u) || (reinterpret_cast<uintptr_t>(blocks) & 1u))
    return fail(KS_ERR_INVALID_ARG, "Q4_0 rows: stride >= (cols/32) * 18 bytes, even, 2-byte aligned");
  if (rows > (size_t(1) << 31)) return fail(KS_ERR_INVALID_ARG, "rows too large");
  int dev = -1, ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return fail(KS_ERR_DEVICE, "no CUDA device");
  }
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto *w = new (std::nothrow) ks_b200_ggml_q4_0;
  if (!w) return fail(KS_ERR_DEVICE, "out of host memory");
  w->rows = rows;
  w->cols = cols;
  w->device = dev;
  const size_t pbytes = rows * (cols / 2), sbytes = rows * (cols / kGroup) * 2;
  if ((e = cudaMalloc(&w->packed, pbytes)) != cudaSuccess || (e = cudaMalloc(&w->scales, sbytes)) != cudaSuccess ||
      (e = cudaMalloc(&w->xq, kTokens * cols)) != cudaSuccess ||
      (e = cudaMalloc(&w->xs, kTokens * sizeof(float))) != cudaSuccess ||
      (e = cudaMalloc(&w->status, KS_B200_STATUS_WORDS * sizeof(uint32_t))) != cudaSuccess) {
    release(w);
    return cuda_fail(e, "cudaMalloc");
  }
  // host blocks are staged through a device copy
  cudaPointerAttributes attr{};
  const bool on_device = cudaPointerGetAttributes(&attr, blocks) == cudaSuccess &&
                         (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged);
  cudaGetLastError();
  void *staged = nullptr;
  const void *src = blocks;
  if (!on_device) {
    const size_t bytes = (rows - 1) * block_row_stride + cols / 32 * 18;
    if ((e = cudaMalloc(&staged, bytes)) != cudaSuccess) {
      release(w);
      return cuda_fail(e, "cudaMalloc(staging)");
    }
    if ((e = cudaMemcpyAsync(staged, blocks, bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess) {
      cudaFree(staged);
      release(w);
      return cuda_fail(e, "cudaMemcpyAsync(blocks)");
    }
    src = staged;
  }
  cudaMemsetAsync(w->status, 0, KS_B200_STATUS_WORDS * sizeof(uint32_t), s);
  int rc = ks_b200_import_ggml_q4_0_async(src, block_row_stride, rows, cols, kGroup, w->packed, cols / 2, w->scales,
                                          KS_B200_SCALE_F16, cols / kGroup, stream);
  e = cudaStreamSynchronize(s);
  if (staged) cudaFree(staged);
  if (rc != KS_OK) {
    release(w);
    return rc;
  }
  if (e != cudaSuccess) {
    release(w);
    return cuda_fail(e, "Q4_0 conversion");
  }
  g_conversions.fetch_add(1, std::memory_order_relaxed);
  *weight = w;
  return KS_OK;
}

extern "C" int ks_b200_ggml_q4_0_destroy(ks_b200_ggml_q4_0 *weight) {
  if (!weight) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  int cur = -1;
  cudaGetDevice(&cur);
  const int dev = weight->device;
  if (cur != dev) cudaSetDevice(dev);
  cudaDeviceSynchronize();  // no queued work may still read the buffers
  release(weight);
  if (cur >= 0 && cur != dev) cudaSetDevice(cur);
  cudaGetLastError();
  return KS_OK;
}

extern "C" int ks_b200_ggml_q4_0_native(const ks_b200_ggml_q4_0 *weight, const uint8_t **packed,
                                        const uint16_t **scales_f16, size_t *rows, size_t *cols) {
  if (!weight) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (packed) *packed = weight->packed;
  if (scales_f16) *scales_f16 = weight->scales;
  if (rows) *rows = weight->rows;
  if (cols) *cols = weight->cols;
  return KS_OK;
}

extern "C" int ks_b200_ggml_mul_mat_q4_0_async(const ks_b200_ggml_q4_0 *weight, const float *src1,
                                               size_t src1_stride, float *dst, size_t dst_stride, size_t n_tokens,
                                               uint32_t *status, void *stream) {
  if (!weight || !src1 || !dst) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  const size_t rows = weight->rows, cols = weight->cols;
  if (n_tokens == 0) return KS_OK;
  if (src1_stride < cols || dst_stride < rows) return fail(KS_ERR_INVALID_ARG, "src1_stride >= cols, dst_stride >= rows");
  if (!aligned16(src1) || (n_tokens > 1 && (src1_stride * sizeof(float)) % 16))
    return fail(KS_ERR_INVALID_ARG, "src1 rows must be 16-byte aligned");
  uint32_t *st = status ? status : weight->status;
  g_calls.fetch_add(1, std::memory_order_relaxed);
  g_tokens.fetch_add(n_tokens, std::memory_order_relaxed);
  auto gemv_tokens = [&](size_t t0, size_t n) {
    for (size_t t = t0; t < t0 + n; ++t) {
      const int rc = ks_b200_matvec_w4a8_f32in_async(src1 + t * src1_stride, weight->packed, cols / 2, weight->scales,
                                                     KS_B200_SCALE_F16, cols / kGroup, dst + t * dst_stride, rows,
                                                     cols, kGroup, nullptr, nullptr, st, stream);
      if (rc != KS_OK) return rc;
      g_gemv.fetch_add(1, std::memory_order_relaxed);
    }
    return KS_OK;
  };
  // one token (the decode GEMV), or output rows the GEMM cannot take
  if (n_tokens == 1 || !aligned16(dst) || (dst_stride * sizeof(float)) % 16) return gemv_tokens(0, n_tokens);
  for (size_t t0 = 0; t0 < n_tokens; t0 += kTokens) {
    const size_t n = n_tokens - t0 < kTokens ? n_tokens - t0 : kTokens;
    int rc = ks_b200_quantize_per_token_async(src1 + t0 * src1_stride, src1_stride, n, cols, weight->xq, cols,
                                              weight->xs, stream);
    if (rc != KS_OK) return rc;
    rc = ks_b200_gemm_w4a8_async(weight->xq, cols, weight->xs, weight->packed, cols / 2, weight->scales,
                                 KS_B200_SCALE_F16, cols / kGroup, dst + t0 * dst_stride, dst_stride, n, rows, cols,
                                 kGroup, st, stream);
    if (rc == KS_ERR_UNSUPPORTED) rc = gemv_tokens(t0, n);
    else if (rc == KS_OK) g_gemm.fetch_add(1, std::memory_order_relaxed);
    if (rc != KS_OK) return rc;
  }
  return KS_OK;
}

extern "C" void ks_b200_ggml_report_get(ks_b200_ggml_report *report) {
  if (!report) return;
  report->conversions = g_conversions.load(std::memory_order_relaxed);
  report->mul_mat_calls = g_calls.load(std::memory_order_relaxed);
  report->tokens = g_tokens.load(std::memory_order_relaxed);
  report->gemv_launches = g_gemv.load(std::memory_order_relaxed);
  report->gemm_launches = g_gemm.load(std::memory_order_relaxed);
}

extern "C" void ks_b200_ggml_report_reset(void) {
  g_conversions.store(0);
  g_calls.store(0);
  g_tokens.store(0);
  g_gemv.store(0);
  g_gemm.store(0);
}
