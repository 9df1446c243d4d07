// ks_capi.cu -- the libkernelsmith C ABI on B200.
//
// Exports every function of kernelsmith/ks_quantized.h and
// kernelsmith/ks_common.h with the reference signatures, plus the extensions
// of ks_b200.h.  Host-side argument checks run first, in the order of the
// reference C (lib/kernelsmith/ks_quantized.c), so an invalid call returns
// the same code without touching the GPU.  Scale validity is checked by the
// kernels while they read the scales and reported through a status word.
//
// There is no CPU fallback: if no CUDA device can run the kernels, compute
// calls return KS_ERR_DEVICE.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ks_b200.h"
#include "ks_internal.h"
#include "b200_sm100a.h"

namespace ksb {
namespace {

constexpr int kMaxDevices = 64;
constexpr uint64_t kWaitLimitNsHost = 1000000000ull;  // the kernels' one-second wait limit
constexpr uint64_t kWaitLimitMaxNs = 10000000000ull;
// kSlotSnap: the caller's device-resident output rows before a W4A8 call;
// kSlotAux: the first-bad-row word of the W4A8 error path.
enum Slot { kSlotX = 0, kSlotW, kSlotS, kSlotY, kSlotS2, kSlotSnap, kSlotAux, kSlots };

struct ThreadState {
  uint32_t *status = nullptr;  // mapped, portable pinned host memory
  struct Buf {
    void *p = nullptr;
    size_t n = 0;
  } bufs[kMaxDevices][kSlots];
  std::vector<unsigned char> host_snap;  // the caller's host-resident output rows before a W4A8 call
  std::string err;
  ~ThreadState() {
    for (int d = 0; d < kMaxDevices; ++d)
      for (int s = 0; s < kSlots; ++s)
        if (bufs[d][s].p) {
          cudaSetDevice(d);
          cudaFree(bufs[d][s].p);
        }
    if (status) cudaFreeHost(status);
  }
};

ThreadState &tls() {
  thread_local ThreadState ts;
  return ts;
}

int fail(int code, const std::string &msg) {
  tls().err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  cudaGetLastError();
  return fail(KS_ERR_DEVICE, m);
}

bool i8_zp_ok(int32_t z) { return z >= -128 && z <= 127; }
bool i4_zp_ok(int32_t z) { return z >= -8 && z <= 7; }
bool pos_finite(float v) { return v > 0.0f && std::isfinite(v); }

size_t packed_row_bytes(size_t cols) { return cols / 2 + (cols & 1); }
size_t scale_groups(size_t cols, size_t g) { return g == 0 ? 0 : cols / g + (cols % g != 0); }

// Where a caller's buffer lives.
struct Where {
  bool device = false;
  int dev = -1;
};

Where classify(const void *p) {
  Where w;
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return w;
  }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
    w.device = true;
    w.dev = at.device;
  }
  return w;
}

// A synchronous call's buffers, resolved to device addresses.  The caller's
// current device is put back when the call returns.
class SyncCall {
 public:
  ~SyncCall() {
    if (prev_dev_ >= 0 && prev_dev_ != dev_) cudaSetDevice(prev_dev_);
  }

  // Pick the device from the device-resident buffers (all must agree) or the
  // thread's current device, and make it current.
  int begin(const void *const *ptrs, int n) {
    int devcount = 0;
    cudaError_t e = cudaGetDeviceCount(&devcount);
    if (e != cudaSuccess || devcount == 0) {
      cudaGetLastError();
      return fail(KS_ERR_DEVICE, "no CUDA device available for the B200 kernels");
    }
    if (cudaGetDevice(&prev_dev_) != cudaSuccess) {
      cudaGetLastError();
      prev_dev_ = -1;
    }
    dev_ = -1;
    for (int i = 0; i < n; ++i) {
      where_[i] = classify(ptrs[i]);
      if (where_[i].device) {
        if (dev_ >= 0 && where_[i].dev != dev_)
          return fail(KS_ERR_INVALID_ARG, "buffers live on different devices");
        dev_ = where_[i].dev;
      }
    }
    if (dev_ < 0 && (e = cudaGetDevice(&dev_)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev_ >= kMaxDevices) return fail(KS_ERR_DEVICE, "device index out of range");
    if ((e = cudaSetDevice(dev_)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    const DeviceProps &dp = device_props(dev_);
    if (dp.cc_major != 10) return fail(KS_ERR_DEVICE, "libkernelsmith (B200) needs an sm_100 device");
    ThreadState &ts = tls();
    if (!ts.status) {
      void *p = nullptr;
      e = cudaHostAlloc(&p, 64, cudaHostAllocMapped | cudaHostAllocPortable);
      if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(status)");
      ts.status = static_cast<uint32_t *>(p);
    }
    ts.status[kStatusBadScale] = 0;
    ts.status[kStatusTimeout] = 0;
    e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&status_dev_), ts.status, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostGetDevicePointer(status)");
    return KS_OK;
  }

  // A thread-local device buffer of at least `bytes` bytes in `slot`.
  int scratch(int slot, size_t bytes, void **out) {
    ThreadState::Buf &b = tls().bufs[dev_][slot];
    if (b.n < bytes) {
      if (b.p) cudaFree(b.p);
      b.p = nullptr;
      b.n = 0;
      cudaError_t e = cudaMalloc(&b.p, bytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
      b.n = bytes;
    }
    *out = b.p;
    return KS_OK;
  }

  bool is_device(int i) const { return where_[i].device; }
  bool bad_scale() const { return static_cast<const volatile uint32_t *>(tls().status)[kStatusBadScale] != 0; }

  // Device address for buffer i of `bytes` bytes; host buffers are staged
  // (inputs copied in now, outputs copied back by finish()).
  int map(int i, int slot, const void *host, size_t bytes, bool input, void **out) {
    if (where_[i].device || bytes == 0) {
      *out = const_cast<void *>(host);
      return KS_OK;
    }
    void *p = nullptr;
    int rc = scratch(slot, bytes, &p);
    if (rc != KS_OK) return rc;
    ThreadState::Buf &b = tls().bufs[dev_][slot];
    if (input) {
      cudaError_t e = cudaMemcpyAsync(b.p, host, bytes, cudaMemcpyHostToDevice, 0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(H2D)");
    } else {
      copy_back_host_ = const_cast<void *>(host);
      copy_back_dev_ = b.p;
      copy_back_bytes_ = bytes;
    }
    *out = b.p;
    return KS_OK;
  }

  int device() const { return dev_; }
  uint32_t *status_dev() const { return status_dev_; }

  // Copy staged outputs back, wait, and turn device status into a code.
  int finish(cudaError_t launch_err) {
    if (launch_err != cudaSuccess) return cuda_fail(launch_err, "kernel launch");
    cudaError_t e;
    if (copy_back_host_) {
      if (height_ > 0)
        e = cudaMemcpy2DAsync(copy_back_host_, pitch_, copy_back_dev_, pitch_, width_, height_,
                              cudaMemcpyDeviceToHost, 0);
      else
        e = cudaMemcpyAsync(copy_back_host_, copy_back_dev_, copy_back_bytes_, cudaMemcpyDeviceToHost, 0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(D2H)");
    }
    e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    const volatile uint32_t *st = tls().status;
    if (st[kStatusTimeout]) return fail(KS_ERR_DEVICE, "a device-side wait timed out");
    if (st[kStatusBadScale]) return fail(KS_ERR_INVALID_ARG, "a weight scale is <= 0, inf or nan");
    return KS_OK;
  }

 private:
  Where where_[8];
  int dev_ = -1;
  int prev_dev_ = -1;
  uint32_t *status_dev_ = nullptr;
  void *copy_back_host_ = nullptr;
  void *copy_back_dev_ = nullptr;
  size_t copy_back_bytes_ = 0;

 public:
  // Stage a strided output of `height` rows of `width` bytes, `pitch` bytes
  // apart: only those bytes are copied back, so the gaps between rows in the
  // caller's buffer keep their contents.
  int map_out_2d(int i, int slot, void *host, size_t pitch, size_t width, size_t height, void **out) {
    if (where_[i].device) {
      *out = host;
      return KS_OK;
    }
    int rc = map(i, slot, host, (height - 1) * pitch + width, false, out);
    if (rc != KS_OK) return rc;
    pitch_ = pitch;
    width_ = width;
    height_ = height;
    return KS_OK;
  }

 private:
  size_t pitch_ = 0, width_ = 0, height_ = 0;
};

// Write a scalar result of a zero-length dot to a device or host pointer.
int write_scalar(void *out, const void *value, size_t bytes) {
  int devcount = 0;
  if (cudaGetDeviceCount(&devcount) != cudaSuccess) cudaGetLastError();
  if (devcount > 0 && classify(out).device) {
    cudaError_t e = cudaMemcpy(out, value, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(scalar)");
  } else {
    std::memcpy(out, value, bytes);
  }
  return KS_OK;
}

// ------------------------------------------------------------- W4A8 core --
int w4a8_sync(const int8_t *x, const uint8_t *w, size_t wstride, const void *s, int stype,
              size_t sstride, float *y, size_t rows, size_t cols, size_t group, float sx,
              int32_t zx, int32_t zw) {
  const size_t ssize = stype == kScaleF16 ? 2 : 4;
  const size_t groups = scale_groups(cols, group);
  SyncCall call;
  const void *ptrs[4] = {x, w, s, y};
  int rc = call.begin(ptrs, 4);
  if (rc != KS_OK) return rc;
  void *dx = nullptr, *dw = nullptr, *ds = nullptr, *dy = nullptr;
  const size_t wbytes = (rows - 1) * wstride + packed_row_bytes(cols);
  const size_t sbytes = ((rows - 1) * sstride + groups) * ssize;
  if ((rc = call.map(0, kSlotX, x, cols, true, &dx)) != KS_OK) return rc;
  if ((rc = call.map(1, kSlotW, w, wbytes, true, &dw)) != KS_OK) return rc;
  if ((rc = call.map(2, kSlotS, s, sbytes, true, &ds)) != KS_OK) return rc;
  if ((rc = call.map(3, kSlotY, y, rows * sizeof(float), false, &dy)) != KS_OK) return rc;
  // The kernels compute every row in one pass, but the reference stops at the
  // first row with a bad scale and leaves that row and all later ones as they
  // were (ks_quantized.c:148-156).  Keep the caller's rows, so the error path
  // below can put them back.
  const size_t ybytes = rows * sizeof(float);
  void *snap = nullptr;
  if (call.is_device(3)) {
    if ((rc = call.scratch(kSlotSnap, ybytes, &snap)) != KS_OK) return rc;
    cudaError_t e = cudaMemcpyAsync(snap, y, ybytes, cudaMemcpyDeviceToDevice, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(output snapshot)");
  } else {
    std::vector<unsigned char> &hs = tls().host_snap;
    if (hs.size() < ybytes) hs.resize(ybytes);
    std::memcpy(hs.data(), y, ybytes);
  }
  W4A8Launch a{};
  a.x = static_cast<const int8_t *>(dx);
  a.w = static_cast<const uint8_t *>(dw);
  a.wstride = (int64_t)wstride;
  a.s = ds;
  a.sstride = (int64_t)sstride;
  a.stype = stype;
  a.y = static_cast<float *>(dy);
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group;
  a.sx = sx;
  a.zx = zx;
  a.zw = zw;
  a.status = call.status_dev();
  rc = call.finish(launch_w4a8(a, 0, call.device()));
  if (rc != KS_ERR_INVALID_ARG || !call.bad_scale()) return rc;
  const std::string msg = tls().err;
  // Bad scale: find the first failing row and restore it and every later row.
  void *aux = nullptr;
  if ((rc = call.scratch(kSlotAux, 256, &aux)) != KS_OK) return rc;
  unsigned long long first = ~0ull;
  cudaError_t e = cudaMemsetAsync(aux, 0xFF, sizeof first, 0);
  if (e == cudaSuccess)
    e = launch_w4a8_first_bad_row(ds, stype, (int64_t)sstride, (int64_t)rows, (int64_t)groups,
                                  static_cast<unsigned long long *>(aux), 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&first, aux, sizeof first, cudaMemcpyDeviceToHost, 0);
  if (e == cudaSuccess) e = cudaStreamSynchronize(0);
  if (e != cudaSuccess) return cuda_fail(e, "first bad scale row");
  if (first < rows) {
    const size_t off = (size_t)first * sizeof(float);
    if (call.is_device(3)) {
      e = cudaMemcpyAsync(reinterpret_cast<unsigned char *>(y) + off, static_cast<unsigned char *>(snap) + off,
                          ybytes - off, cudaMemcpyDeviceToDevice, 0);
      if (e == cudaSuccess) e = cudaStreamSynchronize(0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(output restore)");
    } else {
      std::memcpy(reinterpret_cast<unsigned char *>(y) + off, tls().host_snap.data() + off, ybytes - off);
    }
  }
  return fail(KS_ERR_INVALID_ARG, msg);
}

// Checks of ks_matvec_w4a8 (ks_quantized.c:138-146) followed by the per-row
// checks of ks_dot_w4a8 that do not depend on the row (:100-110).
int w4a8_matvec_checks(const int8_t *x, const uint8_t *w, size_t wstride, const void *s,
                       size_t sstride, const float *y, size_t rows, size_t cols, size_t group,
                       float sx, int32_t zx, int32_t zw) {
  if (!x || !w || !s || !y) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || group == 0) return fail(KS_ERR_INVALID_ARG, "rows, cols and group_size must be > 0");
  if (wstride < packed_row_bytes(cols) || sstride < scale_groups(cols, group))
    return fail(KS_ERR_INVALID_ARG, "stride smaller than one row");
  if (!pos_finite(sx)) return fail(KS_ERR_INVALID_ARG, "input_scale must be > 0 and finite");
  if (!i8_zp_ok(zx) || !i4_zp_ok(zw)) return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  return KS_OK;
}

int i8_sync(const int8_t *x, const int8_t *w, size_t wstride, void *y, size_t rows, size_t cols,
            int32_t zx, int32_t zw, const float *ws, float sa, bool out_f32) {
  SyncCall call;
  const void *ptrs[4] = {x, w, y, ws ? static_cast<const void *>(ws) : static_cast<const void *>(x)};
  int rc = call.begin(ptrs, 4);
  if (rc != KS_OK) return rc;
  void *dx = nullptr, *dw = nullptr, *dy = nullptr, *dws = nullptr;
  const size_t wbytes = (rows - 1) * wstride + cols;
  if ((rc = call.map(0, kSlotX, x, cols, true, &dx)) != KS_OK) return rc;
  if ((rc = call.map(1, kSlotW, w, wbytes, true, &dw)) != KS_OK) return rc;
  if (out_f32 && (rc = call.map(3, kSlotS, ws, rows * sizeof(float), true, &dws)) != KS_OK) return rc;
  if ((rc = call.map(2, kSlotY, y, rows * 4, false, &dy)) != KS_OK) return rc;
  I8Launch a{};
  a.x = static_cast<const int8_t *>(dx);
  a.w = static_cast<const int8_t *>(dw);
  a.wstride = (int64_t)wstride;
  a.y = dy;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.zx = zx;
  a.zw = zw;
  a.ws = static_cast<const float *>(dws);
  a.sa = sa;
  a.out_f32 = out_f32 ? 1 : 0;
  a.status = call.status_dev();
  return call.finish(launch_i8(a, 0, call.device()));
}

int gemm_checks(const int8_t *a, size_t lda, const float *sa, const int8_t *w, size_t ldw, const float *ws,
                float out_scale, const int8_t *out, size_t ldo, size_t m, size_t n, size_t k) {
  if (!a || !sa || !w || !ws || !out) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (m == 0 || n == 0 || k == 0) return fail(KS_ERR_INVALID_ARG, "m, n and k must be > 0");
  if (lda < k || ldw < k || ldo < n) return fail(KS_ERR_INVALID_ARG, "leading dimension too small");
  if (!pos_finite(out_scale)) return fail(KS_ERR_INVALID_ARG, "out_scale must be > 0 and finite");
  if (m > (size_t)INT32_MAX || n > (size_t)INT32_MAX || k > (size_t)INT32_MAX)
    return fail(KS_ERR_UNSUPPORTED, "dimension beyond 2^31 - 1");
  return KS_OK;
}

int gemm_sync(const int8_t *a, size_t lda, const float *sa, const int8_t *w, size_t ldw, const float *ws,
              float out_scale, int8_t *out, size_t ldo, size_t m, size_t n, size_t k) {
  SyncCall call;
  const void *ptrs[5] = {a, w, sa, ws, out};
  int rc = call.begin(ptrs, 5);
  if (rc != KS_OK) return rc;
  void *da = nullptr, *dw = nullptr, *dsa = nullptr, *dws = nullptr, *dout = nullptr;
  if ((rc = call.map(0, kSlotX, a, (m - 1) * lda + k, true, &da)) != KS_OK) return rc;
  if ((rc = call.map(1, kSlotW, w, (n - 1) * ldw + k, true, &dw)) != KS_OK) return rc;
  if ((rc = call.map(2, kSlotS, sa, m * sizeof(float), true, &dsa)) != KS_OK) return rc;
  if ((rc = call.map(3, kSlotS2, ws, n * sizeof(float), true, &dws)) != KS_OK) return rc;
  if ((rc = call.map_out_2d(4, kSlotY, out, ldo, n, m, &dout)) != KS_OK) return rc;
  GemmI8Launch g{};
  g.a = static_cast<const int8_t *>(da);
  g.lda = (int64_t)lda;
  g.sa = static_cast<const float *>(dsa);
  g.w = static_cast<const int8_t *>(dw);
  g.ldw = (int64_t)ldw;
  g.ws = static_cast<const float *>(dws);
  g.out_scale = out_scale;
  g.out = static_cast<int8_t *>(dout);
  g.ldo = (int64_t)ldo;
  g.m = (int64_t)m;
  g.n = (int64_t)n;
  g.k = (int64_t)k;
  g.acc_out = nullptr;
  g.status = call.status_dev();
  return call.finish(launch_gemm_i8(g, 0, call.device()));
}

int current_device(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(KS_ERR_DEVICE, "device index out of range");
  return KS_OK;
}

}  // namespace

void set_last_error(const std::string &msg) { tls().err = msg; }

}  // namespace ksb

using namespace ksb;

// ================================================================ ks_common
extern "C" const char *ks_target_name(void) { return KS_TARGET_NAME; }
extern "C" size_t ks_simd_width_f32(void) { return KS_SIMD_WIDTH_F32; }

// ============================================================= ks_quantized
extern "C" int ks_dot_i8(const int8_t *input, const int8_t *weight, size_t k,
                         int32_t input_zero_point, int32_t weight_zero_point, int32_t *output,
                         void *workspace, size_t ws_size) {
  (void)workspace;
  (void)ws_size;
  if (!input || !weight || !output) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (!i8_zp_ok(input_zero_point) || !i8_zp_ok(weight_zero_point))
    return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  if (k == 0) {
    const int32_t zero = 0;
    return write_scalar(output, &zero, sizeof zero);
  }
  return i8_sync(input, weight, k, output, 1, k, input_zero_point, weight_zero_point, nullptr,
                 0.0f, false);
}

extern "C" int ks_matvec_i8(const int8_t *input, const int8_t *weights, size_t weight_stride,
                            int32_t *output, size_t rows, size_t cols, int32_t input_zero_point,
                            int32_t weight_zero_point, void *workspace, size_t ws_size) {
  (void)workspace;
  (void)ws_size;
  if (!input || !weights || !output) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || weight_stride < cols)
    return fail(KS_ERR_INVALID_ARG, "rows/cols must be > 0 and weight_stride >= cols");
  if (!i8_zp_ok(input_zero_point) || !i8_zp_ok(weight_zero_point))
    return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  return i8_sync(input, weights, weight_stride, output, rows, cols, input_zero_point,
                 weight_zero_point, nullptr, 0.0f, false);
}

extern "C" int ks_dot_w4a8(const int8_t *input, const uint8_t *packed_weight,
                           const float *weight_scales, size_t k, size_t group_size,
                           float input_scale, int32_t input_zero_point, int32_t weight_zero_point,
                           float *output, void *workspace, size_t ws_size) {
  (void)workspace;
  (void)ws_size;
  if (!input || !packed_weight || !weight_scales || !output) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (group_size == 0) return fail(KS_ERR_INVALID_ARG, "group_size must be > 0");
  if (!pos_finite(input_scale)) return fail(KS_ERR_INVALID_ARG, "input_scale must be > 0 and finite");
  if (!i8_zp_ok(input_zero_point) || !i4_zp_ok(weight_zero_point))
    return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  if (k == 0) {
    const float zero = 0.0f;
    return write_scalar(output, &zero, sizeof zero);
  }
  return w4a8_sync(input, packed_weight, packed_row_bytes(k), weight_scales, kScaleF32,
                   scale_groups(k, group_size), output, 1, k, group_size, input_scale,
                   input_zero_point, weight_zero_point);
}

extern "C" int ks_matvec_w4a8(const int8_t *input, const uint8_t *packed_weights,
                              size_t packed_stride_bytes, const float *weight_scales,
                              size_t scale_stride, float *output, size_t rows, size_t cols,
                              size_t group_size, float input_scale, int32_t input_zero_point,
                              int32_t weight_zero_point, void *workspace, size_t ws_size) {
  (void)workspace;
  (void)ws_size;
  int rc = w4a8_matvec_checks(input, packed_weights, packed_stride_bytes, weight_scales,
                              scale_stride, output, rows, cols, group_size, input_scale,
                              input_zero_point, weight_zero_point);
  if (rc != KS_OK) return rc;
  return w4a8_sync(input, packed_weights, packed_stride_bytes, weight_scales, kScaleF32,
                   scale_stride, output, rows, cols, group_size, input_scale, input_zero_point,
                   weight_zero_point);
}

extern "C" size_t ks_dot_i8_workspace(size_t k) { return KS_QUANT_DOT_I8_WORKSPACE_BYTES(k); }
extern "C" size_t ks_matvec_i8_workspace(size_t rows, size_t cols) {
  return KS_QUANT_MATVEC_I8_WORKSPACE_BYTES(rows, cols);
}
extern "C" size_t ks_dot_w4a8_workspace(size_t k, size_t group_size) {
  return KS_QUANT_DOT_W4A8_WORKSPACE_BYTES(k, group_size);
}
extern "C" size_t ks_matvec_w4a8_workspace(size_t rows, size_t cols, size_t group_size) {
  return KS_QUANT_MATVEC_W4A8_WORKSPACE_BYTES(rows, cols, group_size);
}
extern "C" size_t ks_quantized_alignment(void) { return KS_PREFERRED_ALIGN; }
extern "C" size_t ks_w4a8_packed_row_bytes(size_t cols) { return packed_row_bytes(cols); }
extern "C" size_t ks_w4a8_scale_groups(size_t cols, size_t group_size) {
  return scale_groups(cols, group_size);
}

// ================================================================ ks_b200.h
extern "C" const char *ks_b200_version(void) { return KS_B200_VERSION_STRING; }
extern "C" const char *ks_b200_last_error(void) { return tls().err.c_str(); }

extern "C" int ks_b200_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

extern "C" int ks_b200_matvec_w4a8_f16(const int8_t *input, const uint8_t *packed_weights,
                                       size_t packed_stride_bytes, const uint16_t *weight_scales_f16,
                                       size_t scale_stride, float *output, size_t rows, size_t cols,
                                       size_t group_size, float input_scale,
                                       int32_t input_zero_point, int32_t weight_zero_point) {
  int rc = w4a8_matvec_checks(input, packed_weights, packed_stride_bytes, weight_scales_f16,
                              scale_stride, output, rows, cols, group_size, input_scale,
                              input_zero_point, weight_zero_point);
  if (rc != KS_OK) return rc;
  return w4a8_sync(input, packed_weights, packed_stride_bytes, weight_scales_f16, kScaleF16,
                   scale_stride, output, rows, cols, group_size, input_scale, input_zero_point,
                   weight_zero_point);
}

extern "C" int ks_b200_matvec_i8_dequant(const int8_t *input, const int8_t *weights,
                                         size_t weight_stride, const float *weight_scales,
                                         float input_scale, float *output, size_t rows, size_t cols,
                                         int32_t input_zero_point, int32_t weight_zero_point) {
  if (!input || !weights || !output || !weight_scales) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || weight_stride < cols)
    return fail(KS_ERR_INVALID_ARG, "rows/cols must be > 0 and weight_stride >= cols");
  if (!i8_zp_ok(input_zero_point) || !i8_zp_ok(weight_zero_point))
    return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  return i8_sync(input, weights, weight_stride, output, rows, cols, input_zero_point,
                 weight_zero_point, weight_scales, input_scale, true);
}

extern "C" int ks_b200_matvec_w4a8_async(const int8_t *input, const uint8_t *packed_weights,
                                         size_t packed_stride_bytes, const void *weight_scales,
                                         int scale_type, size_t scale_stride, float *output,
                                         size_t rows, size_t cols, size_t group_size,
                                         float input_scale, int32_t input_zero_point,
                                         int32_t weight_zero_point, uint32_t *status, void *stream) {
  if (scale_type != kScaleF32 && scale_type != kScaleF16)
    return fail(KS_ERR_INVALID_ARG, "unknown scale_type");
  int rc = w4a8_matvec_checks(input, packed_weights, packed_stride_bytes, weight_scales,
                              scale_stride, output, rows, cols, group_size, input_scale,
                              input_zero_point, weight_zero_point);
  if (rc != KS_OK) return rc;
  int dev;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  W4A8Launch a{};
  a.x = input;
  a.w = packed_weights;
  a.wstride = (int64_t)packed_stride_bytes;
  a.s = weight_scales;
  a.sstride = (int64_t)scale_stride;
  a.stype = scale_type;
  a.y = output;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  a.sx = input_scale;
  a.zx = input_zero_point;
  a.zw = weight_zero_point;
  a.status = status;
  cudaError_t e = launch_w4a8(a, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

static int i8_async(const int8_t *input, const int8_t *weights, size_t weight_stride, void *output,
                    size_t rows, size_t cols, int32_t zx, int32_t zw, const float *ws, float sa,
                    bool out_f32, void *stream) {
  if (!input || !weights || !output || (out_f32 && !ws)) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || weight_stride < cols)
    return fail(KS_ERR_INVALID_ARG, "rows/cols must be > 0 and weight_stride >= cols");
  if (!i8_zp_ok(zx) || !i8_zp_ok(zw)) return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  I8Launch a{};
  a.x = input;
  a.w = weights;
  a.wstride = (int64_t)weight_stride;
  a.y = output;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.zx = zx;
  a.zw = zw;
  a.ws = ws;
  a.sa = sa;
  a.out_f32 = out_f32 ? 1 : 0;
  a.status = nullptr;
  cudaError_t e = launch_i8(a, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_matvec_i8_async(const int8_t *input, const int8_t *weights,
                                       size_t weight_stride, int32_t *output, size_t rows,
                                       size_t cols, int32_t input_zero_point,
                                       int32_t weight_zero_point, void *stream) {
  return i8_async(input, weights, weight_stride, output, rows, cols, input_zero_point,
                  weight_zero_point, nullptr, 0.0f, false, stream);
}

extern "C" int ks_b200_matvec_i8_dequant_async(const int8_t *input, const int8_t *weights,
                                               size_t weight_stride, const float *weight_scales,
                                               float input_scale, float *output, size_t rows,
                                               size_t cols, int32_t input_zero_point,
                                               int32_t weight_zero_point, void *stream) {
  return i8_async(input, weights, weight_stride, output, rows, cols, input_zero_point,
                  weight_zero_point, weight_scales, input_scale, true, stream);
}

extern "C" int ks_b200_gemm_w4a8_async(const int8_t *a, size_t lda, const float *a_scales,
                                       const uint8_t *packed_weights, size_t packed_stride_bytes,
                                       const void *weight_scales, int scale_type, size_t scale_stride, float *out,
                                       size_t ldo, size_t m, size_t n, size_t k, size_t group_size,
                                       uint32_t *status, void *stream) {
  if (!a || !a_scales || !packed_weights || !weight_scales || !out) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (m == 0 || n == 0 || k == 0 || group_size == 0) return fail(KS_ERR_INVALID_ARG, "m, n, k, group_size must be > 0");
  if (lda < k || ldo < n || packed_stride_bytes < packed_row_bytes(k) || scale_stride < scale_groups(k, group_size))
    return fail(KS_ERR_INVALID_ARG, "lda >= k, ldo >= n, packed stride >= ceil(k/2), scale stride >= ceil(k/group)");
  if (scale_type != KS_B200_SCALE_F32 && scale_type != KS_B200_SCALE_F16)
    return fail(KS_ERR_INVALID_ARG, "scale_type must be KS_B200_SCALE_F32 or KS_B200_SCALE_F16");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  GemmW4A8Launch g{};
  g.a = a;
  g.lda = (int64_t)lda;
  g.sx = a_scales;
  g.w = packed_weights;
  g.wstride = (int64_t)packed_stride_bytes;
  g.s = weight_scales;
  g.sstride = (int64_t)scale_stride;
  g.stype = scale_type;
  g.y = out;
  g.ldy = (int64_t)ldo;
  g.m = (int64_t)m;
  g.n = (int64_t)n;
  g.k = (int64_t)k;
  g.group = (int64_t)group_size;
  g.status = status;
  if (!gemm_w4a8_supported(g))
    return fail(KS_ERR_UNSUPPORTED,
                "tensor-core W4A8 GEMM needs m <= 64, k a multiple of 32 and of group_size (32, 64 or 128), "
                "16-byte aligned a / weights / scales with lda, packed stride and scale-row bytes multiples of 16");
  cudaError_t e = launch_gemm_w4a8(g, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_matvec_w4a8_f32in_async(const float *input, const uint8_t *packed_weights,
                                               size_t packed_stride_bytes, const void *weight_scales, int scale_type,
                                               size_t scale_stride, float *output, size_t rows, size_t cols,
                                               size_t group_size, int8_t *quantized_input, float *input_scale,
                                               uint32_t *status, void *stream) {
  if (!input || !packed_weights || !weight_scales || !output) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || group_size == 0) return fail(KS_ERR_INVALID_ARG, "rows, cols, group_size must be > 0");
  if (packed_stride_bytes < packed_row_bytes(cols) || scale_stride < scale_groups(cols, group_size))
    return fail(KS_ERR_INVALID_ARG, "packed stride >= ceil(cols/2), scale stride >= ceil(cols/group)");
  if (scale_type != KS_B200_SCALE_F32 && scale_type != KS_B200_SCALE_F16)
    return fail(KS_ERR_INVALID_ARG, "scale_type must be KS_B200_SCALE_F32 or KS_B200_SCALE_F16");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  W4A8Launch a{};
  a.w = packed_weights;
  a.wstride = (int64_t)packed_stride_bytes;
  a.s = weight_scales;
  a.sstride = (int64_t)scale_stride;
  a.stype = scale_type;
  a.y = output;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  a.sx = 1.0f;
  a.status = status;
  cudaError_t e = launch_w4a8_f32in(a, input, quantized_input, input_scale, static_cast<cudaStream_t>(stream), dev);
  if (e == cudaErrorNotSupported) {
    cudaGetLastError();
    return fail(KS_ERR_UNSUPPORTED,
                "f32-input W4A8 GEMV needs the streaming kernel's shape: cols a multiple of 32, group a power-of-two "
                "multiple of 32, scale-row bytes a multiple of 16, 16-byte aligned input, weights and scales");
  }
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_quantize_per_token_async(const float *x, size_t ldx, size_t n_tokens, size_t cols,
                                                int8_t *q, size_t ldq, float *scales, void *stream) {
  if (!x || !q || !scales) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (n_tokens == 0 || cols == 0) return fail(KS_ERR_INVALID_ARG, "n_tokens and cols must be > 0");
  if (ldx < cols || ldq < cols) return fail(KS_ERR_INVALID_ARG, "ldx >= cols and ldq >= cols");
  if (n_tokens > 0x7FFFFFFF) return fail(KS_ERR_INVALID_ARG, "n_tokens too large");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  cudaError_t e = launch_quantize_tokens(x, (int64_t)ldx, (int64_t)n_tokens, (int64_t)cols, q, (int64_t)ldq, scales,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_quant_layout_version(void) { return KS_QUANT_LAYOUT_VERSION; }

extern "C" int ks_b200_import_ggml_q4_0_async(const void *blocks, size_t block_row_stride, size_t rows,
                                              size_t cols, size_t group_size, uint8_t *packed_weights,
                                              size_t packed_stride_bytes, void *weight_scales, int scale_type,
                                              size_t scale_stride, void *stream) {
  if (!blocks || !packed_weights || !weight_scales) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || cols % 32)
    return fail(KS_ERR_INVALID_ARG, "rows must be > 0 and cols a positive multiple of 32 (the Q4_0 block)");
  if (group_size != 32 && group_size != 64 && group_size != 128 && group_size != 256)
    return fail(KS_ERR_INVALID_ARG, "group_size must be 32, 64, 128 or 256");
  if (cols % group_size) return fail(KS_ERR_INVALID_ARG, "cols must be a multiple of group_size");
  if (scale_type != KS_B200_SCALE_F32 && scale_type != KS_B200_SCALE_F16)
    return fail(KS_ERR_INVALID_ARG, "scale_type must be KS_B200_SCALE_F32 or KS_B200_SCALE_F16");
  if (block_row_stride < cols / 32 * 18) return fail(KS_ERR_INVALID_ARG, "block_row_stride < (cols/32) * 18");
  if ((reinterpret_cast<uintptr_t>(blocks) | block_row_stride) & 1u)
    return fail(KS_ERR_INVALID_ARG, "Q4_0 blocks must be 2-byte aligned with an even row stride");
  if (packed_stride_bytes < cols / 2 || packed_stride_bytes % 16 ||
      (reinterpret_cast<uintptr_t>(packed_weights) & 15u))
    return fail(KS_ERR_INVALID_ARG, "packed rows must be >= cols/2 bytes, 16-byte aligned with a stride multiple of 16");
  if (scale_stride < cols / group_size) return fail(KS_ERR_INVALID_ARG, "scale_stride < cols / group_size");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  ImportQ4Launch a{};
  a.src = static_cast<const uint8_t *>(blocks);
  a.src_stride = (int64_t)block_row_stride;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  a.packed = packed_weights;
  a.packed_stride = (int64_t)packed_stride_bytes;
  a.scales = weight_scales;
  a.scale_type = scale_type;
  a.scale_stride = (int64_t)scale_stride;
  cudaError_t e = launch_import_q4_0(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_w4a8_kernel_path(const void *input, const void *packed_weights,
                                        size_t packed_stride_bytes, const void *weight_scales,
                                        int scale_type, size_t scale_stride, size_t rows,
                                        size_t cols, size_t group_size) {
  if (rows == 0 || cols == 0 || group_size == 0) return -1;
  if (packed_stride_bytes < packed_row_bytes(cols) || scale_stride < scale_groups(cols, group_size))
    return -1;
  if (ks_b200_device_count() == 0) return -1;
  W4A8Launch a{};
  a.x = static_cast<const int8_t *>(input);
  a.w = static_cast<const uint8_t *>(packed_weights);
  a.wstride = (int64_t)packed_stride_bytes;
  a.s = weight_scales;
  a.sstride = (int64_t)scale_stride;
  a.stype = scale_type;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  return w4a8_path(a);
}

extern "C" int ks_b200_i8_kernel_path(const void *input, const void *weights, size_t weight_stride,
                                      size_t rows, size_t cols) {
  if (rows == 0 || cols == 0 || weight_stride < cols) return -1;
  if (ks_b200_device_count() == 0) return -1;
  I8Launch a{};
  a.x = static_cast<const int8_t *>(input);
  a.w = static_cast<const int8_t *>(weights);
  a.wstride = (int64_t)weight_stride;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  return i8_path(a);
}

extern "C" int ks_b200_gemm_i8_requant(const int8_t *a, size_t lda, const float *a_scales, const int8_t *w,
                                       size_t ldw, const float *w_scales, float out_scale, int8_t *out,
                                       size_t ldo, size_t m, size_t n, size_t k) {
  int rc = gemm_checks(a, lda, a_scales, w, ldw, w_scales, out_scale, out, ldo, m, n, k);
  if (rc != KS_OK) return rc;
  return gemm_sync(a, lda, a_scales, w, ldw, w_scales, out_scale, out, ldo, m, n, k);
}

extern "C" int ks_b200_gemm_i8_requant_async(const int8_t *a, size_t lda, const float *a_scales,
                                             const int8_t *w, size_t ldw, const float *w_scales,
                                             float out_scale, int8_t *out, size_t ldo, size_t m, size_t n,
                                             size_t k, int32_t *acc_out, uint32_t *status, void *stream) {
  int rc = gemm_checks(a, lda, a_scales, w, ldw, w_scales, out_scale, out, ldo, m, n, k);
  if (rc != KS_OK) return rc;
  int dev;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  GemmI8Launch g{};
  g.a = a;
  g.lda = (int64_t)lda;
  g.sa = a_scales;
  g.w = w;
  g.ldw = (int64_t)ldw;
  g.ws = w_scales;
  g.out_scale = out_scale;
  g.out = out;
  g.ldo = (int64_t)ldo;
  g.m = (int64_t)m;
  g.n = (int64_t)n;
  g.k = (int64_t)k;
  g.acc_out = acc_out;
  g.status = status;
  cudaError_t e = launch_gemm_i8(g, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_gemm_i8_requant_batch_async(int count, const int8_t *const *a, size_t lda,
                                                   const float *const *a_scales, const int8_t *const *w,
                                                   size_t ldw, const float *const *w_scales, float out_scale,
                                                   int8_t *const *out, size_t ldo, size_t m, size_t n, size_t k,
                                                   uint32_t *status, void *stream) {
  if (count < 0 || (count > 0 && (!a || !a_scales || !w || !w_scales || !out)))
    return fail(KS_ERR_INVALID_ARG, "bad batch arrays");
  for (int i = 0; i < count; ++i) {
    const int rc = gemm_checks(a[i], lda, a_scales[i], w[i], ldw, w_scales[i], out_scale, out[i], ldo, m, n, k);
    if (rc != KS_OK) return rc;
  }
  if (count == 0) return KS_OK;
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  GemmI8Launch g{};
  g.lda = (int64_t)lda;
  g.ldw = (int64_t)ldw;
  g.out_scale = out_scale;
  g.ldo = (int64_t)ldo;
  g.m = (int64_t)m;
  g.n = (int64_t)n;
  g.k = (int64_t)k;
  g.status = status;
  GemmI8Batch b{count, a, a_scales, w, w_scales, out};
  cudaError_t e = launch_gemm_i8_batch(g, b, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_gemm_i8_kernel_path(const void *a, size_t lda, const void *w, size_t ldw, size_t m,
                                           size_t n, size_t k) {
  if (m == 0 || n == 0 || k == 0 || lda < k || ldw < k) return -1;
  if (ks_b200_device_count() == 0) return -1;
  GemmI8Launch g{};
  g.a = static_cast<const int8_t *>(a);
  g.lda = (int64_t)lda;
  g.w = static_cast<const int8_t *>(w);
  g.ldw = (int64_t)ldw;
  g.m = (int64_t)m;
  g.n = (int64_t)n;
  g.k = (int64_t)k;
  return gemm_i8_path(g);
}

// ===================================================== batched (grouped) GEMV
extern "C" int ks_b200_matvec_w4a8_batch_async(int count, const int8_t *const *inputs,
                                               const uint8_t *const *packed_weights,
                                               const void *const *weight_scales, float *const *outputs,
                                               size_t packed_stride_bytes, int scale_type, size_t scale_stride,
                                               size_t rows, size_t cols, size_t group_size, float input_scale,
                                               int32_t input_zero_point, int32_t weight_zero_point,
                                               uint32_t *status, void *stream) {
  if (count < 0 || (count > 0 && (!inputs || !packed_weights || !weight_scales || !outputs)))
    return fail(KS_ERR_INVALID_ARG, "bad batch arrays");
  if (scale_type != kScaleF32 && scale_type != kScaleF16) return fail(KS_ERR_INVALID_ARG, "unknown scale_type");
  for (int i = 0; i < count; ++i) {
    int rc = w4a8_matvec_checks(inputs[i], packed_weights[i], packed_stride_bytes, weight_scales[i],
                                scale_stride, outputs[i], rows, cols, group_size, input_scale, input_zero_point,
                                weight_zero_point);
    if (rc != KS_OK) return rc;
  }
  if (count == 0) return KS_OK;
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  W4A8Launch a{};
  a.wstride = (int64_t)packed_stride_bytes;
  a.sstride = (int64_t)scale_stride;
  a.stype = scale_type;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  a.sx = input_scale;
  a.zx = input_zero_point;
  a.zw = weight_zero_point;
  a.status = status;
  GemvBatch b{count, inputs, reinterpret_cast<const void *const *>(packed_weights), weight_scales,
              reinterpret_cast<void *const *>(outputs)};
  cudaError_t e = launch_w4a8_batch(a, b, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_matvec_i8_batch_async(int count, const int8_t *const *inputs,
                                             const int8_t *const *weights, const float *const *weight_scales,
                                             void *const *outputs, size_t weight_stride, size_t rows, size_t cols,
                                             int32_t input_zero_point, int32_t weight_zero_point,
                                             float input_scale, void *stream) {
  if (count < 0 || (count > 0 && (!inputs || !weights || !outputs)))
    return fail(KS_ERR_INVALID_ARG, "bad batch arrays");
  if (rows == 0 || cols == 0 || weight_stride < cols)
    return fail(KS_ERR_INVALID_ARG, "rows/cols must be > 0 and weight_stride >= cols");
  if (!i8_zp_ok(input_zero_point) || !i8_zp_ok(weight_zero_point))
    return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  for (int i = 0; i < count; ++i)
    if (!inputs[i] || !weights[i] || !outputs[i] || (weight_scales && !weight_scales[i]))
      return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (count == 0) return KS_OK;
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  I8Launch a{};
  a.wstride = (int64_t)weight_stride;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.zx = input_zero_point;
  a.zw = weight_zero_point;
  a.sa = input_scale;
  a.out_f32 = weight_scales ? 1 : 0;
  GemvBatch b{count, inputs, reinterpret_cast<const void *const *>(weights),
              reinterpret_cast<const void *const *>(weight_scales), outputs};
  cudaError_t e = launch_i8_batch(a, b, static_cast<cudaStream_t>(stream), dev);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

// ============================================ multi-GPU: IPC and peer gather
namespace {
using GetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}
}  // namespace

extern "C" int ks_b200_ipc_get_handle(const void *dev_ptr, unsigned char *handle, size_t *offset) {
  if (!dev_ptr || !handle || !offset) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  Where w = classify(dev_ptr);
  if (!w.device) return fail(KS_ERR_INVALID_ARG, "IPC handles need device memory");
  cudaError_t e = cudaSetDevice(w.dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  GetAddressRangeFn range = address_range_fn();
  if (!range) return fail(KS_ERR_DEVICE, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(KS_ERR_DEVICE, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  if ((e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base))) != cudaSuccess)
    return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof h);
  *offset = reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base);
  return KS_OK;
}

extern "C" int ks_b200_ipc_open_handle(const unsigned char *handle, size_t offset, void **peer_ptr) {
  if (!handle || !peer_ptr) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void *base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *peer_ptr = static_cast<unsigned char *>(base) + offset;
  return KS_OK;
}

extern "C" int ks_b200_ipc_close_handle(void *peer_ptr, size_t offset) {
  if (!peer_ptr) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<unsigned char *>(peer_ptr) - offset);
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

extern "C" int ks_b200_matvec_w4a8_batch_gather_async(
    int count, const int8_t *const *inputs, const uint8_t *const *packed_weights, const void *const *weight_scales,
    int nranks, float *const *rank_outputs, uint32_t *const *rank_counters, size_t matrix_stride, size_t row_offset,
    size_t packed_stride_bytes, int scale_type, size_t scale_stride, size_t rows, size_t cols, size_t group_size,
    float input_scale, int32_t input_zero_point, int32_t weight_zero_point, uint32_t *signals_per_rank,
    uint32_t *status, void *stream) {
  if (!signals_per_rank) return fail(KS_ERR_INVALID_ARG, "NULL signals_per_rank");
  *signals_per_rank = 0;
  if (nranks < 1 || nranks > 8 || !rank_outputs || !rank_counters)
    return fail(KS_ERR_INVALID_ARG, "nranks must be 1..8 with output and counter pointers per rank");
  for (int p = 0; p < nranks; ++p)
    if (!rank_outputs[p] || !rank_counters[p]) return fail(KS_ERR_INVALID_ARG, "NULL rank pointer");
  if (row_offset + rows > matrix_stride) return fail(KS_ERR_INVALID_ARG, "row_offset + rows > matrix_stride");
  if (count < 0 || (count > 0 && (!inputs || !packed_weights || !weight_scales)))
    return fail(KS_ERR_INVALID_ARG, "bad batch arrays");
  if (scale_type != kScaleF32 && scale_type != kScaleF16) return fail(KS_ERR_INVALID_ARG, "unknown scale_type");
  for (int i = 0; i < count; ++i) {
    int rc = w4a8_matvec_checks(inputs[i], packed_weights[i], packed_stride_bytes, weight_scales[i],
                                scale_stride, rank_outputs[0], rows, cols, group_size, input_scale,
                                input_zero_point, weight_zero_point);
    if (rc != KS_OK) return rc;
  }
  if (count == 0) return KS_OK;
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  W4A8Launch a{};
  a.wstride = (int64_t)packed_stride_bytes;
  a.sstride = (int64_t)scale_stride;
  a.stype = scale_type;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  a.sx = input_scale;
  a.zx = input_zero_point;
  a.zw = weight_zero_point;
  a.status = status;
  GemvBatch b{count, inputs, reinterpret_cast<const void *const *>(packed_weights), weight_scales, nullptr};
  PeerGather pg{nranks, rank_outputs, rank_counters, (int64_t)matrix_stride, (int64_t)row_offset};
  cudaError_t e = launch_w4a8_batch_gather(a, b, pg, static_cast<cudaStream_t>(stream), dev, signals_per_rank);
  if (e == cudaErrorInvalidValue)
    return fail(KS_ERR_UNSUPPORTED, "peer-gather GEMV needs the streaming kernel's shape and 16-byte alignment");
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_peer_arrival_wait_async(const uint32_t *counter, uint32_t *expected, uint32_t arrivals,
                                               uint32_t *status, void *stream) {
  if (!counter || !expected) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  cudaError_t e = launch_peer_wait(counter, 1, expected, arrivals, kWaitLimitNsHost, status,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_peer_arrival_wait_ranks_async(const uint32_t *counters, int nranks, uint32_t *expected,
                                                     uint32_t arrivals_per_rank, uint64_t timeout_ns,
                                                     uint32_t *status, void *stream) {
  if (!counters || !expected) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (nranks < 1 || nranks > 8) return fail(KS_ERR_INVALID_ARG, "nranks must be 1..8");
  if (timeout_ns > kWaitLimitMaxNs) return fail(KS_ERR_INVALID_ARG, "timeout_ns above 10 s");
  cudaError_t e = launch_peer_wait(counters, nranks, expected, arrivals_per_rank,
                                   timeout_ns ? timeout_ns : kWaitLimitNsHost, status,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_status_check(const uint32_t *status, void *stream) {
  if (!status) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t words[kStatusWords] = {0, 0};
  e = cudaMemcpy(words, status, sizeof words, cudaMemcpyDefault);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  if (words[kStatusTimeout]) return fail(KS_ERR_DEVICE, "a device-side wait timed out");
  if (words[kStatusBadScale]) return fail(KS_ERR_INVALID_ARG, "a weight scale is <= 0, inf or nan");
  return KS_OK;
}

// ================================================================ decode layer
namespace {
constexpr int kLayerRegions = 11;
// f32 qkv[3h] | h2[h] | gate[i] | up[i] | act[i] | scales[4] | u32 amax[1] |
// int8 q1[h] | q2[h] | q3[h] | q4[i], each region starting on a 256-byte boundary.
void layer_offsets(size_t h, size_t i, size_t off[kLayerRegions + 1]) {
  const size_t sizes[kLayerRegions] = {3 * h * 4, h * 4, i * 4, i * 4, i * 4, 16, 4, h, h, h, i};
  size_t o = 0;
  for (int r = 0; r < kLayerRegions; ++r) {
    off[r] = o;
    o += (sizes[r] + 255) / 256 * 256;
  }
  off[kLayerRegions] = o;
}
}  // namespace

extern "C" size_t ks_b200_decode_layer_workspace(size_t hidden, size_t inter) {
  size_t off[kLayerRegions + 1];
  layer_offsets(hidden, inter, off);
  return off[kLayerRegions];
}

extern "C" int ks_b200_decode_layer_offsets(size_t hidden, size_t inter, size_t *offsets) {
  if (!offsets) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  size_t off[kLayerRegions + 1];
  layer_offsets(hidden, inter, off);
  for (int r = 0; r <= kLayerRegions; ++r) offsets[r] = off[r];
  return KS_OK;
}

extern "C" int ks_b200_decode_layer_w4a8_async(const float *h_in, float *h_out, const float *norm1_w,
                                               const float *norm2_w, float eps, const uint8_t *const *weights,
                                               const uint16_t *const *scales_f16, size_t hidden, size_t inter,
                                               size_t group_size, void *workspace, size_t workspace_bytes,
                                               uint32_t *status, void *stream) {
  if (!h_in || !h_out || !norm1_w || !norm2_w || !weights || !scales_f16 || !workspace)
    return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  for (int k = 0; k < 5; ++k)
    if (!weights[k] || !scales_f16[k]) return fail(KS_ERR_INVALID_ARG, "NULL weight or scale matrix");
  if (!pos_finite(eps)) return fail(KS_ERR_INVALID_ARG, "eps must be > 0 and finite");
  if (hidden == 0 || inter == 0 || hidden % 32 || inter % 32 || group_size < 32 || group_size % 32 ||
      (group_size & (group_size - 1)) || hidden % group_size || inter % group_size)
    return fail(KS_ERR_INVALID_ARG, "hidden and inter must be multiples of 32 and of group_size (a power of two >= 32)");
  if (workspace_bytes < ks_b200_decode_layer_workspace(hidden, inter))
    return fail(KS_ERR_WORKSPACE, "workspace smaller than ks_b200_decode_layer_workspace()");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  size_t off[kLayerRegions + 1];
  layer_offsets(hidden, inter, off);
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  DecodeLayerArgs a{};
  a.h_in = h_in;
  a.h_out = h_out;
  a.norm1_w = norm1_w;
  a.norm2_w = norm2_w;
  a.eps = eps;
  for (int k = 0; k < 5; ++k) {
    a.w[k] = weights[k];
    a.s[k] = scales_f16[k];
  }
  a.hidden = (int64_t)hidden;
  a.inter = (int64_t)inter;
  a.group = (int64_t)group_size;
  a.qkv = reinterpret_cast<float *>(ws + off[0]);
  a.h2 = reinterpret_cast<float *>(ws + off[1]);
  a.gate = reinterpret_cast<float *>(ws + off[2]);
  a.up = reinterpret_cast<float *>(ws + off[3]);
  a.act = reinterpret_cast<float *>(ws + off[4]);
  a.scales = reinterpret_cast<float *>(ws + off[5]);
  a.amax = reinterpret_cast<uint32_t *>(ws + off[6]);
  for (int k = 0; k < 4; ++k) a.q[k] = reinterpret_cast<int8_t *>(ws + off[7 + k]);
  a.status = status;
  cudaError_t e = launch_decode_layer_w4a8(a, static_cast<cudaStream_t>(stream), dev);
  if (e == cudaErrorInvalidValue)
    return fail(KS_ERR_UNSUPPORTED, "decode layer needs 16-byte aligned weights/scales and the streaming shape");
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" size_t ks_b200_decode_layers_workspace(size_t hidden, size_t inter) {
  // the single-layer regions, then the two inter-layer activation vectors
  return ks_b200_decode_layer_workspace(hidden, inter) + 2 * ((hidden * 4 + 255) / 256 * 256);
}

extern "C" int ks_b200_decode_layers_w4a8_async(size_t n_layers, const float *h_in, float *h_out,
                                                const float *const *norm1_w, const float *const *norm2_w,
                                                float eps, const uint8_t *const *weights,
                                                const uint16_t *const *scales_f16, size_t hidden, size_t inter,
                                                size_t group_size, void *workspace, size_t workspace_bytes,
                                                uint32_t *status, void *stream) {
  if (!h_in || !h_out || !norm1_w || !norm2_w || !weights || !scales_f16 || !workspace)
    return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (n_layers == 0 || n_layers > 65536) return fail(KS_ERR_INVALID_ARG, "n_layers must be 1..65536");
  for (size_t l = 0; l < n_layers; ++l) {
    if (!norm1_w[l] || !norm2_w[l]) return fail(KS_ERR_INVALID_ARG, "NULL RMSNorm weight vector");
    for (int k = 0; k < 5; ++k)
      if (!weights[5 * l + k] || !scales_f16[5 * l + k])
        return fail(KS_ERR_INVALID_ARG, "NULL weight or scale matrix");
  }
  if (!pos_finite(eps)) return fail(KS_ERR_INVALID_ARG, "eps must be > 0 and finite");
  if (hidden == 0 || inter == 0 || hidden % 32 || inter % 32 || group_size < 32 || group_size % 32 ||
      (group_size & (group_size - 1)) || hidden % group_size || inter % group_size)
    return fail(KS_ERR_INVALID_ARG, "hidden and inter must be multiples of 32 and of group_size (a power of two >= 32)");
  if (workspace_bytes < ks_b200_decode_layers_workspace(hidden, inter))
    return fail(KS_ERR_WORKSPACE, "workspace smaller than ks_b200_decode_layers_workspace()");
  int dev, rc;
  if ((rc = current_device(&dev)) != KS_OK) return rc;
  size_t off[kLayerRegions + 1];
  layer_offsets(hidden, inter, off);
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  std::vector<DecodeLayerWeights> lw(n_layers);
  for (size_t l = 0; l < n_layers; ++l) {
    for (int k = 0; k < 5; ++k) {
      lw[l].w[k] = weights[5 * l + k];
      lw[l].s[k] = scales_f16[5 * l + k];
    }
    lw[l].norm1_w = norm1_w[l];
    lw[l].norm2_w = norm2_w[l];
  }
  DecodeLayersArgs a{};
  a.layers = (int)n_layers;
  a.lw = lw.data();
  a.h_in = h_in;
  a.h_out = h_out;
  const size_t hb = (hidden * 4 + 255) / 256 * 256;
  a.hbuf[0] = reinterpret_cast<float *>(ws + off[kLayerRegions]);
  a.hbuf[1] = reinterpret_cast<float *>(ws + off[kLayerRegions] + hb);
  a.eps = eps;
  a.hidden = (int64_t)hidden;
  a.inter = (int64_t)inter;
  a.group = (int64_t)group_size;
  a.qkv = reinterpret_cast<float *>(ws + off[0]);
  a.h2 = reinterpret_cast<float *>(ws + off[1]);
  a.gate = reinterpret_cast<float *>(ws + off[2]);
  a.up = reinterpret_cast<float *>(ws + off[3]);
  a.act = reinterpret_cast<float *>(ws + off[4]);
  a.scales = reinterpret_cast<float *>(ws + off[5]);
  a.amax = reinterpret_cast<uint32_t *>(ws + off[6]);
  for (int k = 0; k < 4; ++k) a.q[k] = reinterpret_cast<int8_t *>(ws + off[7 + k]);
  a.status = status;
  cudaError_t e = launch_decode_layers_w4a8(a, static_cast<cudaStream_t>(stream), dev);
  if (e == cudaErrorInvalidValue)
    return fail(KS_ERR_UNSUPPORTED, "decode layers need 16-byte aligned weights/scales and the streaming shape");
  return e == cudaSuccess ? KS_OK : cuda_fail(e, "kernel launch");
}

extern "C" int ks_b200_decode_layer_launches(size_t hidden, size_t inter, size_t group_size) {
  if (hidden == 0 || inter == 0 || hidden % 32 || inter % 32 || group_size < 32 || group_size % 32 ||
      (group_size & (group_size - 1)) || hidden % group_size || inter % group_size)
    return 0;
  int dev;
  if (current_device(&dev) != KS_OK) return 0;
  // 16-byte aligned stand-ins: the dry run checks addresses, never reads them
  const auto *fake = reinterpret_cast<const uint8_t *>(uintptr_t(256));
  DecodeLayerWeights lw{};
  lw.norm1_w = lw.norm2_w = reinterpret_cast<const float *>(fake);
  for (int k = 0; k < 5; ++k) {
    lw.w[k] = fake;
    lw.s[k] = fake;
  }
  DecodeLayersArgs a{};
  a.layers = 1;
  a.lw = &lw;
  a.h_in = reinterpret_cast<const float *>(fake);
  a.hidden = (int64_t)hidden;
  a.inter = (int64_t)inter;
  a.group = (int64_t)group_size;
  const cudaError_t e = launch_decode_layers_persistent(a, nullptr, dev, /*dry=*/true);
  cudaGetLastError();
  return e == cudaSuccess ? 1 : 4;
}
