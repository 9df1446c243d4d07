// ks_noalloc.cu -- a W4A8 GEMV entry point that allocates no memory.
//
// The synchronous entry points of this library get their scratch memory --
// the device copies of host-resident activations and outputs, and the status
// words the kernels write -- from allocations the library makes on first use
// (cudaMalloc, cudaHostAlloc).  Some callers cannot let a library allocate:
// an inference loop that must reserve every byte of device memory up front
// and treat any later allocation as a fault, a process whose device memory is
// handed out by a framework allocator that nothing may bypass, or a host
// thread with real-time deadlines on which an allocation (and the device
// synchronisation cudaFree implies) is not acceptable.
//
// ks_b200_matvec_w4a8_f16_noalloc serves them.  Its scratch is one file-scope
// __device__ array of fixed size, which the CUDA runtime places in device
// memory when the library's module is loaded on a device and which stays
// there until the process exits.  It holds the staged activation vector, a
// staged output (or, for a device-resident output, the caller's rows as they
// were before the call) and the status words.  The weights and scales must
// already be in device memory (they are never staged); the activation vector
// and the output may be host or device memory.  Device-resident activations
// and outputs are used in place.
//
// Host code cannot use the array's name as a device address (on the host it
// names a host-side stand-in), so the address is looked up once per device
// with cudaGetSymbolAddress, with that device current, the first time the
// entry point runs on the device.  That first call should therefore come
// before any stream capture begins.  The address stays cached for the life of
// the process: after a cudaDeviceReset the module is loaded again elsewhere,
// so calls must not follow a reset.
//
// All calls share the one array and it keeps whatever the last call left:
// the status words are cleared at the start of every call.  Two calls whose
// work overlaps on the GPU (from two host threads, say) race on the array and
// must be serialised by the caller.

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "ks_b200.h"
#include "ks_internal.h"

namespace {

// Limits of the no-allocation entry point.
constexpr size_t kNoAllocMaxCols = 16384;   // activation bytes staged
constexpr size_t kNoAllocMaxRows = 131072;  // f32 outputs staged (or kept)
constexpr size_t kNoAllocXOffset = 0;
constexpr size_t kNoAllocYOffset = kNoAllocMaxCols;
constexpr size_t kNoAllocStatusOffset = kNoAllocYOffset + kNoAllocMaxRows * sizeof(float);
constexpr size_t kNoAllocFirstBadOffset = kNoAllocStatusOffset + 64;  // u64: first row with a bad scale
constexpr size_t kNoAllocBytes = kNoAllocStatusOffset + 256;          // 540,928 bytes per device

static __device__ __align__(256) unsigned char ks_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::once_flag g_lookup_once[kMaxDevices];
unsigned char *g_scratch[kMaxDevices];
cudaError_t g_lookup_err[kMaxDevices];

int fail(int code, const std::string &msg) {
  ksb::set_last_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  const std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
  cudaGetLastError();
  return fail(KS_ERR_DEVICE, msg);
}

bool on_device(const void *p, int *dev) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged) return false;
  *dev = at.device;
  return true;
}

// The calling thread's current device, put back when the call returns.
struct KeepCurrentDevice {
  int prev = -1;
  KeepCurrentDevice() {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      cudaGetLastError();
      prev = -1;
    }
  }
  ~KeepCurrentDevice() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int ks_b200_matvec_w4a8_f16_noalloc(const int8_t *input, const uint8_t *packed_weights,
                                               size_t packed_stride_bytes, const uint16_t *weight_scales_f16,
                                               size_t scale_stride, float *output, size_t rows, size_t cols,
                                               size_t group_size, float input_scale, int32_t input_zero_point,
                                               int32_t weight_zero_point) {
  // The argument checks of ks_matvec_w4a8, in the same order.
  if (!input || !packed_weights || !weight_scales_f16 || !output) return fail(KS_ERR_INVALID_ARG, "NULL pointer");
  if (rows == 0 || cols == 0 || group_size == 0)
    return fail(KS_ERR_INVALID_ARG, "rows, cols and group_size must be > 0");
  const size_t row_bytes = cols / 2 + (cols & 1);
  const size_t groups = cols / group_size + (cols % group_size != 0);
  if (packed_stride_bytes < row_bytes || scale_stride < groups)
    return fail(KS_ERR_INVALID_ARG, "stride smaller than one row");
  if (!(input_scale > 0.0f && std::isfinite(input_scale)))
    return fail(KS_ERR_INVALID_ARG, "input_scale must be > 0 and finite");
  if (input_zero_point < -128 || input_zero_point > 127 || weight_zero_point < -8 || weight_zero_point > 7)
    return fail(KS_ERR_INVALID_ARG, "zero point out of range");
  // Valid arguments this entry point cannot serve: larger than its fixed
  // scratch array, or weights it would have to stage.
  if (rows > kNoAllocMaxRows || cols > kNoAllocMaxCols)
    return fail(KS_ERR_UNSUPPORTED,
                "ks_b200_matvec_w4a8_f16_noalloc handles at most 131072 rows and 16384 cols "
                "(its scratch array is fixed); use ks_b200_matvec_w4a8_f16");

  int devcount = 0;
  if (cudaGetDeviceCount(&devcount) != cudaSuccess || devcount == 0) {
    cudaGetLastError();
    return fail(KS_ERR_DEVICE, "no CUDA device available for the B200 kernels");
  }
  int dev = -1, dev_s = -1;
  if (!on_device(packed_weights, &dev) || !on_device(weight_scales_f16, &dev_s))
    return fail(KS_ERR_UNSUPPORTED,
                "ks_b200_matvec_w4a8_f16_noalloc needs weights and scales in device memory "
                "(it stages only the activation vector and the output)");
  int dev_x = -1, dev_y = -1;
  const bool x_on = on_device(input, &dev_x), y_on = on_device(output, &dev_y);
  if (dev != dev_s || (x_on && dev_x != dev) || (y_on && dev_y != dev))
    return fail(KS_ERR_INVALID_ARG, "buffers live on different devices");
  if (dev >= kMaxDevices) return fail(KS_ERR_DEVICE, "device index out of range");
  KeepCurrentDevice keep;
  cudaError_t e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  if (ksb::device_props(dev).cc_major != 10)
    return fail(KS_ERR_DEVICE, "libkernelsmith (B200) needs an sm_100 device");

  // Set-up, once per device with that device current: the array's device
  // address.
  std::call_once(g_lookup_once[dev], [dev] {
    void *p = nullptr;
    g_lookup_err[dev] = cudaGetSymbolAddress(&p, ks_noalloc_scratch);
    g_scratch[dev] = static_cast<unsigned char *>(p);
  });
  if (g_lookup_err[dev] != cudaSuccess) return cuda_fail(g_lookup_err[dev], "cudaGetSymbolAddress(scratch)");
  unsigned char *scratch = g_scratch[dev];
  int8_t *x_stage = reinterpret_cast<int8_t *>(scratch + kNoAllocXOffset);
  float *y_stage = reinterpret_cast<float *>(scratch + kNoAllocYOffset);
  uint32_t *status_dev = reinterpret_cast<uint32_t *>(scratch + kNoAllocStatusOffset);
  auto *first_bad_dev = reinterpret_cast<unsigned long long *>(scratch + kNoAllocFirstBadOffset);
  const size_t ybytes = rows * sizeof(float);

  // The status words must start at zero; the array holds the last call's.
  if ((e = cudaMemsetAsync(status_dev, 0, ksb::kStatusWords * sizeof(uint32_t), 0)) != cudaSuccess)
    return cuda_fail(e, "cudaMemsetAsync(status)");
  if (!x_on && (e = cudaMemcpyAsync(x_stage, input, cols, cudaMemcpyHostToDevice, 0)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(input)");
  // A device-resident output is written in place; its rows as they were go to
  // the array first, so that a bad scale can leave them as the reference
  // does (rows from the first bad one untouched, ks_quantized.c:148-156).
  if (y_on && (e = cudaMemcpyAsync(y_stage, output, ybytes, cudaMemcpyDeviceToDevice, 0)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(output rows)");
  ksb::W4A8Launch a{};
  a.x = x_on ? input : x_stage;
  a.w = packed_weights;
  a.wstride = (int64_t)packed_stride_bytes;
  a.s = weight_scales_f16;
  a.sstride = (int64_t)scale_stride;
  a.stype = ksb::kScaleF16;
  a.y = y_on ? output : y_stage;
  a.rows = (int64_t)rows;
  a.cols = (int64_t)cols;
  a.group = (int64_t)group_size;
  a.sx = input_scale;
  a.zx = input_zero_point;
  a.zw = weight_zero_point;
  a.status = status_dev;
  if ((e = ksb::launch_w4a8(a, 0, dev)) != cudaSuccess) return cuda_fail(e, "kernel launch");
  uint32_t status[ksb::kStatusWords] = {0, 0};
  if ((e = cudaMemcpyAsync(status, status_dev, sizeof status, cudaMemcpyDeviceToHost, 0)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(status)");
  if ((e = cudaStreamSynchronize(0)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  if (status[ksb::kStatusTimeout]) return fail(KS_ERR_DEVICE, "a device-side wait timed out");
  size_t keep_rows = rows;  // rows [0, keep_rows) carry this call's results
  if (status[ksb::kStatusBadScale]) {
    unsigned long long first = ~0ull;
    e = cudaMemsetAsync(first_bad_dev, 0xFF, sizeof first, 0);
    if (e == cudaSuccess)
      e = ksb::launch_w4a8_first_bad_row(weight_scales_f16, ksb::kScaleF16, (int64_t)scale_stride, (int64_t)rows,
                                         (int64_t)groups, first_bad_dev, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&first, first_bad_dev, sizeof first, cudaMemcpyDeviceToHost, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) return cuda_fail(e, "first bad scale row");
    keep_rows = first < rows ? (size_t)first : rows;
  }
  if (y_on && keep_rows < rows) {  // put back the rows from the first bad one on
    e = cudaMemcpyAsync(output + keep_rows, y_stage + keep_rows, (rows - keep_rows) * sizeof(float),
                        cudaMemcpyDeviceToDevice, 0);
  } else if (!y_on && keep_rows > 0) {
    e = cudaMemcpyAsync(output, y_stage, keep_rows * sizeof(float), cudaMemcpyDeviceToHost, 0);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(output)");
  if (status[ksb::kStatusBadScale]) return fail(KS_ERR_INVALID_ARG, "a weight scale is <= 0, inf or nan");
  return KS_OK;
}
