// ks_gemv.cu -- INT8 and W4A8 GEMV kernels for B200 (sm_100a).
//
// Two kernel families per operation:
//
//  * gemv_stream_kernel<Op>: the HBM-streaming path.  One CTA per SM owns a
//    contiguous block of rows.  A producer warp streams the block's weight
//    rows (and their scale rows) into a ring of shared-memory stages with
//    cp.async.bulk (the TMA engine, 1-D bulk form, no tensor map, no
//    multicast), one mbarrier per stage.  Consumer warps take rows
//    round-robin, keep the activation vector in registers, unpack int4 with
//    LOP3, multiply with dp4a and reduce each row with warp shuffles in a
//    fixed order, so results are bitwise reproducible run to run.
//  * *_generic_kernel: a warp-per-row, byte-load path for any stride,
//    alignment, odd column count or group size.  Same contract, slower.
//
// Arithmetic contract (matches the reference C, lib/kernelsmith/ks_quantized.c):
//  * INT8: y[r] = sum_k (x[k]-zx)*(W[r,k]-zw) in int32 with two's-complement
//    wrap, bit-exact (ks_quantized.c:57-61).  The zero points are applied as
//    sum(xw) - zw*sum(x) - zx*sum(w) + n*zx*zw, exact mod 2^32.
//  * W4A8: per 32-element chunk an exact int32 dot of (x-zx)(w-zw); the f32
//    result is sx * sum_chunks f32(acc_chunk) * scale[group].  The reference
//    sums per element in f32 (ks_quantized.c:116-123); the two orders agree
//    to within 1e-4 of max(|y|, rms(y)).
//
// Signed int4 nibbles (bits 0..3 = even k, bits 4..7 = odd k) are consumed as
// u = w + 8 in [0, 15]: (v & 0x0F0F0F0F) ^ 0x08080808 gives the even k as
// unsigned bytes, (v & 0xF0F0F0F0) ^ 0x80808080 gives 16*u for odd k.  With
// dp4a.u32.s32 against the matching even/odd activation bytes,
// sum(w*x) = sum(u*x) - 8*sum(x), exactly.

#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "ks_internal.h"
#include "ks_ptx.cuh"

namespace ksb {

constexpr int kConsumerWarps = 16;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;

// Geometry of the streamed weight block, shared by all stream kernels.
struct StreamGeom {
  const uint8_t *w;     // first weight row
  int64_t wstride;      // bytes between weight rows
  const uint8_t *s;     // first side row (scales) or null
  int64_t sstride;      // bytes between side rows
  int64_t rows;
  int32_t n_cta;
  int32_t rps;          // rows per stage
  int32_t nst;          // stages in the ring
  int32_t row_bytes;    // streamed bytes per weight row
  int32_t srow_bytes;   // streamed bytes per side row (0: none)
  int32_t stage_bytes;
  int32_t w_contig;     // wstride == row_bytes: one copy per stage
  int32_t s_contig;
  uint32_t *status;
};

__host__ __device__ constexpr int bar_area_bytes(int nst) { return ((nst * 16 + 127) / 128) * 128; }

__device__ __forceinline__ void set_status(uint32_t *status, int word) {
  if (status) *reinterpret_cast<volatile uint32_t *>(status + word) = 1u;
}

template <typename T>
__device__ __forceinline__ float scale_to_f32(T v);
template <>
__device__ __forceinline__ float scale_to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float scale_to_f32<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ bool scale_ok(float v) { return v > 0.0f && v < __int_as_float(0x7f800000); }

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Load 32 activation bytes starting at p (16-byte aligned if al16).
__device__ __forceinline__ void load_x32(const int8_t *p, bool al16, uint32_t (&X)[8]) {
  if (al16) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint4 b = __ldg(reinterpret_cast<const uint4 *>(p) + 1);
    X[0] = a.x; X[1] = a.y; X[2] = a.z; X[3] = a.w;
    X[4] = b.x; X[5] = b.y; X[6] = b.z; X[7] = b.w;
  } else {
    const uint8_t *q = reinterpret_cast<const uint8_t *>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      X[i] = (uint32_t)q[4 * i] | ((uint32_t)q[4 * i + 1] << 8) | ((uint32_t)q[4 * i + 2] << 16) |
             ((uint32_t)q[4 * i + 3] << 24);
  }
}

__device__ __forceinline__ void load_x16(const int8_t *p, bool al16, uint32_t (&X)[4]) {
  if (al16) {
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p));
    X[0] = a.x; X[1] = a.y; X[2] = a.z; X[3] = a.w;
  } else {
    const uint8_t *q = reinterpret_cast<const uint8_t *>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      X[i] = (uint32_t)q[4 * i] | ((uint32_t)q[4 * i + 1] << 8) | ((uint32_t)q[4 * i + 2] << 16) |
             ((uint32_t)q[4 * i + 3] << 24);
  }
}

// ---------------------------------------------------------------- W4A8 op --
struct W4A8OpParams {
  const int8_t *x;
  float *y;
  int32_t chunks;  // 32-element chunks per row (cols / 32)
  int32_t gshift;  // log2(group / 32)
  float sx;
  int32_t zx, zw;
  int32_t x_al16;
};

template <typename ST, int NCPL>
struct W4A8Op {
  using Params = W4A8OpParams;
  struct Lane {
    uint32_t xe[NCPL][4];  // activation bytes at even k of each packed word
    uint32_t xo[NCPL][4];  // ... at odd k
    int kc[NCPL];          // (8 + zw) * sum(x - zx) over the chunk
  };

  __device__ __forceinline__ static void init(const Params &p, Lane &L, int lane) {
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      uint32_t X[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (c < p.chunks) load_x32(p.x + 32 * c, p.x_al16 != 0, X);
      int sumx = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        L.xe[j][q] = prmt(X[2 * q], X[2 * q + 1], 0x6420);
        L.xo[j][q] = prmt(X[2 * q], X[2 * q + 1], 0x7531);
        sumx = dp4a_ss(X[2 * q], 0x01010101u, sumx);
        sumx = dp4a_ss(X[2 * q + 1], 0x01010101u, sumx);
      }
      L.kc[j] = (8 + p.zw) * (sumx - 32 * p.zx);
    }
  }

  // One weight row (in shared memory) -> y[row].  Returns true if a scale of
  // this row is invalid.
  __device__ __forceinline__ static bool row(const Params &p, const Lane &L, const uint8_t *wrow,
                                             const uint8_t *srow, int64_t grow, int lane) {
    const ST *sc = reinterpret_cast<const ST *>(srow);
    float part = 0.0f;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) {
        const uint4 v = lds128(wrow + 16 * c);
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
        int lo = 0, hi = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          lo = dp4a_us(and_xor(vw[q], 0x0F0F0F0Fu, 0x08080808u), L.xe[j][q], lo);
          hi = dp4a_us(and_xor(vw[q], 0xF0F0F0F0u, 0x80808080u), L.xo[j][q], hi);
        }
        int acc = lo + (hi >> 4) - L.kc[j];
        if (p.zx != 0) {
          uint32_t su = 0, sh = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            su = dp4a_uu(and_xor(vw[q], 0x0F0F0F0Fu, 0x08080808u), 0x01010101u, su);
            sh = dp4a_uu(and_xor(vw[q], 0xF0F0F0F0u, 0x80808080u), 0x01010101u, sh);
          }
          acc -= p.zx * (int)(su + (sh >> 4));
        }
        const float s = scale_to_f32(sc[c >> p.gshift]);
        bad |= !scale_ok(s);
        part = fmaf((float)acc, s, part);
      }
    }
    part = warp_sum_f32(part);
    if (lane == 0) p.y[grow] = part * p.sx;
    return bad;
  }
};

// ---------------------------------------------------------------- INT8 op --
struct I8OpParams {
  const int8_t *x;
  void *y;
  const float *ws;
  float sa;
  int32_t chunks;  // 16-element chunks per row (cols / 16)
  int32_t zx, zw;
  int32_t x_al16;
};

template <int NCPL, bool OUT_F32>
struct I8Op {
  using Params = I8OpParams;
  struct Lane {
    uint32_t xr[NCPL][4];
    int kl;  // sum over this lane's chunks of zw*sum(x) - 16*zx*zw
  };

  __device__ __forceinline__ static void init(const Params &p, Lane &L, int lane) {
    uint32_t kl = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      uint32_t X[4] = {0, 0, 0, 0};
      if (c < p.chunks) {
        load_x16(p.x + 16 * c, p.x_al16 != 0, X);
        int sumx = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) sumx = dp4a_ss(X[q], 0x01010101u, sumx);
        kl += (uint32_t)p.zw * (uint32_t)sumx - 16u * (uint32_t)p.zx * (uint32_t)p.zw;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) L.xr[j][q] = X[q];
    }
    L.kl = (int)kl;
  }

  __device__ __forceinline__ static bool row(const Params &p, const Lane &L, const uint8_t *wrow,
                                             const uint8_t * /*srow*/, int64_t grow, int lane) {
    int acc = 0, sw = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) {
        const uint4 v = lds128(wrow + 16 * c);
        acc = dp4a_ss(v.x, L.xr[j][0], acc);
        acc = dp4a_ss(v.y, L.xr[j][1], acc);
        acc = dp4a_ss(v.z, L.xr[j][2], acc);
        acc = dp4a_ss(v.w, L.xr[j][3], acc);
        if (p.zx != 0) {
          sw = dp4a_ss(v.x, 0x01010101u, sw);
          sw = dp4a_ss(v.y, 0x01010101u, sw);
          sw = dp4a_ss(v.z, 0x01010101u, sw);
          sw = dp4a_ss(v.w, 0x01010101u, sw);
        }
      }
    }
    uint32_t t = (uint32_t)acc - (uint32_t)p.zx * (uint32_t)sw - (uint32_t)L.kl;
    const int total = warp_sum_i32((int)t);
    if (lane == 0) {
      if (OUT_F32) {
        const float d = __fmul_rn((float)total, __ldg(p.ws + grow));
        reinterpret_cast<float *>(p.y)[grow] = __fmul_rn(d, p.sa);
      } else {
        reinterpret_cast<int32_t *>(p.y)[grow] = total;
      }
    }
    return false;
  }
};

// ------------------------------------------------------ streaming skeleton --
template <class Op>
__global__ void __launch_bounds__(kStreamThreads, 1)
    gemv_stream_kernel(const StreamGeom g, const typename Op::Params op) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + g.nst;
  uint8_t *stages = smem + bar_area_bytes(g.nst);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)blockIdx.x * g.rows / g.n_cta;
  const int64_t r1 = (int64_t)(blockIdx.x + 1) * g.rows / g.n_cta;
  const int rows_cta = (int)(r1 - r0);
  const int nstages = (rows_cta + g.rps - 1) / g.rps;

  if (threadIdx.x == 0) {
    for (int b = 0; b < g.nst; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], kConsumerWarps);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer: one thread issues every bulk copy ----------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int st = 0; st < nstages; ++st) {
        const int b = st % g.nst;
        if (st >= g.nst && !mbar_wait(&empty[b], (uint32_t)((st / g.nst) - 1) & 1u)) {
          set_status(g.status, kStatusTimeout);
          break;
        }
        const int lo = st * g.rps;
        const int n = min(g.rps, rows_cta - lo);
        const uint32_t wbytes = (uint32_t)n * (uint32_t)g.row_bytes;
        const uint32_t sbytes = (uint32_t)n * (uint32_t)g.srow_bytes;
        uint8_t *dst = stages + (size_t)b * g.stage_bytes;
        mbar_arrive_expect_tx(&full[b], wbytes + sbytes);
        const uint8_t *wsrc = g.w + (r0 + lo) * g.wstride;
        if (g.w_contig) {
          bulk_g2s_hint(dst, wsrc, wbytes, &full[b], pol);
        } else {
          for (int r = 0; r < n; ++r)
            bulk_g2s_hint(dst + (size_t)r * g.row_bytes, wsrc + (int64_t)r * g.wstride, g.row_bytes,
                          &full[b], pol);
        }
        if (g.srow_bytes) {
          uint8_t *sdst = dst + (size_t)g.rps * g.row_bytes;
          const uint8_t *ssrc = g.s + (r0 + lo) * g.sstride;
          if (g.s_contig) {
            bulk_g2s(sdst, ssrc, sbytes, &full[b]);
          } else {
            for (int r = 0; r < n; ++r)
              bulk_g2s(sdst + (size_t)r * g.srow_bytes, ssrc + (int64_t)r * g.sstride, g.srow_bytes,
                       &full[b]);
          }
        }
        ++issued;
      }
      // Before the CTA may exit, every copy it issued must have landed.
      for (int st = max(0, issued - g.nst); st < issued; ++st) {
        if (!mbar_wait(&full[st % g.nst], (uint32_t)(st / g.nst) & 1u)) {
          set_status(g.status, kStatusTimeout);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  typename Op::Lane L;
  Op::init(op, L, lane);  // overlaps the first copies' latency
  bool bad = false;
  for (int st = 0; st < nstages; ++st) {
    const int b = st % g.nst;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[b], (uint32_t)(st / g.nst) & 1u));
    if (!ok) {
      if (lane == 0) set_status(g.status, kStatusTimeout);
      break;
    }
    const int lo = st * g.rps;
    const int hi = min(lo + g.rps, rows_cta);
    const uint8_t *base = stages + (size_t)b * g.stage_bytes;
    const uint8_t *sbase = base + (size_t)g.rps * g.row_bytes;
    int i = lo + ((warp - lo % kConsumerWarps) + kConsumerWarps) % kConsumerWarps;
    for (; i < hi; i += kConsumerWarps) {
      bad |= Op::row(op, L, base + (size_t)(i - lo) * g.row_bytes,
                     sbase + (size_t)(i - lo) * g.srow_bytes, r0 + i, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[b]);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) set_status(g.status, kStatusBadScale);
}

// ------------------------------------------------------- generic kernels --
template <typename ST>
__global__ void __launch_bounds__(256)
    w4a8_generic_kernel(const int8_t *__restrict__ x, const uint8_t *__restrict__ w, int64_t wstride,
                        const ST *__restrict__ s, int64_t sstride, float *__restrict__ y,
                        int64_t rows, int64_t cols, int64_t group, float sx, int zx, int zw,
                        uint32_t *status) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  bool bad = false;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const uint8_t *wr = w + r * wstride;
    const ST *sr = s + r * sstride;
    float acc = 0.0f;
    for (int64_t k = lane; k < cols; k += 32) {
      const uint32_t byte = wr[k >> 1];
      const int nib = (int)((k & 1) ? (byte >> 4) : (byte & 15u));
      const int wv = ((nib ^ 8) - 8) - zw;
      const int xv = (int)x[k] - zx;
      const float sc = scale_to_f32(sr[k / group]);
      bad |= !scale_ok(sc);
      acc = fmaf((float)(xv * wv), sc, acc);
    }
    acc = warp_sum_f32(acc);
    if (lane == 0) y[r] = acc * sx;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) set_status(status, kStatusBadScale);
}

template <bool OUT_F32>
__global__ void __launch_bounds__(256)
    i8_generic_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w, int64_t wstride,
                      void *__restrict__ y, int64_t rows, int64_t cols, int zx, int zw,
                      const float *__restrict__ ws, float sa) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const int8_t *wr = w + r * wstride;
    uint32_t acc = 0;
    for (int64_t k = lane; k < cols; k += 32)
      acc += (uint32_t)(((int)x[k] - zx) * ((int)wr[k] - zw));
    const int total = warp_sum_i32((int)acc);
    if (lane == 0) {
      if (OUT_F32) {
        const float d = __fmul_rn((float)total, ws[r]);
        reinterpret_cast<float *>(y)[r] = __fmul_rn(d, sa);
      } else {
        reinterpret_cast<int32_t *>(y)[r] = total;
      }
    }
  }
}

// ------------------------------------------------------------ host side --
namespace {

std::once_flag g_props_once[64];
DeviceProps g_props[64];

int env_int(const char *name, int dflt) {
  const char *v = std::getenv(name);
  return v && *v ? std::atoi(v) : dflt;
}

// Tunables, read once per process: target stage size and the shared-memory
// budget of the ring.
int stage_target_bytes() {
  static const int v = env_int("KS_B200_STAGE_BYTES", 32 * 1024);
  return v;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ilog2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return s;
}

// Fill the ring geometry; false if the rows are too long to stage.
bool plan_stream(StreamGeom &g, int64_t rows, int row_bytes, int srow_bytes, int sm_count,
                 int smem_optin) {
  const int row_total = row_bytes + srow_bytes;
  int rps = std::max(1, stage_target_bytes() / row_total);
  rps = std::min(rps, 2 * kConsumerWarps);
  const int64_t n_cta = std::min<int64_t>(rows, sm_count);
  const int64_t rows_cta_max = (rows + n_cta - 1) / n_cta;
  rps = (int)std::min<int64_t>(rps, rows_cta_max);
  const int stage_bytes = ((rps * row_total + 127) / 128) * 128;
  const int budget = smem_optin - 1024;
  int nst = budget / stage_bytes;
  const int64_t need = (rows_cta_max + rps - 1) / rps;
  nst = (int)std::min<int64_t>(nst, need);
  if (nst < 1 || (nst < 2 && need > 1)) return false;
  g.rows = rows;
  g.n_cta = (int32_t)n_cta;
  g.rps = rps;
  g.nst = nst;
  g.row_bytes = row_bytes;
  g.srow_bytes = srow_bytes;
  g.stage_bytes = stage_bytes;
  return true;
}

size_t stream_smem_bytes(const StreamGeom &g) {
  return (size_t)bar_area_bytes(g.nst) + (size_t)g.nst * g.stage_bytes;
}

template <class Op>
cudaError_t launch_stream(const StreamGeom &g, const typename Op::Params &op, cudaStream_t stream) {
  const size_t smem = stream_smem_bytes(g);
  static std::once_flag attr_once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(attr_once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(gemv_stream_kernel<Op>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              device_props(dev).smem_optin);
  });
  if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
  gemv_stream_kernel<Op><<<g.n_cta, kStreamThreads, smem, stream>>>(g, op);
  return cudaGetLastError();
}

struct W4A8Plan {
  bool fast = false;
  StreamGeom g{};
  W4A8OpParams op{};
  int ncpl = 0;
};

W4A8Plan plan_w4a8(const W4A8Launch &a, int device) {
  W4A8Plan P;
  const int ssize = a.stype == kScaleF16 ? 2 : 4;
  const int64_t groups = (a.cols + a.group - 1) / a.group;
  const int gshift = ilog2_exact(a.group / 32);
  const bool shape_ok = a.cols % 32 == 0 && a.group % 32 == 0 && gshift >= 0 &&
                        a.cols <= 8192 && a.wstride % 16 == 0 && aligned16(a.w) &&
                        (groups * ssize) % 16 == 0 && (a.sstride * ssize) % 16 == 0 &&
                        aligned16(a.s) && a.rows < (int64_t(1) << 31);
  if (!shape_ok) return P;
  const DeviceProps &dp = device_props(device);
  const int row_bytes = (int)(a.cols / 2);
  const int srow_bytes = (int)(groups * ssize);
  StreamGeom g{};
  if (!plan_stream(g, a.rows, row_bytes, srow_bytes, dp.sm_count, dp.smem_optin)) return P;
  g.w = a.w;
  g.wstride = a.wstride;
  g.s = reinterpret_cast<const uint8_t *>(a.s);
  g.sstride = a.sstride * ssize;
  g.w_contig = a.wstride == row_bytes;
  g.s_contig = g.sstride == srow_bytes;
  g.status = a.status;
  P.g = g;
  P.op.x = a.x;
  P.op.y = a.y;
  P.op.chunks = (int32_t)(a.cols / 32);
  P.op.gshift = gshift;
  P.op.sx = a.sx;
  P.op.zx = a.zx;
  P.op.zw = a.zw;
  P.op.x_al16 = aligned16(a.x);
  const int c = P.op.chunks;
  P.ncpl = c <= 32 ? 1 : c <= 64 ? 2 : c <= 128 ? 4 : 8;
  P.fast = true;
  return P;
}

template <typename ST>
cudaError_t launch_w4a8_fast(const W4A8Plan &P, cudaStream_t stream) {
  switch (P.ncpl) {
    case 1: return launch_stream<W4A8Op<ST, 1>>(P.g, P.op, stream);
    case 2: return launch_stream<W4A8Op<ST, 2>>(P.g, P.op, stream);
    case 4: return launch_stream<W4A8Op<ST, 4>>(P.g, P.op, stream);
    default: return launch_stream<W4A8Op<ST, 8>>(P.g, P.op, stream);
  }
}

struct I8Plan {
  bool fast = false;
  StreamGeom g{};
  I8OpParams op{};
  int ncpl = 0;
};

I8Plan plan_i8(const I8Launch &a, int device) {
  I8Plan P;
  const bool shape_ok = a.cols % 16 == 0 && a.cols <= 4096 && a.wstride % 16 == 0 &&
                        aligned16(a.w) && a.rows < (int64_t(1) << 31);
  if (!shape_ok) return P;
  const DeviceProps &dp = device_props(device);
  StreamGeom g{};
  if (!plan_stream(g, a.rows, (int)a.cols, 0, dp.sm_count, dp.smem_optin)) return P;
  g.w = reinterpret_cast<const uint8_t *>(a.w);
  g.wstride = a.wstride;
  g.s = nullptr;
  g.sstride = 0;
  g.w_contig = a.wstride == a.cols;
  g.s_contig = 1;
  g.status = a.status;
  P.g = g;
  P.op.x = a.x;
  P.op.y = a.y;
  P.op.ws = a.ws;
  P.op.sa = a.sa;
  P.op.chunks = (int32_t)(a.cols / 16);
  P.op.zx = a.zx;
  P.op.zw = a.zw;
  P.op.x_al16 = aligned16(a.x);
  const int c = P.op.chunks;
  P.ncpl = c <= 32 ? 1 : c <= 64 ? 2 : c <= 128 ? 4 : 8;
  P.fast = true;
  return P;
}

template <bool F32>
cudaError_t launch_i8_fast(const I8Plan &P, cudaStream_t stream) {
  switch (P.ncpl) {
    case 1: return launch_stream<I8Op<1, F32>>(P.g, P.op, stream);
    case 2: return launch_stream<I8Op<2, F32>>(P.g, P.op, stream);
    case 4: return launch_stream<I8Op<4, F32>>(P.g, P.op, stream);
    default: return launch_stream<I8Op<8, F32>>(P.g, P.op, stream);
  }
}

int generic_grid(int64_t rows, int sm_count) {
  const int64_t blocks = (rows + 7) / 8;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sm_count * 8));
}

}  // namespace

const DeviceProps &device_props(int device) {
  const int d = device & 63;
  std::call_once(g_props_once[d], [d] {
    DeviceProps p;
    cudaDeviceGetAttribute(&p.sm_count, cudaDevAttrMultiProcessorCount, d);
    cudaDeviceGetAttribute(&p.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d);
    cudaDeviceGetAttribute(&p.cc_major, cudaDevAttrComputeCapabilityMajor, d);
    cudaDeviceGetAttribute(&p.cc_minor, cudaDevAttrComputeCapabilityMinor, d);
    g_props[d] = p;
  });
  return g_props[d];
}

int w4a8_path(const W4A8Launch &a) {
  int dev = 0;
  cudaGetDevice(&dev);
  return plan_w4a8(a, dev).fast ? 1 : 0;
}

int i8_path(const I8Launch &a) {
  int dev = 0;
  cudaGetDevice(&dev);
  return plan_i8(a, dev).fast ? 1 : 0;
}

cudaError_t launch_w4a8(const W4A8Launch &a, cudaStream_t stream, int device) {
  const W4A8Plan P = plan_w4a8(a, device);
  if (P.fast) {
    return a.stype == kScaleF16 ? launch_w4a8_fast<__half>(P, stream)
                                : launch_w4a8_fast<float>(P, stream);
  }
  const int grid = generic_grid(a.rows, device_props(device).sm_count);
  if (a.stype == kScaleF16) {
    w4a8_generic_kernel<__half><<<grid, 256, 0, stream>>>(
        a.x, a.w, a.wstride, reinterpret_cast<const __half *>(a.s), a.sstride, a.y, a.rows, a.cols,
        a.group, a.sx, a.zx, a.zw, a.status);
  } else {
    w4a8_generic_kernel<float><<<grid, 256, 0, stream>>>(
        a.x, a.w, a.wstride, reinterpret_cast<const float *>(a.s), a.sstride, a.y, a.rows, a.cols,
        a.group, a.sx, a.zx, a.zw, a.status);
  }
  return cudaGetLastError();
}

cudaError_t launch_i8(const I8Launch &a, cudaStream_t stream, int device) {
  const I8Plan P = plan_i8(a, device);
  if (P.fast) return a.out_f32 ? launch_i8_fast<true>(P, stream) : launch_i8_fast<false>(P, stream);
  const int grid = generic_grid(a.rows, device_props(device).sm_count);
  if (a.out_f32) {
    i8_generic_kernel<true><<<grid, 256, 0, stream>>>(a.x, a.w, a.wstride, a.y, a.rows, a.cols,
                                                      a.zx, a.zw, a.ws, a.sa);
  } else {
    i8_generic_kernel<false><<<grid, 256, 0, stream>>>(a.x, a.w, a.wstride, a.y, a.rows, a.cols,
                                                       a.zx, a.zw, a.ws, a.sa);
  }
  return cudaGetLastError();
}

}  // namespace ksb
