// ks_gemv.cu -- INT8 and W4A8 GEMV kernels for B200 (sm_100a).
//
// Two kernel families per operation:
//
//  * gemv_stream_kernel<Op>: the HBM-streaming path.  One CTA per SM owns a
//    contiguous block of rows.  A producer warp streams the block's weight
//    rows (and their scale rows) into a ring of shared-memory stages with
//    cp.async.bulk (the TMA engine, 1-D bulk form, no tensor map, no
//    multicast), one mbarrier per stage.  Eight consumer warps take pairs of
//    rows, unpack int4 with LOP3, multiply with dp4a and reduce each row with
//    warp shuffles in a fixed order, so results are bitwise reproducible.
//    A CTA uses at most ~108 KB of shared memory and 288 threads, so two CTAs
//    fit on an SM: with programmatic dependent launch the next GEMV on the
//    stream starts streaming its weights while the current one finishes, and
//    only waits for the previous kernel (griddepcontrol.wait) before it reads
//    the activation vector or writes its output.
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
//
// Weights and scales are read before griddepcontrol.wait.  Only the kernels of
// this library trigger an early launch, and none of them writes weights or
// scales, so the weights a GEMV reads early are never being written.

#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "ks_internal.h"
#include "ks_ptx.cuh"

namespace ksb {

constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxStages = 16;
constexpr int kBarBytes = 1024;  // barrier area at the start of shared memory
// Shared memory per CTA: two CTAs must fit in the SM's 228 KB (1 KB of each
// CTA is reserved by the hardware).
constexpr int kSmemPerCta = 108 * 1024;

// Geometry of the streamed weight block, shared by all stream kernels.
struct StreamGeom {
  const uint8_t *w;     // first weight row
  int64_t wstride;      // bytes between weight rows
  const uint8_t *s;     // first side row (scales) or null
  int64_t sstride;      // bytes between side rows
  int64_t rows;
  int32_t n_cta;
  int32_t rps;          // rows per stage (even)
  int32_t nst;          // stages in the ring
  int32_t row_bytes;    // streamed bytes per weight row
  int32_t srow_bytes;   // streamed bytes per side row (0: none)
  int32_t stage_bytes;
  int32_t x_bytes;      // shared-memory activation area (0: activations in registers)
  int32_t w_contig;     // wstride == row_bytes: one copy per stage
  int32_t s_contig;
  uint32_t *status;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t lds_u16(const void *p) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
  return v;
}

// Scale element traits: raw-bit load, validity (> 0 and finite) and widening.
template <typename ST>
struct ScaleBits;
template <>
struct ScaleBits<float> {
  static constexpr int kBytes = 4;
  __device__ __forceinline__ static uint32_t load(const uint8_t *p) { return lds_u32(p); }
  __device__ __forceinline__ static uint32_t gload(const float *p) { return __float_as_uint(__ldg(p)); }
  // 0 < bits < +inf; negative values, zero, inf and nan fail
  __device__ __forceinline__ static bool bad(uint32_t b) { return (b - 1u) >= 0x7F7FFFFFu; }
  __device__ __forceinline__ static float f32(uint32_t b) { return __uint_as_float(b); }
};
template <>
struct ScaleBits<__half> {
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static uint32_t load(const uint8_t *p) { return lds_u16(p); }
  __device__ __forceinline__ static uint32_t gload(const __half *p) {
    return __half_as_ushort(__ldg(p));
  }
  __device__ __forceinline__ static bool bad(uint32_t b) { return (b - 1u) >= 0x7BFFu; }
  __device__ __forceinline__ static float f32(uint32_t b) {
    return __half2float(__ushort_as_half((unsigned short)b));
  }
};

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load_bytes(const int8_t *p, bool al16, uint32_t *X, int words) {
  if (al16) {
    for (int i = 0; i < words; i += 4) {
      const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p) + i / 4);
      X[i] = a.x; X[i + 1] = a.y; X[i + 2] = a.z; X[i + 3] = a.w;
    }
  } else {
    const uint8_t *q = reinterpret_cast<const uint8_t *>(p);
    for (int i = 0; i < words; ++i)
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

// Per chunk of 32 activations: the even-k and odd-k bytes of each packed
// word, and kc = (8 + zw) * sum(x - zx) over the chunk.
__device__ __forceinline__ void w4a8_prep_chunk(const W4A8OpParams &p, int c, uint32_t (&xe)[4],
                                                uint32_t (&xo)[4], int &kc) {
  uint32_t X[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c < p.chunks) load_bytes(p.x + 32 * c, p.x_al16 != 0, X, 8);
  int sumx = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    xe[q] = prmt(X[2 * q], X[2 * q + 1], 0x6420);
    xo[q] = prmt(X[2 * q], X[2 * q + 1], 0x7531);
    sumx = dp4a_ss(X[2 * q], 0x01010101u, sumx);
    sumx = dp4a_ss(X[2 * q + 1], 0x01010101u, sumx);
  }
  kc = (8 + p.zw) * (sumx - 32 * p.zx);
}

// int32 dot of one 32-element chunk (packed word v) against prepared x.
__device__ __forceinline__ int w4a8_chunk_dot(const uint4 v, const uint32_t (&xe)[4], const uint32_t (&xo)[4],
                                              int kc, int zx) {
  const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
  int lo = 0, hi = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    lo = dp4a_us(and_xor(vw[q], 0x0F0F0F0Fu, 0x08080808u), xe[q], lo);
    hi = dp4a_us(and_xor(vw[q], 0xF0F0F0F0u, 0x80808080u), xo[q], hi);
  }
  int acc = lo + (hi >> 4) - kc;
  if (zx != 0) {
    uint32_t su = 0, sh = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      su = dp4a_uu(and_xor(vw[q], 0x0F0F0F0Fu, 0x08080808u), 0x01010101u, su);
      sh = dp4a_uu(and_xor(vw[q], 0xF0F0F0F0u, 0x80808080u), 0x01010101u, sh);
    }
    acc -= zx * (int)(su + (sh >> 4));
  }
  return acc;
}

// XS: activations staged in shared memory (long rows) instead of registers.
template <typename ST, int NCPL, bool XS>
struct W4A8Op {
  using Params = W4A8OpParams;
  using SB = ScaleBits<ST>;
  struct Lane {
    uint32_t xe[XS ? 1 : NCPL][4];
    uint32_t xo[XS ? 1 : NCPL][4];
    int kc[XS ? 1 : NCPL];
  };

  // Called by every consumer thread after griddepcontrol.wait.
  __device__ __forceinline__ static void init(const Params &p, Lane &L, int lane, uint8_t *xs, int ctid) {
    if (XS) {
      for (int c = ctid; c < p.chunks; c += kConsumerWarps * 32) {
        uint32_t xe[4], xo[4];
        int kc;
        w4a8_prep_chunk(p, c, xe, xo, kc);
        uint4 *d = reinterpret_cast<uint4 *>(xs + 32 * c);
        d[0] = make_uint4(xe[0], xe[1], xe[2], xe[3]);
        d[1] = make_uint4(xo[0], xo[1], xo[2], xo[3]);
        reinterpret_cast<int *>(xs + 32 * p.chunks)[c] = kc;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    } else {
#pragma unroll
      for (int j = 0; j < NCPL; ++j) w4a8_prep_chunk(p, lane + 32 * j, L.xe[j], L.xo[j], L.kc[j]);
    }
  }

  // Two rows (b valid if has_b) whose weights and scale rows are in shared
  // memory -> y.  Returns true if a scale of a processed row is invalid.
  __device__ __forceinline__ static bool rows2(const Params &p, const Lane &L, const uint8_t *xs,
                                               const uint8_t *wa, const uint8_t *sa, const uint8_t *wb,
                                               const uint8_t *sb, int64_t ga, bool has_b, int lane) {
    float pa = 0.0f, pb = 0.0f;
    uint32_t bad = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) {
        uint32_t xe[4], xo[4];
        int kc;
        if (XS) {
          const uint4 e = lds128(xs + 32 * c), o = lds128(xs + 32 * c + 16);
          xe[0] = e.x; xe[1] = e.y; xe[2] = e.z; xe[3] = e.w;
          xo[0] = o.x; xo[1] = o.y; xo[2] = o.z; xo[3] = o.w;
          kc = (int)lds_u32(xs + 32 * p.chunks + 4 * c);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            xe[q] = L.xe[XS ? 0 : j][q];
            xo[q] = L.xo[XS ? 0 : j][q];
          }
          kc = L.kc[XS ? 0 : j];
        }
        const int g = c >> p.gshift;
        const uint4 va = lds128(wa + 16 * c);
        const uint4 vb = lds128(wb + 16 * c);
        const uint32_t ba = SB::load(sa + g * SB::kBytes);
        const uint32_t bb = SB::load(sb + g * SB::kBytes);
        const int acc_a = w4a8_chunk_dot(va, xe, xo, kc, p.zx);
        const int acc_b = w4a8_chunk_dot(vb, xe, xo, kc, p.zx);
        bad |= (uint32_t)SB::bad(ba) | ((uint32_t)SB::bad(bb) & (uint32_t)has_b);
        pa = fmaf((float)acc_a, SB::f32(ba), pa);
        pb = fmaf((float)acc_b, SB::f32(bb), pb);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pa += __shfl_xor_sync(0xffffffffu, pa, o);
      pb += __shfl_xor_sync(0xffffffffu, pb, o);
    }
    if (lane == 0) p.y[ga] = pa * p.sx;
    if (lane == 1 && has_b) p.y[ga + 1] = pb * p.sx;
    return bad != 0;
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

template <int NCPL, bool OUT_F32, bool XS>
struct I8Op {
  using Params = I8OpParams;
  struct Lane {
    uint32_t xr[XS ? 1 : NCPL][4];
    int kl;  // sum over this lane's chunks of zw*sum(x) - 16*zx*zw
  };

  __device__ __forceinline__ static void init(const Params &p, Lane &L, int lane, uint8_t *xs, int ctid) {
    if (XS) {
      for (int c = ctid; c < p.chunks; c += kConsumerWarps * 32) {
        uint32_t X[4];
        load_bytes(p.x + 16 * c, p.x_al16 != 0, X, 4);
        reinterpret_cast<uint4 *>(xs)[c] = make_uint4(X[0], X[1], X[2], X[3]);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    }
    uint32_t kl = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      uint32_t X[4] = {0, 0, 0, 0};
      if (c < p.chunks) {
        if (XS) {
          const uint4 v = lds128(xs + 16 * c);
          X[0] = v.x; X[1] = v.y; X[2] = v.z; X[3] = v.w;
        } else {
          load_bytes(p.x + 16 * c, p.x_al16 != 0, X, 4);
        }
        int sumx = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) sumx = dp4a_ss(X[q], 0x01010101u, sumx);
        kl += (uint32_t)p.zw * (uint32_t)sumx - 16u * (uint32_t)p.zx * (uint32_t)p.zw;
      }
      if (!XS) {
#pragma unroll
        for (int q = 0; q < 4; ++q) L.xr[XS ? 0 : j][q] = X[q];
      }
    }
    L.kl = (int)kl;
  }

  __device__ __forceinline__ static bool rows2(const Params &p, const Lane &L, const uint8_t *xs,
                                               const uint8_t *wa, const uint8_t *, const uint8_t *wb,
                                               const uint8_t *, int64_t ga, bool has_b, int lane) {
    float wsa = 0.0f, wsb = 0.0f;
    if (OUT_F32) {  // issue the per-channel scale loads early
      if (lane == 0) wsa = __ldg(p.ws + ga);
      if (lane == 1 && has_b) wsb = __ldg(p.ws + ga + 1);
    }
    int acc_a = 0, acc_b = 0, sw_a = 0, sw_b = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) {
        uint32_t xr[4];
        if (XS) {
          const uint4 v = lds128(xs + 16 * c);
          xr[0] = v.x; xr[1] = v.y; xr[2] = v.z; xr[3] = v.w;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) xr[q] = L.xr[XS ? 0 : j][q];
        }
        const uint4 va = lds128(wa + 16 * c);
        const uint4 vb = lds128(wb + 16 * c);
        acc_a = dp4a_ss(va.x, xr[0], acc_a);
        acc_b = dp4a_ss(vb.x, xr[0], acc_b);
        acc_a = dp4a_ss(va.y, xr[1], acc_a);
        acc_b = dp4a_ss(vb.y, xr[1], acc_b);
        acc_a = dp4a_ss(va.z, xr[2], acc_a);
        acc_b = dp4a_ss(vb.z, xr[2], acc_b);
        acc_a = dp4a_ss(va.w, xr[3], acc_a);
        acc_b = dp4a_ss(vb.w, xr[3], acc_b);
        if (p.zx != 0) {
          sw_a = dp4a_ss(va.x, 0x01010101u, sw_a);
          sw_a = dp4a_ss(va.y, 0x01010101u, sw_a);
          sw_a = dp4a_ss(va.z, 0x01010101u, sw_a);
          sw_a = dp4a_ss(va.w, 0x01010101u, sw_a);
          sw_b = dp4a_ss(vb.x, 0x01010101u, sw_b);
          sw_b = dp4a_ss(vb.y, 0x01010101u, sw_b);
          sw_b = dp4a_ss(vb.z, 0x01010101u, sw_b);
          sw_b = dp4a_ss(vb.w, 0x01010101u, sw_b);
        }
      }
    }
    uint32_t ta = (uint32_t)acc_a - (uint32_t)p.zx * (uint32_t)sw_a - (uint32_t)L.kl;
    uint32_t tb = (uint32_t)acc_b - (uint32_t)p.zx * (uint32_t)sw_b - (uint32_t)L.kl;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ta += __shfl_xor_sync(0xffffffffu, ta, o);
      tb += __shfl_xor_sync(0xffffffffu, tb, o);
    }
    if (OUT_F32) {
      if (lane == 0) reinterpret_cast<float *>(p.y)[ga] = __fmul_rn(__fmul_rn((float)(int)ta, wsa), p.sa);
      if (lane == 1 && has_b)
        reinterpret_cast<float *>(p.y)[ga + 1] = __fmul_rn(__fmul_rn((float)(int)tb, wsb), p.sa);
    } else {
      if (lane == 0) reinterpret_cast<int32_t *>(p.y)[ga] = (int32_t)ta;
      if (lane == 1 && has_b) reinterpret_cast<int32_t *>(p.y)[ga + 1] = (int32_t)tb;
    }
    return false;
  }
};

// ------------------------------------------------------ streaming skeleton --
template <class Op>
__global__ void __launch_bounds__(kStreamThreads, 2)
    gemv_stream_kernel(const StreamGeom g, const typename Op::Params op) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + g.nst;
  uint8_t *xs = smem + kBarBytes;
  uint8_t *stages = xs + g.x_bytes;

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
    // Weights and scales do not depend on the previous kernel: no wait here.
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      for (int st = 0; st < nstages; ++st) {
        const int b = st % g.nst;
        if (st == g.nst) pdl_launch_dependents();
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
      if (nstages <= g.nst) pdl_launch_dependents();
      // Before the CTA may exit, every copy it issued must have landed.
      for (int st = max(0, issued - g.nst); st < issued; ++st) {
        if (!mbar_wait(&full[st % g.nst], (uint32_t)(st / g.nst) & 1u)) set_status(g.status, kStatusTimeout);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  // The activation vector (and the output) belong to the previous kernel on
  // the stream until it has completed.
  pdl_wait();
  typename Op::Lane L;
  Op::init(op, L, lane, xs, threadIdx.x);
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
    // row pairs (lo + 2q, lo + 2q + 1); pair q goes to warp (lo/2 + q) % warps
    const int pair0 = lo / 2;
    int q = ((warp - pair0 % kConsumerWarps) + kConsumerWarps) % kConsumerWarps;
    for (; lo + 2 * q < hi; q += kConsumerWarps) {
      const int i = lo + 2 * q;
      const int li = i - lo;
      bad |= Op::rows2(op, L, xs, base + (size_t)li * g.row_bytes, sbase + (size_t)li * g.srow_bytes,
                       base + (size_t)(li + 1) * g.row_bytes, sbase + (size_t)(li + 1) * g.srow_bytes, r0 + i,
                       i + 1 < hi, lane);
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
  using SB = ScaleBits<ST>;
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
      const uint32_t sb = SB::gload(sr + k / group);
      bad |= SB::bad(sb);
      acc = fmaf((float)(xv * wv), SB::f32(sb), acc);
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
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      if (OUT_F32) {
        const float d = __fmul_rn((float)(int)acc, ws[r]);
        reinterpret_cast<float *>(y)[r] = __fmul_rn(d, sa);
      } else {
        reinterpret_cast<int32_t *>(y)[r] = (int32_t)acc;
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

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ilog2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return s;
}

// Fill the ring geometry; false if the rows are too long to stage.
bool plan_stream(StreamGeom &g, int64_t rows, int row_bytes, int srow_bytes, int x_bytes, int sm_count) {
  static const int smem_cta = std::min(kSmemPerCta, env_int("KS_B200_SMEM_PER_CTA", kSmemPerCta));
  static const int min_stages = std::max(2, env_int("KS_B200_MIN_STAGES", 3));
  const int row_total = row_bytes + srow_bytes;
  const int budget = smem_cta - kBarBytes - x_bytes;
  const int64_t n_cta = std::min<int64_t>(rows, sm_count);
  const int64_t rows_cta_max = (rows + n_cta - 1) / n_cta;
  int rps = (budget / min_stages) / row_total;
  rps = std::min(rps, 2 * kConsumerWarps);
  rps = (int)std::min<int64_t>(rps, (rows_cta_max + 1) & ~int64_t(1));
  rps &= ~1;
  if (rps < 2) rps = 2;
  const int stage_bytes = ((rps * row_total + 127) / 128) * 128;
  int nst = budget / stage_bytes;
  const int64_t need = (rows_cta_max + rps - 1) / rps;
  nst = (int)std::min<int64_t>(std::min(nst, kMaxStages), need);
  if (nst < 1 || (nst < 2 && need > 1)) return false;
  g.rows = rows;
  g.n_cta = (int32_t)n_cta;
  g.rps = rps;
  g.nst = nst;
  g.row_bytes = row_bytes;
  g.srow_bytes = srow_bytes;
  g.stage_bytes = stage_bytes;
  g.x_bytes = x_bytes;
  return true;
}

size_t stream_smem_bytes(const StreamGeom &g) {
  return (size_t)kBarBytes + (size_t)g.x_bytes + (size_t)g.nst * g.stage_bytes;
}

bool pdl_enabled(cudaStream_t stream) {
  static const bool on = env_int("KS_B200_PDL", 1) != 0;
  return on && stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread;
}

template <class Op>
cudaError_t launch_stream(const StreamGeom &g, const typename Op::Params &op, cudaStream_t stream, int dev) {
  const size_t smem = stream_smem_bytes(g);
  static std::once_flag attr_once[64];
  static cudaError_t attr_err[64];
  std::call_once(attr_once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(gemv_stream_kernel<Op>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemPerCta);
  });
  if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g.n_cta);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled(stream)) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<Op>, g, op);
}

struct W4A8Plan {
  bool fast = false;
  StreamGeom g{};
  W4A8OpParams op{};
  int ncpl = 0;
};

constexpr int kMaxStreamChunks = 512;  // W4A8 rows up to 16384 columns, INT8 up to 8192

W4A8Plan plan_w4a8(const W4A8Launch &a, int device) {
  W4A8Plan P;
  const int ssize = a.stype == kScaleF16 ? 2 : 4;
  const int64_t groups = (a.cols + a.group - 1) / a.group;
  const int gshift = ilog2_exact(a.group / 32);
  const bool shape_ok = a.cols % 32 == 0 && a.group % 32 == 0 && gshift >= 0 &&
                        a.cols / 32 <= kMaxStreamChunks && a.wstride % 16 == 0 && aligned16(a.w) &&
                        (groups * ssize) % 16 == 0 && (a.sstride * ssize) % 16 == 0 && aligned16(a.s) &&
                        a.rows < (int64_t(1) << 31);
  if (!shape_ok) return P;
  const DeviceProps &dp = device_props(device);
  const int chunks = (int)(a.cols / 32);
  P.ncpl = chunks <= 32 ? 1 : chunks <= 64 ? 2 : chunks <= 128 ? 4 : chunks <= 256 ? 8 : 16;
  const bool xs = P.ncpl > 4;
  const int x_bytes = xs ? ((chunks * 36 + 127) / 128) * 128 : 0;
  StreamGeom g{};
  if (!plan_stream(g, a.rows, (int)(a.cols / 2), (int)(groups * ssize), x_bytes, dp.sm_count)) return P;
  g.w = a.w;
  g.wstride = a.wstride;
  g.s = reinterpret_cast<const uint8_t *>(a.s);
  g.sstride = a.sstride * ssize;
  g.w_contig = a.wstride == a.cols / 2;
  g.s_contig = g.sstride == g.srow_bytes;
  g.status = a.status;
  P.g = g;
  P.op.x = a.x;
  P.op.y = a.y;
  P.op.chunks = chunks;
  P.op.gshift = gshift;
  P.op.sx = a.sx;
  P.op.zx = a.zx;
  P.op.zw = a.zw;
  P.op.x_al16 = aligned16(a.x);
  P.fast = true;
  return P;
}

template <typename ST>
cudaError_t launch_w4a8_fast(const W4A8Plan &P, cudaStream_t stream, int dev) {
  switch (P.ncpl) {
    case 1: return launch_stream<W4A8Op<ST, 1, false>>(P.g, P.op, stream, dev);
    case 2: return launch_stream<W4A8Op<ST, 2, false>>(P.g, P.op, stream, dev);
    case 4: return launch_stream<W4A8Op<ST, 4, false>>(P.g, P.op, stream, dev);
    case 8: return launch_stream<W4A8Op<ST, 8, true>>(P.g, P.op, stream, dev);
    default: return launch_stream<W4A8Op<ST, 16, true>>(P.g, P.op, stream, dev);
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
  const bool shape_ok = a.cols % 16 == 0 && a.cols / 16 <= kMaxStreamChunks && a.wstride % 16 == 0 &&
                        aligned16(a.w) && a.rows < (int64_t(1) << 31);
  if (!shape_ok) return P;
  const DeviceProps &dp = device_props(device);
  const int chunks = (int)(a.cols / 16);
  P.ncpl = chunks <= 32 ? 1 : chunks <= 64 ? 2 : chunks <= 128 ? 4 : chunks <= 256 ? 8 : 16;
  const bool xs = P.ncpl > 8;
  const int x_bytes = xs ? ((chunks * 16 + 127) / 128) * 128 : 0;
  StreamGeom g{};
  if (!plan_stream(g, a.rows, (int)a.cols, 0, x_bytes, dp.sm_count)) return P;
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
  P.op.chunks = chunks;
  P.op.zx = a.zx;
  P.op.zw = a.zw;
  P.op.x_al16 = aligned16(a.x);
  P.fast = true;
  return P;
}

template <bool F32>
cudaError_t launch_i8_fast(const I8Plan &P, cudaStream_t stream, int dev) {
  switch (P.ncpl) {
    case 1: return launch_stream<I8Op<1, F32, false>>(P.g, P.op, stream, dev);
    case 2: return launch_stream<I8Op<2, F32, false>>(P.g, P.op, stream, dev);
    case 4: return launch_stream<I8Op<4, F32, false>>(P.g, P.op, stream, dev);
    case 8: return launch_stream<I8Op<8, F32, false>>(P.g, P.op, stream, dev);
    default: return launch_stream<I8Op<16, F32, true>>(P.g, P.op, stream, dev);
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
    return a.stype == kScaleF16 ? launch_w4a8_fast<__half>(P, stream, device)
                                : launch_w4a8_fast<float>(P, stream, device);
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
  if (P.fast) {
    return a.out_f32 ? launch_i8_fast<true>(P, stream, device) : launch_i8_fast<false>(P, stream, device);
  }
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
