// ks_gemv.cu -- INT8 and W4A8 GEMV kernels for B200 (sm_100a).
//
// Two kernel families per operation:
//
//  * gemv_stream_kernel<Op, CW>: the HBM-streaming path.  One CTA per SM
//    owns a contiguous block of rows of every matrix of a batch (a single
//    GEMV is a batch of one).  A producer warp streams those rows -- the
//    weights and their scale rows, matrix after matrix -- into a ring of
//    shared-memory stages with cp.async.bulk (the TMA engine, 1-D bulk form,
//    no tensor map, no multicast), one mbarrier per stage.  CW consumer warps
//    take pairs of rows, unpack int4 with LOP3, multiply with dp4a and reduce
//    each row with warp shuffles in a fixed order, so results are bitwise
//    reproducible.  Each matrix's activation vector is prepared once per CTA
//    into a double-buffered shared-memory slot (the next one while the current
//    matrix is computed), so the ring never drains between matrices.
//      - single GEMV: CW = 8, at most ~108 KB of shared memory, two CTAs per
//        SM.  With programmatic dependent launch the next GEMV on the stream
//        starts streaming its weights while this one finishes and waits for
//        it (griddepcontrol.wait) only before reading x or writing y.
//      - batch: CW = 16, one CTA per SM with a deep ring (~220 KB).
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
#include "ks_stream.cuh"

namespace ksb {

template <class Op, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, CW <= 8 ? 2 : 1)
    gemv_stream_kernel(const StreamGeom g, const typename Op::Params op, const GemvItems items,
                       const LayerExt ext) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + g.nst;
  uint8_t *xbufs = smem + kBarBytes;
  float *ostage = reinterpret_cast<float *>(xbufs + 2 * g.xbuf_bytes);  // 2 buffers (peer gather only)
  uint8_t *stages = xbufs + 2 * g.xbuf_bytes + 2 * g.ostage_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)blockIdx.x * g.rows / g.n_cta;
  const int64_t r1 = (int64_t)(blockIdx.x + 1) * g.rows / g.n_cta;
  const int rows_cta = (int)(r1 - r0);
  const int nstages = (rows_cta + g.rps - 1) / g.rps;  // per matrix
  const int total = nstages * g.count;

  if (threadIdx.x == 0) {
    for (int b = 0; b < g.nst; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], CW);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == CW) {
    // ---------------- producer: one thread issues every bulk copy ----------
    // Weights and scales do not depend on the previous kernel: no wait here.
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      // Stages beyond the ring are prefetched into L2 l2_ahead stages before
      // their copy: HBM keeps streaming while the ring is full (consumers
      // waiting for the previous kernel or for the activations), and the
      // copies of those stages then come from L2.
      auto prefetch_stage = [&](int j) {
        const GemvItem &it = items.it[j / nstages];
        const int lo = (j % nstages) * g.rps;
        const int n = min(g.rps, rows_cta - lo);
        const uint8_t *wsrc = it.w + (r0 + lo) * g.wstride;
        if (g.w_contig) {
          bulk_prefetch_l2(wsrc, (uint32_t)n * (uint32_t)g.row_bytes);
        } else {
          for (int r = 0; r < n; ++r) bulk_prefetch_l2(wsrc + (int64_t)r * g.wstride, (uint32_t)g.row_bytes);
        }
        if (g.srow_bytes) {
          const uint8_t *ssrc = it.s + (r0 + lo) * g.sstride;
          if (g.s_contig) {
            bulk_prefetch_l2(ssrc, (uint32_t)n * (uint32_t)g.srow_bytes);
          } else {
            for (int r = 0; r < n; ++r) bulk_prefetch_l2(ssrc + (int64_t)r * g.sstride, (uint32_t)g.srow_bytes);
          }
        }
      };
      const int ahead = g.l2_ahead;
      for (int j = g.nst; j < min(total, g.nst + ahead); ++j) prefetch_stage(j);
      int gs = 0;
      bool stop = false;
      for (int m = 0; m < g.count && !stop; ++m) {
        const GemvItem &it = items.it[m];
        for (int st = 0; st < nstages; ++st, ++gs) {
          const int b = gs % g.nst;
          if (gs == g.nst) pdl_launch_dependents();
          if (gs >= g.nst && !mbar_wait(&empty[b], (uint32_t)((gs / g.nst) - 1) & 1u)) {
            set_status(g.status, kStatusTimeout);
            stop = true;
            break;
          }
          const int lo = st * g.rps;
          const int n = min(g.rps, rows_cta - lo);
          const uint32_t wbytes = (uint32_t)n * (uint32_t)g.row_bytes;
          const uint32_t sbytes = (uint32_t)n * (uint32_t)g.srow_bytes;
          uint8_t *dst = stages + (size_t)b * g.stage_bytes;
          mbar_arrive_expect_tx(&full[b], wbytes + sbytes);
          const uint8_t *wsrc = it.w + (r0 + lo) * g.wstride;
          if (g.w_contig) {
            bulk_g2s_hint(dst, wsrc, wbytes, &full[b], pol);
          } else {
            for (int r = 0; r < n; ++r)
              bulk_g2s_hint(dst + (size_t)r * g.row_bytes, wsrc + (int64_t)r * g.wstride, g.row_bytes,
                            &full[b], pol);
          }
          if (g.srow_bytes) {
            uint8_t *sdst = dst + (size_t)g.rps * g.row_bytes;
            const uint8_t *ssrc = it.s + (r0 + lo) * g.sstride;
            if (g.s_contig) {
              bulk_g2s(sdst, ssrc, sbytes, &full[b]);
            } else {
              for (int r = 0; r < n; ++r)
                bulk_g2s(sdst + (size_t)r * g.srow_bytes, ssrc + (int64_t)r * g.sstride, g.srow_bytes,
                         &full[b]);
            }
          }
          if (ahead > 0 && gs >= g.nst && gs + ahead < total) prefetch_stage(gs + ahead);
        }
      }
      if (total <= g.nst) pdl_launch_dependents();
      // Before the CTA may exit, every copy it issued must have landed.
      for (int s2 = max(0, gs - g.nst); s2 < gs; ++s2) {
        if (!mbar_wait(&full[s2 % g.nst], (uint32_t)(s2 / g.nst) & 1u)) set_status(g.status, kStatusTimeout);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  // Activations (and outputs) belong to the previous kernel on the stream
  // until it has completed.
  pdl_wait();
  const int ctid = threadIdx.x;
  constexpr int NT = CW * 32;
  constexpr int RW = Op::kRawWords;
  float *red = reinterpret_cast<float *>(smem + kBarBytes - 128);  // CW <= 16 floats
  if (ext.reset_amax && blockIdx.x == 0 && ctid == 0) *ext.reset_amax = 0u;
  if (ext.xmode == kXInt8) {
    for (int c = ctid; c < op.chunks; c += NT) {
      uint32_t raw[RW];
      Op::load_raw(items.it[0].x, c, g.x_al16 != 0, raw);
      Op::store_prep(op, raw, c, xbufs);
    }
    if (ctid == 0) Op::set_sx(op, xbufs, Op::default_sx(op));
  } else {
    prep_x_f32<Op, CW>(op, ext, xbufs, red, ctid);
  }
  consumers_sync<CW>();

  // next matrix's raw int8 x fits in registers
  const bool prefetch = ext.xmode == kXInt8 && op.chunks <= 2 * NT;
  uint32_t mx = 0;
  int gs = 0;
  int pair_base = 0;
  bool stop = false;  // this warp hit a wait limit: it skips work but keeps every barrier
  for (int m = 0; m < g.count; ++m) {
    const GemvItem &it = items.it[m];
    float *ost = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ostage) + (size_t)(m & 1) * g.ostage_bytes);
    const OutRef out{it.y, &items, (int64_t)m * items.mstride + items.row_offset, &ext, m, ost, r0};
    // f32 inputs: one vector (ext.xf) for every matrix of the launch, prepared once
    const uint8_t *xb = xbufs + (ext.xmode != kXInt8 ? 0 : (size_t)(m & 1) * g.xbuf_bytes);
    uint32_t pre[2][RW];
    const bool more = m + 1 < g.count;
    if (more && prefetch && !stop) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int c = ctid + k * NT;
        if (c < op.chunks) Op::load_raw(items.it[m + 1].x, c, g.x_al16 != 0, pre[k]);
      }
    }
    typename Op::Lane L;
    Op::lane_init(op, L, xb, lane);
    for (int st = 0; st < nstages && !stop; ++st, ++gs) {
      const int b = gs % g.nst;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[b], (uint32_t)(gs / g.nst) & 1u));
      if (!ok) {
        if (lane == 0) set_status(g.status, kStatusTimeout);
        stop = true;
        break;
      }
      const int lo = st * g.rps;
      const int hi = min(lo + g.rps, rows_cta);
      const uint8_t *base = stages + (size_t)b * g.stage_bytes;
      const uint8_t *sbase = base + (size_t)g.rps * g.row_bytes;
      // row pairs (lo + 2q, lo + 2q + 1); the pair's running index across the
      // launch picks the warp, so stages alternate between warp groups
      const int pair0 = pair_base + lo / 2;
      int q = ((warp - pair0 % CW) + CW) % CW;
      for (; lo + 2 * q < hi; q += CW) {
        const int li = 2 * q;
        mx = max(mx, Op::rows2(op, L, xb, base + (size_t)li * g.row_bytes, sbase + (size_t)li * g.srow_bytes,
                               base + (size_t)(li + 1) * g.row_bytes, sbase + (size_t)(li + 1) * g.srow_bytes,
                               out, it, r0 + lo + li, lo + li + 1 < hi, lane, L));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[b]);
    }
    pair_base += (rows_cta + 1) / 2;
    if (more) {
      uint8_t *xn = xbufs + (size_t)((m + 1) & 1) * g.xbuf_bytes;
      // f32 inputs were prepared once for every matrix; the barrier below also
      // orders this matrix's output stores before the next matrix's epilogue
      // reads them (silu(gate[r]) * up[r] reads gate rows other warps wrote)
      if (!stop && ext.xmode == kXInt8) {
        if (ctid == 0) Op::set_sx(op, xn, Op::default_sx(op));
        if (prefetch) {
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int c = ctid + k * NT;
            if (c < op.chunks) Op::store_prep(op, pre[k], c, xn);
          }
        } else {
          for (int c = ctid; c < op.chunks; c += NT) {
            uint32_t raw[RW];
            Op::load_raw(items.it[m + 1].x, c, g.x_al16 != 0, raw);
            Op::store_prep(op, raw, c, xn);
          }
        }
      }
      consumers_sync<CW>();  // every consumer warp, stopped or not, takes this barrier
    }
    if (items.npeers > 0) {
      // the matrix's rows are all staged once every consumer passed a barrier
      // after them; the other staging buffer takes the next matrix's rows
      if (!more) consumers_sync<CW>();
      flush_peer_rows<CW>(items, ost, out.peer_off + r0, rows_cta, ctid);
    }
  }
  if (__any_sync(0xffffffffu, Op::bad(mx)) && lane == 0) set_status(g.status, kStatusBadScale);
  if (items.npeers > 0) {
    // all of this CTA's peer stores happen-before thread 0's system fence
    consumers_sync<CW>();
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < items.npeers; ++p)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(items.peer_cnt[p]) : "memory");
    }
  }
}

// Waits until each of this rank's `ncounters` arrival counters (one word per
// source rank) reaches the running target: the target (kept in expected[0])
// grows by `arrivals` per call -- the number of CTA signals the preceding
// sharded launches send from each source.  Lane s polls counter s.  A
// separate word per source means a fast rank's arrivals for the next run
// can never stand in for a slow rank's arrivals for this one.  Bounded by
// limit_ns of %globaltimer; a timeout sets status word 1 and the kernel
// returns (expected[0] still advances, so the next call targets the next
// run).
__global__ void peer_arrival_wait_kernel(const uint32_t *counters, int ncounters, uint32_t *expected,
                                         uint32_t arrivals, uint64_t limit_ns, uint32_t *status) {
  const int lane = threadIdx.x;
  const uint32_t target = expected[0] + arrivals;
  bool done = lane >= ncounters;
  const uint64_t t0 = globaltimer_ns();
  while (!__all_sync(0xffffffffu, done)) {
    if (!done) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(counters + lane) : "memory");
      done = (int32_t)(v - target) >= 0;
    }
    if (globaltimer_ns() - t0 > limit_ns) {
      if (lane == 0) set_status(status, kStatusTimeout);
      break;
    }
  }
  __syncwarp();
  if (lane == 0) expected[0] = target;
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

// Error path of the synchronous W4A8 calls: the reference stops at the first
// row whose scales fail validation (ks_quantized.c:148-156 with :112-114), so
// the library needs that row's index.  A warp per row tests the row's
// `groups` scales with the kernels' own bit test; the smallest failing row
// wins (atomicMin).
template <typename ST>
__global__ void __launch_bounds__(256)
    w4a8_first_bad_row_kernel(const ST *__restrict__ s, int64_t sstride, int64_t rows, int64_t groups,
                              unsigned long long *first_bad) {
  using SB = ScaleBits<ST>;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    bool bad = false;
    for (int64_t gi = lane; gi < groups; gi += 32) bad |= SB::bad(SB::gload(s + r * sstride + gi));
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicMin(first_bad, (unsigned long long)r);
  }
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

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ilog2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int s = 0;
  while ((int64_t(1) << s) < v) ++s;
  return s;
}

// Fill the ring geometry for one configuration (single or batch); false if
// the rows are too long to stage.
// l2_ahead: L2 prefetch distance in stages (measured best on B200: W4A8 1
// single / 0 batched, INT8 1 single / 0 batched; farther prefetches compete
// with the ring's own copies).  Batched W4A8 without the prefetch, per GEMV:
// 3.92 against 3.95 us at 11008 x 4096 G32, 16.99 against 17.22 us at
// 28672 x 8192 G128, 5.39 against 5.40 at 7168 x 8192.
// peer: the launch gathers its outputs by peer stores and stages each
// matrix's rows in two shared-memory buffers of rows_cta_max floats.
bool plan_stream(StreamGeom &g, int64_t rows, int row_bytes, int srow_bytes, int xbuf_bytes, int sm_count,
                 bool batch, int cw, int l2_ahead, bool peer = false) {
  static const int min_single = std::max(2, env_int("KS_B200_MIN_STAGES", 2));
  static const int ahead_single = env_int("KS_B200_L2_AHEAD_SINGLE", -1);
  static const int ahead_batch = env_int("KS_B200_L2_AHEAD_BATCH", -1);
  static const int rps_cap_batch = std::max(2, env_int("KS_B200_BATCH_ROWS_PER_STAGE", 24));
  static const int min_batch_env = env_int("KS_B200_BATCH_MIN_STAGES", -1);
  const int smem_cta = batch ? kSmemBatch : kSmemSingle;
  const int row_total = row_bytes + srow_bytes;
  const int64_t n_cta = std::min<int64_t>(rows, sm_count);
  const int64_t rows_cta_max = (rows + n_cta - 1) / n_cta;
  const int64_t ostage = peer ? (rows_cta_max * 4 + 127) / 128 * 128 : 0;
  if (ostage > smem_cta / 8) return false;
  const int budget = smem_cta - kBarBytes - 2 * xbuf_bytes - 2 * (int)ostage;
  if (budget <= 0) return false;
  int rps;
  const int64_t half = budget / 2;
  const int64_t bytes_cta = rows_cta_max * (int64_t)row_total;  // one matrix, one CTA
  if (batch && min_batch_env < 0 && bytes_cta <= 2 * half) {
    // A short stream per matrix: one or two stages of equal size per matrix,
    // as large as two fit in the ring.  Every stage is a producer / consumer
    // barrier round trip, and a small last stage of a matrix would cost one
    // for few bytes (measured on B200: 11008 x 4096 W4A8, 75 rows per CTA,
    // 4.36 us per GEMV with four stages of 22 rows, 3.99 with two of 38).
    const int64_t per_matrix = (bytes_cta + half - 1) / half;  // 1 or 2
    rps = (int)((rows_cta_max + per_matrix - 1) / per_matrix);
    rps = (rps + 1) & ~1;
  } else {
    // A long stream per matrix (or the single-GEMV kernel): a deeper ring.
    const int min_stages = batch ? std::max(2, min_batch_env > 0 ? min_batch_env : 4) : min_single;
    rps = (budget / min_stages) / row_total;
    rps = std::min(rps, batch ? rps_cap_batch : 2 * cw);
  }
  rps = (int)std::min<int64_t>(rps, (rows_cta_max + 1) & ~int64_t(1));
  rps &= ~1;
  if (rps < 2) rps = 2;
  const int stage_bytes = ((rps * row_total + 127) / 128) * 128;
  int nst = budget / stage_bytes;
  nst = std::min(nst, kMaxStages);
  if (nst < 2) return false;
  g.rows = rows;
  g.n_cta = (int32_t)n_cta;
  g.rps = rps;
  g.nst = nst;
  g.row_bytes = row_bytes;
  g.srow_bytes = srow_bytes;
  g.stage_bytes = stage_bytes;
  g.xbuf_bytes = xbuf_bytes;
  g.ostage_bytes = (int32_t)ostage;
  const int ahead_env = batch ? ahead_batch : ahead_single;
  g.l2_ahead = ahead_env >= 0 ? ahead_env : l2_ahead;
  return true;
}

size_t stream_smem_bytes(const StreamGeom &g) {
  return (size_t)kBarBytes + 2 * (size_t)g.xbuf_bytes + 2 * (size_t)g.ostage_bytes + (size_t)g.nst * g.stage_bytes;
}

template <class Op, int CW>
cudaError_t launch_stream(const StreamGeom &g, const typename Op::Params &op, const GemvItems &items,
                          cudaStream_t stream, int dev, const LayerExt &ext = LayerExt{}) {
  static std::once_flag attr_once[64];
  static cudaError_t attr_err[64];
  std::call_once(attr_once[dev & 63], [&] {
    const int want = std::min(device_props(dev).smem_optin, CW <= 8 ? kSmemSingle : kSmemBatch);
    attr_err[dev & 63] =
        cudaFuncSetAttribute(gemv_stream_kernel<Op, CW>, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
  });
  if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g.n_cta);
  cfg.blockDim = dim3((CW + 1) * 32);
  cfg.dynamicSmemBytes = stream_smem_bytes(g);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled(stream)) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<Op, CW>, g, op, items, ext);
}

int ncpl_of(int chunks) {
  return chunks <= 32 ? 1 : chunks <= 64 ? 2 : chunks <= 128 ? 4 : chunks <= 256 ? 8 : 16;
}

// ---- W4A8 ---------------------------------------------------------------
struct W4A8Plan {
  bool fast = false;
  StreamGeom g{};
  W4A8OpParams op{};
  int ncpl = 0;
};

bool w4a8_shape_ok(const W4A8Launch &a) {
  const int ssize = a.stype == kScaleF16 ? 2 : 4;
  const int64_t groups = (a.cols + a.group - 1) / a.group;
  return a.cols % 32 == 0 && a.group % 32 == 0 && ilog2_exact(a.group / 32) >= 0 &&
         a.cols / 32 <= kMaxStreamChunks && a.wstride % 16 == 0 && (groups * ssize) % 16 == 0 &&
         (a.sstride * ssize) % 16 == 0 && a.rows < (int64_t(1) << 31);
}

W4A8Plan plan_w4a8(const W4A8Launch &a, int device, bool batch, bool peer = false) {
  W4A8Plan P;
  if (!w4a8_shape_ok(a)) return P;
  const int ssize = a.stype == kScaleF16 ? 2 : 4;
  const int64_t groups = (a.cols + a.group - 1) / a.group;
  const int chunks = (int)(a.cols / 32);
  const int xbuf = ((chunks * 36 + 4 + 127) / 128) * 128;
  StreamGeom g{};
  if (!plan_stream(g, a.rows, (int)(a.cols / 2), (int)(groups * ssize), xbuf, device_props(device).sm_count,
                   batch, batch ? 16 : 8, batch ? 0 : 1, peer))
    return P;
  g.wstride = a.wstride;
  g.sstride = a.sstride * ssize;
  g.w_contig = a.wstride == a.cols / 2;
  g.s_contig = g.sstride == g.srow_bytes;
  g.status = a.status;
  P.g = g;
  P.op.chunks = chunks;
  P.op.gshift = ilog2_exact(a.group / 32);
  P.op.sx = a.sx;
  P.op.zx = a.zx;
  P.op.zw = a.zw;
  P.ncpl = ncpl_of(chunks);
  P.fast = true;
  return P;
}

template <typename ST, bool ZX, int CW>
cudaError_t launch_w4a8_ncpl(const W4A8Plan &P, const GemvItems &items, cudaStream_t stream, int dev,
                             const LayerExt &ext) {
  switch (P.ncpl) {
    case 1: return launch_stream<W4A8Op<ST, 1, ZX>, CW>(P.g, P.op, items, stream, dev, ext);
    case 2: return launch_stream<W4A8Op<ST, 2, ZX>, CW>(P.g, P.op, items, stream, dev, ext);
    case 4: return launch_stream<W4A8Op<ST, 4, ZX>, CW>(P.g, P.op, items, stream, dev, ext);
    case 8: return launch_stream<W4A8Op<ST, 8, ZX>, CW>(P.g, P.op, items, stream, dev, ext);
    default: return launch_stream<W4A8Op<ST, 16, ZX>, CW>(P.g, P.op, items, stream, dev, ext);
  }
}

template <int CW>
cudaError_t launch_w4a8_cw(const W4A8Plan &P, int stype, const GemvItems &items, cudaStream_t stream, int dev,
                           const LayerExt &ext = LayerExt{}) {
  const bool zx = P.op.zx != 0;
  if (stype == kScaleF16)
    return zx ? launch_w4a8_ncpl<__half, true, CW>(P, items, stream, dev, ext)
              : launch_w4a8_ncpl<__half, false, CW>(P, items, stream, dev, ext);
  return zx ? launch_w4a8_ncpl<float, true, CW>(P, items, stream, dev, ext)
            : launch_w4a8_ncpl<float, false, CW>(P, items, stream, dev, ext);
}

// ---- INT8 ---------------------------------------------------------------
struct I8Plan {
  bool fast = false;
  StreamGeom g{};
  I8OpParams op{};
  int ncpl = 0;
};

bool i8_shape_ok(const I8Launch &a) {
  return a.cols % 16 == 0 && a.cols / 16 <= kMaxStreamChunks && a.wstride % 16 == 0 &&
         a.rows < (int64_t(1) << 31);
}

I8Plan plan_i8(const I8Launch &a, int device, bool batch) {
  I8Plan P;
  if (!i8_shape_ok(a)) return P;
  const int chunks = (int)(a.cols / 16);
  const int xbuf = ((chunks * 20 + 127) / 128) * 128;
  StreamGeom g{};
  if (!plan_stream(g, a.rows, (int)a.cols, 0, xbuf, device_props(device).sm_count, batch, batch ? 16 : 8,
                   batch ? 0 : 1))
    return P;
  g.wstride = a.wstride;
  g.sstride = 0;
  g.w_contig = a.wstride == a.cols;
  g.s_contig = 1;
  g.status = a.status;
  P.g = g;
  P.op.sa = a.sa;
  P.op.chunks = chunks;
  P.op.zx = a.zx;
  P.op.zw = a.zw;
  P.ncpl = ncpl_of(chunks);
  P.fast = true;
  return P;
}

template <bool F32, bool ZX, int CW>
cudaError_t launch_i8_ncpl(const I8Plan &P, const GemvItems &items, cudaStream_t stream, int dev) {
  switch (P.ncpl) {
    case 1: return launch_stream<I8Op<1, F32, ZX>, CW>(P.g, P.op, items, stream, dev);
    case 2: return launch_stream<I8Op<2, F32, ZX>, CW>(P.g, P.op, items, stream, dev);
    case 4: return launch_stream<I8Op<4, F32, ZX>, CW>(P.g, P.op, items, stream, dev);
    case 8: return launch_stream<I8Op<8, F32, ZX>, CW>(P.g, P.op, items, stream, dev);
    default: return launch_stream<I8Op<16, F32, ZX>, CW>(P.g, P.op, items, stream, dev);
  }
}

template <int CW>
cudaError_t launch_i8_cw(const I8Plan &P, bool f32, const GemvItems &items, cudaStream_t stream, int dev) {
  const bool zx = P.op.zx != 0;
  if (f32)
    return zx ? launch_i8_ncpl<true, true, CW>(P, items, stream, dev)
              : launch_i8_ncpl<true, false, CW>(P, items, stream, dev);
  return zx ? launch_i8_ncpl<false, true, CW>(P, items, stream, dev)
            : launch_i8_ncpl<false, false, CW>(P, items, stream, dev);
}

int generic_grid(int64_t rows, int sm_count) {
  const int64_t blocks = (rows + 7) / 8;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sm_count * 8));
}

cudaError_t launch_w4a8_generic(const W4A8Launch &a, cudaStream_t stream, int device) {
  const int grid = generic_grid(a.rows, device_props(device).sm_count);
  if (a.stype == kScaleF16) {
    w4a8_generic_kernel<__half><<<grid, 256, 0, stream>>>(
        a.x, a.w, a.wstride, reinterpret_cast<const __half *>(a.s), a.sstride, a.y, a.rows, a.cols, a.group,
        a.sx, a.zx, a.zw, a.status);
  } else {
    w4a8_generic_kernel<float><<<grid, 256, 0, stream>>>(
        a.x, a.w, a.wstride, reinterpret_cast<const float *>(a.s), a.sstride, a.y, a.rows, a.cols, a.group,
        a.sx, a.zx, a.zw, a.status);
  }
  return cudaGetLastError();
}

cudaError_t launch_first_bad(const void *s, int stype, int64_t sstride, int64_t rows, int64_t groups,
                             unsigned long long *first_bad, cudaStream_t stream, int device) {
  const int grid = generic_grid(rows, device_props(device).sm_count);
  if (stype == kScaleF16)
    w4a8_first_bad_row_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half *>(s), sstride, rows,
                                                                groups, first_bad);
  else
    w4a8_first_bad_row_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float *>(s), sstride, rows,
                                                               groups, first_bad);
  return cudaGetLastError();
}

cudaError_t launch_i8_generic(const I8Launch &a, cudaStream_t stream, int device) {
  const int grid = generic_grid(a.rows, device_props(device).sm_count);
  if (a.out_f32) {
    i8_generic_kernel<true><<<grid, 256, 0, stream>>>(a.x, a.w, a.wstride, a.y, a.rows, a.cols, a.zx, a.zw,
                                                      a.ws, a.sa);
  } else {
    i8_generic_kernel<false><<<grid, 256, 0, stream>>>(a.x, a.w, a.wstride, a.y, a.rows, a.cols, a.zx, a.zw,
                                                       a.ws, a.sa);
  }
  return cudaGetLastError();
}

bool batch_aligned(const GemvBatch &b, bool need_s) {
  for (int i = 0; i < b.count; ++i) {
    if (!aligned16(b.w[i])) return false;
    if (need_s && !aligned16(b.s[i])) return false;
  }
  return true;
}

bool batch_x_aligned(const GemvBatch &b, int from, int n) {
  for (int i = from; i < from + n; ++i)
    if (!aligned16(b.x[i])) return false;
  return true;
}

}  // namespace

int env_int(const char *name, int dflt) {
  const char *v = std::getenv(name);
  return v && *v ? std::atoi(v) : dflt;
}

bool pdl_enabled(cudaStream_t stream) {
  static const bool on = env_int("KS_B200_PDL", 1) != 0;
  return on && stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread;
}

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
  return (aligned16(a.w) && aligned16(a.s) && plan_w4a8(a, dev, false).fast) ? 1 : 0;
}

int i8_path(const I8Launch &a) {
  int dev = 0;
  cudaGetDevice(&dev);
  return (aligned16(a.w) && plan_i8(a, dev, false).fast) ? 1 : 0;
}

// A single GEMV whose rows give each CTA at least this many bytes to stream
// takes the one-CTA-per-SM geometry with the deep (~200 KB) ring instead of
// the two-CTA form (~100 KB each, so that the next launch of a chain can
// start beside it).  Measured on B200, W4A8 G128 f16, one launch per matrix
// in a dependent chain: 28672 x 8192 (800 KB per CTA) 21.4 against 25.8 us,
// 7168 x 8192 (207 KB) 8.53 against 8.72 us; 11008 x 4096 G32 (171 KB)
// 7.56 against 7.37 us, so it keeps the two-CTA form.
constexpr int64_t kDeepSingleBytes = 192 * 1024;

cudaError_t launch_w4a8(const W4A8Launch &a, cudaStream_t stream, int device) {
  W4A8Plan P;
  if (aligned16(a.w) && aligned16(a.s)) P = plan_w4a8(a, device, false);
  if (!P.fast) return launch_w4a8_generic(a, stream, device);
  GemvItems items{};
  items.it[0] = GemvItem{a.x, a.w, reinterpret_cast<const uint8_t *>(a.s), a.y};
  const int64_t cta_bytes = (P.g.rows + P.g.n_cta - 1) / P.g.n_cta * (int64_t)(P.g.row_bytes + P.g.srow_bytes);
  if (cta_bytes >= kDeepSingleBytes) {
    W4A8Plan Q = plan_w4a8(a, device, true);
    if (Q.fast) {
      Q.g.count = 1;
      Q.g.x_al16 = aligned16(a.x);
      return launch_w4a8_cw<16>(Q, a.stype, items, stream, device);
    }
  }
  P.g.count = 1;
  P.g.x_al16 = aligned16(a.x);
  return launch_w4a8_cw<8>(P, a.stype, items, stream, device);
}

// f32 activations, quantised per token inside the kernel (s = max|x| / 127,
// round half to even; the decode layer's kXF32 preparation), then the W4A8
// GEMV.  Streaming kernel only (its shape rules, 16-byte aligned x, zero
// points 0), else cudaErrorNotSupported.
cudaError_t launch_w4a8_f32in(const W4A8Launch &a, const float *xf, int8_t *xq_out, float *xs_out,
                              cudaStream_t stream, int device) {
  if (!aligned16(a.w) || !aligned16(a.s) || !aligned16(xf) || a.zx != 0 || a.zw != 0) return cudaErrorNotSupported;
  W4A8Plan P = plan_w4a8(a, device, false);
  if (!P.fast) return cudaErrorNotSupported;
  LayerExt ext{};
  ext.xmode = kXF32;
  ext.xf = xf;
  ext.xq_out = xq_out;
  ext.xs_out = xs_out;
  GemvItems items{};
  items.it[0] = GemvItem{nullptr, a.w, reinterpret_cast<const uint8_t *>(a.s), a.y};
  P.g.count = 1;
  P.g.x_al16 = 1;
  return launch_w4a8_cw<8>(P, a.stype, items, stream, device, ext);
}

cudaError_t launch_w4a8_batch(const W4A8Launch &shape, const GemvBatch &b, cudaStream_t stream, int device) {
  if (b.count <= 0) return cudaSuccess;
  W4A8Plan P;
  if (batch_aligned(b, true)) P = plan_w4a8(shape, device, b.count > 1);
  for (int i0 = 0; i0 < b.count; i0 += kMaxItems) {
    const int n = std::min(kMaxItems, b.count - i0);
    cudaError_t e;
    if (!P.fast) {
      for (int i = i0; i < i0 + n; ++i) {
        W4A8Launch a = shape;
        a.x = b.x[i];
        a.w = static_cast<const uint8_t *>(b.w[i]);
        a.s = b.s[i];
        a.y = static_cast<float *>(b.y[i]);
        if ((e = launch_w4a8_generic(a, stream, device)) != cudaSuccess) return e;
      }
      continue;
    }
    GemvItems items{};
    for (int i = 0; i < n; ++i)
      items.it[i] = GemvItem{b.x[i0 + i], static_cast<const uint8_t *>(b.w[i0 + i]),
                             static_cast<const uint8_t *>(b.s[i0 + i]), b.y[i0 + i]};
    W4A8Plan Q = P;
    Q.g.count = n;
    Q.g.x_al16 = batch_x_aligned(b, i0, n);
    e = b.count > 1 ? launch_w4a8_cw<16>(Q, shape.stype, items, stream, device)
                    : launch_w4a8_cw<8>(Q, shape.stype, items, stream, device);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_i8(const I8Launch &a, cudaStream_t stream, int device) {
  I8Plan P;
  if (aligned16(a.w)) P = plan_i8(a, device, false);
  if (!P.fast) return launch_i8_generic(a, stream, device);
  GemvItems items{};
  items.it[0] = GemvItem{a.x, reinterpret_cast<const uint8_t *>(a.w), reinterpret_cast<const uint8_t *>(a.ws), a.y};
  P.g.count = 1;
  P.g.x_al16 = aligned16(a.x);
  return launch_i8_cw<8>(P, a.out_f32 != 0, items, stream, device);
}

cudaError_t launch_i8_batch(const I8Launch &shape, const GemvBatch &b, cudaStream_t stream, int device) {
  if (b.count <= 0) return cudaSuccess;
  I8Plan P;
  if (batch_aligned(b, false)) P = plan_i8(shape, device, b.count > 1);
  for (int i0 = 0; i0 < b.count; i0 += kMaxItems) {
    const int n = std::min(kMaxItems, b.count - i0);
    cudaError_t e;
    if (!P.fast) {
      for (int i = i0; i < i0 + n; ++i) {
        I8Launch a = shape;
        a.x = b.x[i];
        a.w = static_cast<const int8_t *>(b.w[i]);
        a.ws = static_cast<const float *>(b.s ? b.s[i] : nullptr);
        a.y = b.y[i];
        if ((e = launch_i8_generic(a, stream, device)) != cudaSuccess) return e;
      }
      continue;
    }
    GemvItems items{};
    for (int i = 0; i < n; ++i)
      items.it[i] = GemvItem{b.x[i0 + i], static_cast<const uint8_t *>(b.w[i0 + i]),
                             static_cast<const uint8_t *>(b.s ? b.s[i0 + i] : nullptr), b.y[i0 + i]};
    I8Plan Q = P;
    Q.g.count = n;
    Q.g.x_al16 = batch_x_aligned(b, i0, n);
    e = b.count > 1 ? launch_i8_cw<16>(Q, shape.out_f32 != 0, items, stream, device)
                    : launch_i8_cw<8>(Q, shape.out_f32 != 0, items, stream, device);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_w4a8_batch_gather(const W4A8Launch &shape, const GemvBatch &b, const PeerGather &pg,
                                     cudaStream_t stream, int device, uint32_t *signals_per_rank) {
  *signals_per_rank = 0;
  if (pg.npeers < 1 || pg.npeers > kMaxPeers) return cudaErrorInvalidValue;
  if (b.count <= 0) return cudaSuccess;
  if (!batch_aligned(b, true)) return cudaErrorInvalidValue;
  W4A8Plan P = plan_w4a8(shape, device, b.count > 1, /*peer=*/true);
  if (!P.fast) return cudaErrorInvalidValue;
  const bool wide = b.count > 1;
  for (int i0 = 0; i0 < b.count; i0 += kMaxItems) {
    const int n = std::min(kMaxItems, b.count - i0);
    GemvItems items{};
    for (int i = 0; i < n; ++i)
      items.it[i] = GemvItem{b.x[i0 + i], static_cast<const uint8_t *>(b.w[i0 + i]),
                             static_cast<const uint8_t *>(b.s[i0 + i]), nullptr};
    for (int p = 0; p < pg.npeers; ++p) {
      items.peer_y[p] = pg.peer_y[p] + (int64_t)i0 * pg.mstride;
      items.peer_cnt[p] = pg.peer_cnt[p];
    }
    items.npeers = pg.npeers;
    items.mstride = pg.mstride;
    items.row_offset = pg.row_offset;
    W4A8Plan Q = P;
    Q.g.count = n;
    Q.g.x_al16 = batch_x_aligned(b, i0, n);
    cudaError_t e = wide ? launch_w4a8_cw<16>(Q, shape.stype, items, stream, device)
                         : launch_w4a8_cw<8>(Q, shape.stype, items, stream, device);
    if (e != cudaSuccess) return e;
    *signals_per_rank += (uint32_t)Q.g.n_cta;
  }
  return cudaSuccess;
}

cudaError_t launch_w4a8_first_bad_row(const void *s, int stype, int64_t sstride, int64_t rows, int64_t groups,
                                      unsigned long long *first_bad, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  return launch_first_bad(s, stype, sstride, rows, groups, first_bad, stream, dev);
}

cudaError_t launch_peer_wait(const uint32_t *counters, int ncounters, uint32_t *expected, uint32_t arrivals,
                             uint64_t limit_ns, uint32_t *status, cudaStream_t stream) {
  if (ncounters < 1 || ncounters > 32) return cudaErrorInvalidValue;
  peer_arrival_wait_kernel<<<1, 32, 0, stream>>>(counters, ncounters, expected, arrivals, limit_ns, status);
  return cudaGetLastError();
}

// One quantised decode layer (batch 1): four chained launches of the
// streaming W4A8 kernel with fused activation preparation and epilogues.
//   1  qkv  = W_qkv . q(RMSNorm(h_in, norm1))            (RMSNorm + quantise in the prologue)
//   2  h2   = h_in + W_o . q(qkv[2h:3h])                  (attention at one position is V)
//   3  gate = W_g . q(RMSNorm(h2, norm2)), up = W_u . (same); act = silu(gate) * up, max|act|
//   4  h_out = h2 + W_d . q(act)                          (scale from max|act|)
cudaError_t launch_decode_layer_w4a8(const DecodeLayerArgs &a, cudaStream_t stream, int device) {
  DecodeLayerWeights lw{};
  for (int k = 0; k < 5; ++k) {
    lw.w[k] = a.w[k];
    lw.s[k] = a.s[k];
  }
  lw.norm1_w = a.norm1_w;
  lw.norm2_w = a.norm2_w;
  DecodeLayersArgs c{};
  c.layers = 1;
  c.lw = &lw;
  c.h_in = a.h_in;
  c.h_out = a.h_out;
  c.eps = a.eps;
  c.hidden = a.hidden;
  c.inter = a.inter;
  c.group = a.group;
  c.qkv = a.qkv;
  c.h2 = a.h2;
  c.gate = a.gate;
  c.up = a.up;
  c.act = a.act;
  c.scales = a.scales;
  c.amax = a.amax;
  for (int k = 0; k < 4; ++k) c.q[k] = a.q[k];
  c.status = a.status;
  return launch_decode_layers_w4a8(c, stream, device);
}

cudaError_t launch_decode_layer_four(const DecodeLayerArgs &a, cudaStream_t stream, int device) {
  const int64_t h = a.hidden, i = a.inter;
  struct Stage {
    int64_t rows, cols;
    int count;
    const uint8_t *w[2];
    const void *s[2];
    float *y[2];
    LayerExt ext;
  } st[4] = {};
  st[0] = {3 * h, h, 1, {a.w[0]}, {a.s[0]}, {a.qkv}, LayerExt{}};
  st[0].ext.xmode = kXRmsNorm;
  st[0].ext.xf = a.h_in;
  st[0].ext.norm_w = a.norm1_w;
  st[0].ext.eps = a.eps;
  st[0].ext.reset_amax = a.amax;
  st[1] = {h, h, 1, {a.w[1]}, {a.s[1]}, {a.h2}, LayerExt{}};
  st[1].ext.xmode = kXF32;
  st[1].ext.xf = a.qkv + 2 * h;
  st[1].ext.epi = kEpiResidual;
  st[1].ext.res = a.h_in;
  st[2] = {i, h, 2, {a.w[2], a.w[3]}, {a.s[2], a.s[3]}, {a.gate, a.up}, LayerExt{}};
  st[2].ext.xmode = kXRmsNorm;
  st[2].ext.xf = a.h2;
  st[2].ext.norm_w = a.norm2_w;
  st[2].ext.eps = a.eps;
  st[2].ext.epi = kEpiSiluMul;
  st[2].ext.gate = a.gate;
  st[2].ext.act_out = a.act;
  st[2].ext.amax_out = a.amax;
  st[3] = {h, i, 1, {a.w[4]}, {a.s[4]}, {a.h_out}, LayerExt{}};
  st[3].ext.xmode = kXF32Amax;
  st[3].ext.xf = a.act;
  st[3].ext.amax_in = a.amax;
  st[3].ext.epi = kEpiResidual;
  st[3].ext.res = a.h2;
  for (int k = 0; k < 4; ++k) {
    Stage &S = st[k];
    S.ext.xq_out = a.q[k];
    S.ext.xs_out = a.scales + k;
    W4A8Launch shape{};
    shape.wstride = S.cols / 2;
    shape.sstride = S.cols / a.group;
    shape.stype = kScaleF16;
    shape.rows = S.rows;
    shape.cols = S.cols;
    shape.group = a.group;
    shape.sx = 1.0f;
    shape.status = a.status;
    for (int m = 0; m < S.count; ++m)
      if (!aligned16(S.w[m]) || !aligned16(S.s[m])) return cudaErrorInvalidValue;
    W4A8Plan P = plan_w4a8(shape, device, false);
    if (!P.fast) return cudaErrorInvalidValue;
    GemvItems items{};
    for (int m = 0; m < S.count; ++m) items.it[m] = GemvItem{nullptr, S.w[m], static_cast<const uint8_t *>(S.s[m]), S.y[m]};
    P.g.count = S.count;
    P.g.x_al16 = 1;
    cudaError_t e = launch_w4a8_cw<8>(P, kScaleF16, items, stream, device, S.ext);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ksb
