// ks_decode.cu -- the fused W4A8 decode layer (hidden h, intermediate i,
// batch 1) as ONE persistent kernel on B200 (sm_100a).
//
//   1  qkv   = W_qkv . q(RMSNorm(h_in, norm1))        [3h x h]
//   2  h2    = h_in + W_o . q(qkv[2h:3h])             [h x h]   (attention at one position is V)
//   3  gate  = W_g . q(RMSNorm(h2, norm2)),  up = W_u . (same)   [i x h] twice
//      act   = silu(gate) * up,  max|act| (atomicMax on the bits)
//   4  h_out = h2 + W_d . q(act)                      [h x i]   (scale from max|act|)
//
// q(v) is the per-token int8 quantisation (s = max|v| / 127, round half to
// even); every GEMV is the W4A8 streaming dot of ks_gemv.cu (int32 per
// 32-element chunk, f16 group scales), so each stage's results are the same
// as the four-launch path's for the same quantised input.
//
// Why one kernel: the layer is a chain of four dependent GEMVs whose weights
// (114 MB for h = 4096, i = 11008) are the whole cost.  Launched one by one,
// each stage waits for the previous one to drain, then prepares its input,
// and HBM idles in between.  Here a cooperative grid of one CTA per SM runs
// all four stages:
//   * warp 16 (producer) streams this CTA's rows of all five matrices, stage
//     after stage, weights and f16 scale rows with cp.async.bulk (1-D, no
//     tensor map, no multicast) into a ring of ~24 KB slots.  Weights do not
//     depend on the activations, so it never waits for anything but a free
//     slot and keeps HBM busy across the stage boundaries.
//   * warps 0-15 (consumers), per stage: wait at a grid barrier for the
//     previous stage's outputs, prepare the input vector (RMSNorm /
//     quantisation, identical in every CTA; each thread holds its 8-element
//     groups in registers from one load to the quantised bytes), then take
//     pairs of rows from the ring and write the stage's outputs with its
//     epilogue.
// The ring (~8 slots, ~195 KB per SM) holds about 4 us of HBM traffic.
//
// Grid barrier: a 64-bit arrival counter in the workspace that only grows
// (see grid_barrier); every spin is bounded (about one second) and on a
// timeout the status word records it and the CTA goes on, so the kernel
// always terminates.  All CTAs are resident at once (cooperative launch), so
// no CTA waits for one that cannot run.
//
// Within one launch no SM reads an activation address before another SM's
// last write to it (each intermediate is written in one stage and read only
// in later ones), so plain cached loads see the current data; max|act| is
// updated with atomics in L2 and read with an L2 load.

#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "ks_internal.h"
#include "ks_ptx.cuh"
#include "ks_stream.cuh"

namespace ksb {

namespace {

constexpr int kDecCW = 16;  // consumer warps
constexpr int kDecThreads = (kDecCW + 1) * 32;
constexpr int kDecMaxSlots = 16;
constexpr int kDecSlotTarget = 64 * 1024;  // bytes of one ring slot, about (fewer, longer copies)

// One stage as both the producer and the consumers walk it.
struct DecStage {
  const uint8_t *w[2];  // packed int4 rows, dense (row stride = row_bytes)
  const uint8_t *s[2];  // f16 group-scale rows, dense (row stride = srow_bytes)
  int32_t count;        // matrices (2: gate and up)
  int32_t rows, cols;
  int32_t row_bytes, srow_bytes;
  int32_t rps;  // rows per ring slot (even)
};

struct DecParams {
  DecStage st[4];
  int32_t nslots, slot_bytes, xbuf_bytes;
  int32_t gshift;    // log2(group / 32)
  int32_t inflight;  // slots issued and not yet landed, at most (0: up to the ring)
  int32_t l2_ahead;  // slots prefetched into L2 ahead of their copy
  // activations and workspace
  const float *h_in;
  float *h_out;
  const float *norm1_w, *norm2_w;
  float eps;
  float *qkv, *h2, *gate, *up, *act, *scales;
  uint32_t *amax;
  unsigned long long *bar_count;  // 64-bit grid-barrier arrival counter
  int8_t *q[4];
  uint32_t *status;
};

// ---- epilogues (Out types of W4A8Op::rows2) -------------------------------
// pre(r, ok) issues the epilogue's global load for row r before the row's dot
// product (ok: this lane writes row r); store(r, v, pre) writes the result.
struct PlainOut {
  float *y;
  struct Pre {};
  __device__ __forceinline__ Pre pre(int64_t, bool) const { return {}; }
  __device__ __forceinline__ void store(int64_t r, float v, Pre) const { y[r] = v; }
};
struct ResidualOut {
  float *y;
  const float *res;
  struct Pre {
    float res;
  };
  __device__ __forceinline__ Pre pre(int64_t r, bool ok) const { return {ok ? res[r] : 0.0f}; }
  __device__ __forceinline__ void store(int64_t r, float v, Pre p) const { y[r] = __fadd_rn(v, p.res); }
};
// up[r] = v;  act[r] = silu(gate[r]) * v;  max|act| bits into a shared-memory
// word (one global atomicMax per CTA afterwards, not one per row)
struct SiluMulOut {
  float *up;
  const float *gate;
  float *act;
  uint32_t *amax_cta;  // shared memory
  struct Pre {
    float g;
  };
  __device__ __forceinline__ Pre pre(int64_t r, bool ok) const { return {ok ? gate[r] : 0.0f}; }
  __device__ __forceinline__ void store(int64_t r, float v, Pre p) const {
    const float a = __fmul_rn(__fdiv_rn(p.g, __fadd_rn(1.0f, expf(-p.g))), v);
    act[r] = a;
    atomicMax(amax_cta, __float_as_uint(fabsf(a)));
    up[r] = v;
  }
};

// ---- grid barrier ----------------------------------------------------------
// A 64-bit arrival counter in the workspace that only grows: every CTA adds 1
// per barrier, kBarriers barriers per launch, so at the start of a launch it
// holds kBarriers * grid * (launches so far) plus at most grid - 1 arrivals
// of this launch; rounding down to a multiple of kBarriers * grid gives the
// launch's base, and barrier k is passed once the counter reaches
// base + (k + 1) * grid.  No reset, so the last arrival costs no extra round
// trip.
constexpr int kBarriers = 3;

__device__ __forceinline__ uint64_t ld_acquire_gpu_u64(const unsigned long long *p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t barrier_base(const unsigned long long *count) {
  const uint64_t per_launch = (uint64_t)kBarriers * gridDim.x;
  const uint64_t v = ld_acquire_gpu_u64(count);
  return v - v % per_launch;
}

// Every consumer thread of every CTA calls it, k = 0, 1, 2 in order.  All of
// this CTA's consumer writes before it are visible to every consumer thread
// of the grid after it.
__device__ void grid_barrier(unsigned long long *count, uint64_t base, int k, int ctid, uint32_t *status) {
  consumers_sync<kDecCW>();
  if (ctid == 0) {
    // release: this CTA's writes (ordered before it by the CTA barrier) are
    // visible to whoever acquires a count that includes this arrival
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(count) : "memory");
    const uint64_t target = base + (uint64_t)(k + 1) * gridDim.x;
    const uint64_t t0 = globaltimer_ns();
    while ((int64_t)(ld_acquire_gpu_u64(count) - target) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(status, kStatusTimeout);
        break;
      }
      __nanosleep(32);
    }
  }
  consumers_sync<kDecCW>();  // the acquire above, passed on to every consumer thread
}

// ---- input preparation in registers ---------------------------------------
// Consumer thread t owns the 8-element groups t, t + NT, ... (NT = 512) of the
// stage's input vector, i.e. words 2q, 2q+1 (q = group % 4) of chunk group / 4,
// and keeps them in registers from the load through the quantisation: one
// memory round trip per stage.  The prepared layout is W4A8Op::store_prep's:
// even-k bytes of the chunk's word pairs at xb + 16c + 4q, odd-k bytes at
// xb + 16 * chunks + 16c + 4q, kc = 8 * sum(chunk) at xb + 32 * chunks + 4c (zero
// points are 0), the scale at xb + 36 * chunks.
constexpr int kNT = kDecCW * 32;

template <int J>
__device__ __forceinline__ void load_groups(const float *x, int ngroups, int ctid, float (&v)[J][8]) {
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int gi = ctid + j * kNT;
    const float4 *p = reinterpret_cast<const float4 *>(x + 8 * (size_t)min(gi, ngroups - 1));
    const float4 a = p[0], b = p[1];
    const bool ok = gi < ngroups;
    v[j][0] = ok ? a.x : 0.0f;
    v[j][1] = ok ? a.y : 0.0f;
    v[j][2] = ok ? a.z : 0.0f;
    v[j][3] = ok ? a.w : 0.0f;
    v[j][4] = ok ? b.x : 0.0f;
    v[j][5] = ok ? b.y : 0.0f;
    v[j][6] = ok ? b.z : 0.0f;
    v[j][7] = ok ? b.w : 0.0f;
  }
}

enum PrepMode { kPrepPlain, kPrepRms, kPrepAmaxGiven };

// v: the thread's groups (loaded); nw: RMSNorm weights of the same groups.
template <int J>
__device__ void prep_groups(int K, int mode, float (&v)[J][8], const float (&nw)[J][8], float eps, float amax_given,
                            uint8_t *xb, int8_t *xq_out, float *xs_out, float *red, int ctid) {
  const int ngroups = K / 8, chunks = K / 32;
  if (mode == kPrepRms) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) ss = __fadd_rn(ss, __fmul_rn(v[j][t], v[j][t]));
    ss = consumers_sum<kDecCW>(ss, red, ctid);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) v[j][t] = __fmul_rn(__fmul_rn(v[j][t], scale), nw[j][t]);
  }
  float amax;
  if (mode == kPrepAmaxGiven) {
    amax = amax_given;
  } else {
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) m = fmaxf(m, fabsf(v[j][t]));
    amax = consumers_max<kDecCW>(m, red, ctid);
  }
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, s);
  const bool fast = isfinite(inv);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int gi = ctid + j * kNT;  // groups of one chunk: 4 consecutive lanes
    uint32_t w[2] = {0u, 0u};
    if (gi < ngroups) {
      bool near = !fast;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          bool nb;
          w[h] |= quant_rne_byte_inv(v[j][4 * h + b], inv, nb) << (8 * b);
          near = near || nb;
        }
      }
      if (near) {  // rare: a value near a rounding tie, divide
#pragma unroll
        for (int h = 0; h < 2; ++h)
          w[h] = quant_rne_byte(v[j][4 * h], s) | (quant_rne_byte(v[j][4 * h + 1], s) << 8) |
                 (quant_rne_byte(v[j][4 * h + 2], s) << 16) | (quant_rne_byte(v[j][4 * h + 3], s) << 24);
      }
      const int c = gi >> 2, q = gi & 3;
      *reinterpret_cast<uint32_t *>(xb + 16 * c + 4 * q) = prmt(w[0], w[1], 0x6420);
      *reinterpret_cast<uint32_t *>(xb + 16 * chunks + 16 * c + 4 * q) = prmt(w[0], w[1], 0x7531);
      if (xq_out && blockIdx.x == 0) *reinterpret_cast<uint2 *>(xq_out + 8 * (size_t)gi) = make_uint2(w[0], w[1]);
    }
    int sum = dp4a_ss(w[1], 0x01010101u, dp4a_ss(w[0], 0x01010101u, 0));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (gi < ngroups && (gi & 3) == 0) reinterpret_cast<int *>(xb + 32 * chunks)[gi >> 2] = 8 * sum;
  }
  if (ctid == 0) {
    *reinterpret_cast<float *>(xb + 36 * chunks) = s;
    if (xs_out && blockIdx.x == 0) *xs_out = s;
  }
  consumers_sync<kDecCW>();
}

// ---- consumers: one matrix of one stage -------------------------------------
template <int NCPL, class Out>
__device__ __forceinline__ void consume_matrix(const DecParams &P, const DecStage &S, const Out &out,
                                               const uint8_t *xb, const uint8_t *ring, uint64_t *full,
                                               uint64_t *empty, int64_t r0, int rows_cta, int &gs, int &pair_base,
                                               uint32_t &mx, bool &stop, int warp, int lane) {
  using Op = W4A8Op<__half, NCPL, false>;
  const W4A8OpParams op{S.cols / 32, P.gshift, 1.0f, 0, 0};
  typename Op::Lane L;
  Op::lane_init(op, L, xb, lane);
  const GemvItem none{};
  const int nblk = (rows_cta + S.rps - 1) / S.rps;
  for (int st = 0; st < nblk; ++st, ++gs) {
    if (stop) continue;  // keeps gs in step with the producer's numbering
    const int b = gs % P.nslots;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[b], (uint32_t)(gs / P.nslots) & 1u));
    if (!ok) {
      if (lane == 0) set_status(P.status, kStatusTimeout);
      stop = true;
      continue;
    }
    const int lo = st * S.rps;
    const int hi = min(lo + S.rps, rows_cta);
    const uint8_t *base = ring + (size_t)b * P.slot_bytes;
    const uint8_t *sbase = base + (size_t)S.rps * S.row_bytes;
    // row pairs (lo + 2q, lo + 2q + 1); the pair's running index picks the
    // warp, so consecutive slots start on different warps
    const int pair0 = pair_base + lo / 2;
    for (int q = ((warp - pair0 % kDecCW) + kDecCW) % kDecCW; lo + 2 * q < hi; q += kDecCW) {
      const int li = 2 * q;
      mx = max(mx, Op::rows2(op, L, xb, base + (size_t)li * S.row_bytes, sbase + (size_t)li * S.srow_bytes,
                             base + (size_t)(li + 1) * S.row_bytes, sbase + (size_t)(li + 1) * S.srow_bytes, out,
                             none, r0 + lo + li, lo + li + 1 < hi, lane, L));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[b]);
  }
  pair_base += (rows_cta + 1) / 2;
}

__device__ __forceinline__ void rows_of(const DecStage &S, int64_t &r0, int &n) {
  r0 = (int64_t)blockIdx.x * S.rows / gridDim.x;
  n = (int)((int64_t)(blockIdx.x + 1) * S.rows / gridDim.x - r0);
}

// NH, NI: 32-element chunks per lane for rows of h and of i columns.
template <int NH, int NI>
__global__ void __launch_bounds__(kDecThreads, 1) decode_layer_kernel(const __grid_constant__ DecParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + P.nslots;
  float *red = reinterpret_cast<float *>(smem + kBarBytes - 128);  // kDecCW floats
  uint32_t *amax_cta = reinterpret_cast<uint32_t *>(smem + kBarBytes - 192);  // this CTA's max|act| bits
  uint8_t *xb = smem + kBarBytes;
  uint8_t *ring = xb + P.xbuf_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < P.nslots; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], kDecCW);
    }
    *amax_cta = 0u;
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == kDecCW) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      // L2 prefetch cursor, l2_ahead slots ahead of the copies: while the
      // consumers sit at a grid barrier and the ring is full, HBM keeps
      // streaming the next slots into L2, and their copies then come from L2.
      int cs = 0, cm = 0, clo = 0, cn = 0;
      int64_t cr0 = 0;
      rows_of(P.st[0], cr0, cn);
      auto settle = [&]() {
        while (cs < 4 && clo >= cn) {
          clo = 0;
          if (++cm >= P.st[cs].count) {
            cm = 0;
            if (++cs < 4) rows_of(P.st[cs], cr0, cn);
          }
        }
      };
      auto advance = [&]() {
        clo += P.st[cs].rps;
        settle();
      };
      auto prefetch = [&]() {
        const DecStage &S = P.st[cs];
        const uint32_t n = (uint32_t)min(S.rps, cn - clo);
        bulk_prefetch_l2(S.w[cm] + (cr0 + clo) * S.row_bytes, n * (uint32_t)S.row_bytes);
        bulk_prefetch_l2(S.s[cm] + (cr0 + clo) * S.srow_bytes, n * (uint32_t)S.srow_bytes);
        advance();
      };
      settle();
      for (int j = 0; j < P.nslots && cs < 4; ++j) advance();
      for (int j = 0; j < P.l2_ahead && cs < 4; ++j) prefetch();
      int gs = 0;
      bool stop = false;
      for (int s = 0; s < 4 && !stop; ++s) {
        const DecStage &S = P.st[s];
        int64_t r0;
        int rows_cta;
        rows_of(S, r0, rows_cta);
        for (int m = 0; m < S.count && !stop; ++m) {
          for (int lo = 0; lo < rows_cta; lo += S.rps, ++gs) {
            const int b = gs % P.nslots;
            if (gs >= P.nslots && !mbar_wait(&empty[b], (uint32_t)((gs / P.nslots) - 1) & 1u)) {
              set_status(P.status, kStatusTimeout);
              stop = true;
              break;
            }
            // at most `inflight` slots issued and not yet landed: a shorter
            // memory queue keeps the barrier's and the input loads' latency low
            if (P.inflight > 0 && gs >= P.inflight) {
              const int g2 = gs - P.inflight;
              if (!mbar_wait(&full[g2 % P.nslots], (uint32_t)(g2 / P.nslots) & 1u)) {
                set_status(P.status, kStatusTimeout);
                stop = true;
                break;
              }
            }
            const int n = min(S.rps, rows_cta - lo);
            const uint32_t wbytes = (uint32_t)n * (uint32_t)S.row_bytes;
            const uint32_t sbytes = (uint32_t)n * (uint32_t)S.srow_bytes;
            uint8_t *dst = ring + (size_t)b * P.slot_bytes;
            mbar_arrive_expect_tx(&full[b], wbytes + sbytes);
            bulk_g2s_hint(dst, S.w[m] + (r0 + lo) * S.row_bytes, wbytes, &full[b], pol);
            bulk_g2s(dst + (size_t)S.rps * S.row_bytes, S.s[m] + (r0 + lo) * S.srow_bytes, sbytes, &full[b]);
            if (gs >= P.nslots && P.l2_ahead > 0 && cs < 4) prefetch();
          }
        }
      }
      // every copy issued must land before the CTA may exit
      for (int g2 = max(0, gs - P.nslots); g2 < gs; ++g2)
        if (!mbar_wait(&full[g2 % P.nslots], (uint32_t)(g2 / P.nslots) & 1u)) set_status(P.status, kStatusTimeout);
    }
    return;
  }

  // ------------------------------------------------------------- consumers --
  constexpr int JH = NH / 4, JI = NI / 4;  // 8-element groups per thread (NT = 512)
  const int ctid = threadIdx.x;
  const int64_t h = P.st[1].rows, inter = P.st[2].rows;
  int gs = 0, pair_base = 0;
  uint32_t mx = 0;
  bool stop = false;
  int64_t r0;
  int nr;
  const uint64_t base = ctid == 0 ? barrier_base(P.bar_count) : 0;
  // RMSNorm weights of this thread's groups, for stages 1 and 3, loaded once
  float n1[JH][8], n2[JH][8];
  load_groups<JH>(P.norm1_w, (int)(h / 8), ctid, n1);
  load_groups<JH>(P.norm2_w, (int)(h / 8), ctid, n2);

  // stage 1: qkv = W_qkv . q(RMSNorm(h_in, norm1))
  if (blockIdx.x == 0 && ctid == 0) atomicExch(P.amax, 0u);
  {
    float v[JH][8];
    load_groups<JH>(P.h_in, (int)(h / 8), ctid, v);
    prep_groups<JH>((int)h, kPrepRms, v, n1, P.eps, 0.0f, xb, P.q[0], P.scales + 0, red, ctid);
    rows_of(P.st[0], r0, nr);
    consume_matrix<NH>(P, P.st[0], PlainOut{P.qkv}, xb, ring, full, empty, r0, nr, gs, pair_base, mx, stop, warp,
                       lane);
  }
  grid_barrier(P.bar_count, base, 0, ctid, P.status);

  // stage 2: h2 = h_in + W_o . q(qkv[2h:3h])
  {
    float v[JH][8];
    load_groups<JH>(P.qkv + 2 * h, (int)(h / 8), ctid, v);
    prep_groups<JH>((int)h, kPrepPlain, v, n1, P.eps, 0.0f, xb, P.q[1], P.scales + 1, red, ctid);
    rows_of(P.st[1], r0, nr);
    consume_matrix<NH>(P, P.st[1], ResidualOut{P.h2, P.h_in}, xb, ring, full, empty, r0, nr, gs, pair_base, mx,
                       stop, warp, lane);
  }
  grid_barrier(P.bar_count, base, 1, ctid, P.status);

  // stage 3: gate, up = W_g, W_u . q(RMSNorm(h2, norm2)); act = silu(gate) * up
  {
    float v[JH][8];
    load_groups<JH>(P.h2, (int)(h / 8), ctid, v);
    prep_groups<JH>((int)h, kPrepRms, v, n2, P.eps, 0.0f, xb, P.q[2], P.scales + 2, red, ctid);
    rows_of(P.st[2], r0, nr);
    consume_matrix<NH>(P, P.st[2], PlainOut{P.gate}, xb, ring, full, empty, r0, nr, gs, pair_base, mx, stop, warp,
                       lane);
    consumers_sync<kDecCW>();  // gate rows (any warp) before the up pass reads them
    consume_matrix<NH>(P, P.st[2], SiluMulOut{P.up, P.gate, P.act, amax_cta}, xb, ring, full, empty, r0, nr, gs,
                       pair_base, mx, stop, warp, lane);
    consumers_sync<kDecCW>();
    if (ctid == 0) atomicMax(P.amax, *amax_cta);
  }
  grid_barrier(P.bar_count, base, 2, ctid, P.status);

  // stage 4: h_out = h2 + W_d . q(act), scale from max|act| (atomics, read from L2)
  {
    float v[JI][8];
    const float amax = __uint_as_float(__ldcg(P.amax));
    load_groups<JI>(P.act, (int)(inter / 8), ctid, v);
    float unused[JI][8] = {};
    prep_groups<JI>((int)inter, kPrepAmaxGiven, v, unused, P.eps, amax, xb, P.q[3], P.scales + 3, red, ctid);
    rows_of(P.st[3], r0, nr);
    consume_matrix<NI>(P, P.st[3], ResidualOut{P.h_out, P.h2}, xb, ring, full, empty, r0, nr, gs, pair_base, mx,
                       stop, warp, lane);
  }
  if (__any_sync(0xffffffffu, W4A8Op<__half, NH, false>::bad(mx)) && lane == 0) set_status(P.status, kStatusBadScale);
}

// chunks per lane the kernel is instantiated for
int ncpl_for(int64_t cols) {
  const int64_t per_lane = (cols / 32 + 31) / 32;
  for (int n : {4, 8, 12, 16})
    if (per_lane <= n) return n;
  return 0;
}

template <int NH, int NI>
cudaError_t launch_persistent(const DecParams &P, size_t smem, cudaStream_t stream, int device, bool dry) {
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  static int fits[64];
  auto *kern = decode_layer_kernel<NH, NI>;
  std::call_once(once[device & 63], [&] {
    attr_err[device & 63] =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, device_props(device).smem_optin);
    int nb = 0;
    if (attr_err[device & 63] == cudaSuccess)
      attr_err[device & 63] = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kDecThreads,
                                                                             device_props(device).smem_optin);
    fits[device & 63] = nb;
  });
  if (attr_err[device & 63] != cudaSuccess) return attr_err[device & 63];
  if (fits[device & 63] < 1) return cudaErrorNotSupported;
  if (dry) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)device_props(device).sm_count);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, P);
}

}  // namespace

cudaError_t launch_decode_layer_persistent(const DecodeLayerArgs &a, cudaStream_t stream, int device, bool dry) {
  if (env_int("KS_B200_DECODE_PERSISTENT", 1) == 0) return cudaErrorNotSupported;
  const int64_t h = a.hidden, i = a.inter, G = a.group;
  const int NH = ncpl_for(h), NI = ncpl_for(i);
  if (!((NH == 4 && (NI == 12 || NI == 16)) || (NH == 8 && NI == 16))) return cudaErrorNotSupported;
  DecParams P{};
  const int64_t rows[4] = {3 * h, h, i, h}, cols[4] = {h, h, h, i};
  const int counts[4] = {1, 1, 2, 1};
  const int widx[4][2] = {{0, 0}, {1, 1}, {2, 3}, {4, 4}};
  int slot = 0, xbuf = 0;
  for (int s = 0; s < 4; ++s) {
    DecStage &S = P.st[s];
    S.count = counts[s];
    S.rows = (int32_t)rows[s];
    S.cols = (int32_t)cols[s];
    S.row_bytes = (int32_t)(cols[s] / 2);
    S.srow_bytes = (int32_t)(cols[s] / G * 2);
    if (S.row_bytes % 16 || S.srow_bytes % 16) return cudaErrorNotSupported;  // bulk-copy granularity
    for (int m = 0; m < 2; ++m) {
      S.w[m] = a.w[widx[s][m]];
      S.s[m] = static_cast<const uint8_t *>(a.s[widx[s][m]]);
      if ((reinterpret_cast<uintptr_t>(S.w[m]) | reinterpret_cast<uintptr_t>(S.s[m])) & 15u)
        return cudaErrorNotSupported;
    }
    const int rt = S.row_bytes + S.srow_bytes;
    const int target = std::max(8, env_int("KS_B200_DECODE_SLOT_KB", kDecSlotTarget / 1024)) * 1024;
    S.rps = std::max(2, (target / rt) & ~1);
    slot = std::max(slot, S.rps * rt);
    xbuf = std::max(xbuf, W4A8Op<__half, 4, false>::xbuf_bytes((int)(cols[s] / 32)));
  }
  if ((reinterpret_cast<uintptr_t>(a.h_in) | reinterpret_cast<uintptr_t>(a.norm1_w) |
       reinterpret_cast<uintptr_t>(a.norm2_w)) & 15u)
    return cudaErrorNotSupported;  // 16-byte vector loads of the inputs
  slot = (slot + 127) / 128 * 128;
  const DeviceProps &dp = device_props(device);
  const int nslots = std::min(kDecMaxSlots, (dp.smem_optin - kBarBytes - xbuf) / slot);
  if (nslots < 3) return cudaErrorNotSupported;
  P.nslots = nslots;
  P.slot_bytes = slot;
  P.xbuf_bytes = xbuf;
  int gshift = 0;
  while ((int64_t(32) << gshift) < G) ++gshift;
  P.gshift = gshift;
  P.inflight = std::max(0, std::min(env_int("KS_B200_DECODE_INFLIGHT", 0), nslots - 1));
  // off by default: measured slower (the prefetches queue ahead of the
  // grid barrier's and the input vector's latency-bound accesses)
  P.l2_ahead = std::max(0, env_int("KS_B200_DECODE_L2_AHEAD", 0));
  P.h_in = a.h_in;
  P.h_out = a.h_out;
  P.norm1_w = a.norm1_w;
  P.norm2_w = a.norm2_w;
  P.eps = a.eps;
  P.qkv = a.qkv;
  P.h2 = a.h2;
  P.gate = a.gate;
  P.up = a.up;
  P.act = a.act;
  P.scales = a.scales;
  P.amax = a.amax;
  P.bar_count = reinterpret_cast<unsigned long long *>(a.amax + 32);  // +128 bytes, same 256-byte region
  for (int k = 0; k < 4; ++k) P.q[k] = a.q[k];
  P.status = a.status;
  const size_t smem = (size_t)kBarBytes + xbuf + (size_t)nslots * slot;
  if (NH == 4 && NI == 12) return launch_persistent<4, 12>(P, smem, stream, device, dry);
  if (NH == 4 && NI == 16) return launch_persistent<4, 16>(P, smem, stream, device, dry);
  return launch_persistent<8, 16>(P, smem, stream, device, dry);
}

}  // namespace ksb
