// ks_decode.cu -- fused W4A8 decode layers (hidden h, intermediate i,
// batch 1) as ONE persistent kernel on B200 (sm_100a), up to 32 layers per
// launch.  Per layer:
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
// Why one kernel: a layer is a chain of four dependent GEMVs whose weights
// (114 MB for h = 4096, i = 11008) are the whole cost.  Launched one by one,
// each stage waits for the previous one to drain, then prepares its input,
// and HBM idles in between.  Here a cooperative grid of one CTA per SM runs
// all four stages of every layer of the launch:
//   * warp 16 (producer) streams this CTA's rows of all five matrices of
//     every layer, stage after stage and layer after layer, weights and f16
//     scale rows with cp.async.bulk (1-D, no tensor map, no multicast) into a
//     ring of ~64 KB slots.  Weights do not depend on the activations, so it
//     never waits for anything but a free slot and keeps HBM busy across the
//     stage and layer boundaries (layer l + 1's QKV rows stream while layer
//     l's down projection finishes).
//   * warps 0-15 (consumers), per stage: wait at a grid barrier for the
//     previous stage's outputs, prepare the input vector (RMSNorm /
//     quantisation, identical in every CTA; each thread holds its 8-element
//     groups in registers from one load to the quantised bytes), then take
//     pairs of rows from the ring and write the stage's outputs with its
//     epilogue.  Between layers a fourth grid barrier hands the layer's
//     output to the next layer's RMSNorm.  Only V (qkv[2h:3h]) feeds stage
//     2, so V's rows stream first; a CTA arrives at the barrier that
//     publishes V, then computes its Q rows, then waits -- and likewise
//     computes its K rows between arriving at and waiting for the barrier
//     that publishes h2: two of the four barriers per layer overlap rows
//     that nothing waits for.
// The ring (3 slots, ~195 KB per SM) holds about 4 us of HBM traffic; while
// it is full (the consumers held at a stage boundary) the producer brings the
// next three slots into L2, so HBM keeps streaming through the boundary.
// Layer g of a call reads the previous layer's output and writes hbuf[g & 1]
// (the last layer writes h_out); the intermediates (qkv, h2, gate, up, act)
// are reused by every layer, each written after the barrier that ends the
// previous layer's last read of it (Q and K are read by nothing; a CTA
// writes the same rows of them in every layer, in program order).
//
// Grid barrier: a 64-bit arrival counter in the workspace that only grows
// (see grid_barrier); every spin is bounded (about one second) and on a
// timeout the status word records it and the CTA goes on, so the kernel
// always terminates.  All CTAs are resident at once (cooperative launch), so
// no CTA waits for one that cannot run.
//
// Every read of an intermediate follows, through at least one grid barrier,
// the write it must see (and every rewrite by a later layer follows the last
// read of the previous value): the writers' CTA barrier and release
// arrival, then the reader's acquire at GPU scope and CTA barrier, order
// them for all threads of both CTAs, so plain loads see the current data;
// max|act| is updated with atomics in L2 and read with an L2 load.

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
constexpr int kDecMaxLayers = 32;          // layers per launch (the parameter block holds their pointers)

// One segment of a layer -- rows [row_off, row_off + rows) of the layer's
// matrix `mat` -- as both the producer and the consumers walk it (the same
// for every layer).  Segments in stream order: V, Q (W_qkv rows 2h.., 0..),
// O, K (W_qkv rows h..), gate, up, down.  V comes first because only V feeds
// the layer's next stage; each CTA computes its Q rows after arriving at the
// barrier that publishes V and its K rows after arriving at the one that
// publishes h2, so those barriers' latency is spent on rows nobody waits for.
constexpr int kSegs = 7;
enum Seg { kSegV, kSegQ, kSegO, kSegK, kSegGate, kSegUp, kSegDown };
struct DecStage {
  int32_t mat;                    // 0 qkv, 1 o, 2 gate, 3 up, 4 down
  int32_t row_off, rows, cols;
  int32_t row_bytes, srow_bytes;  // dense rows: the row strides
  int32_t rps;                    // rows per ring slot (even)
};

// One layer's operands: packed int4 weights and f16 scale rows of qkv, o,
// gate, up, down; the RMSNorm weight vectors.
struct DecLayer {
  const uint8_t *w[5];
  const uint8_t *s[5];
  const float *norm1_w, *norm2_w;
};

struct DecParams {
  DecStage st[kSegs];
  int32_t nslots, slot_bytes;
  int32_t xbuf_bytes;   // the first input buffer (h columns: the inputs of V, Q, K and of gate, up)
  int32_t xbuf2_bytes;  // the second (max(h, i) columns: the inputs of O and of down)
  int32_t gshift;    // log2(group / 32)
  int32_t inflight;  // slots issued and not yet landed, at most (0: up to the ring)
  int32_t l2_ahead;  // slots beyond the ring brought into L2 while the ring is full (0: none)
  int32_t layers;        // layers in this launch
  int32_t layer0;        // index of its first layer in the call
  int32_t total_layers;  // layers in the call
  // activations and workspace
  const float *h_in;  // input of the call's first layer
  float *h_out;       // output of the call's last layer
  float *hbuf[2];     // layer g (not the last) writes hbuf[g & 1]
  float eps;
  float *qkv, *h2, *gate, *up, *act, *scales;
  uint32_t *amax;
  unsigned long long *bar_count;  // 64-bit grid-barrier arrival counter
  int8_t *q[4];
  uint32_t *status;
  DecLayer layer[kDecMaxLayers];
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
// per barrier and, after its last barrier, the arrivals of the barriers its
// launch did not use, so every launch adds exactly kBarriers * grid.  At the
// start of a launch the counter holds kBarriers * grid * (launches so far)
// plus at most grid - 1 arrivals of this launch's first barrier; rounding
// down to a multiple of kBarriers * grid gives the launch's base, and
// barrier k is passed once the counter reaches base + (k + 1) * grid.  No
// reset, so the last arrival costs no extra round trip.
constexpr int kBarriers = 4 * kDecMaxLayers;

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

// Barrier k in two halves, every consumer thread of every CTA calling each,
// k = 0, 1, 2, ... in order: all of this CTA's consumer writes before
// grid_arrive(k) are visible to every consumer thread of the grid after
// grid_wait(k).  Work between the halves overlaps the barrier's latency.
// base: the launch's barrier base, in shared memory (read by thread 0 only).
__device__ void grid_arrive(unsigned long long *count, int ctid) {
  consumers_sync<kDecCW>();
  if (ctid == 0) {
    // release: this CTA's writes (ordered before it by the CTA barrier) are
    // visible to whoever acquires a count that includes this arrival
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(count) : "memory");
  }
}
__device__ void grid_wait(unsigned long long *count, const uint64_t *base, int k, int ctid, uint32_t *status) {
  if (ctid == 0) {
    const uint64_t target = *base + (uint64_t)(k + 1) * gridDim.x;
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
__device__ void grid_barrier(unsigned long long *count, const uint64_t *base, int k, int ctid, uint32_t *status) {
  grid_arrive(count, ctid);
  grid_wait(count, base, k, ctid, status);
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

// Sum / max over the consumer threads in a fixed order (bitwise the same in
// every CTA) with one CTA barrier each: the two reductions of a preparation
// use their own word arrays, and the preparation's closing barrier orders
// every read of them before the next preparation writes them again.
__device__ __forceinline__ float prep_sum(float v, float *red, int ctid) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((ctid & 31) == 0) red[ctid >> 5] = v;
  consumers_sync<kDecCW>();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kDecCW; ++w) t += red[w];
  return t;
}
__device__ __forceinline__ float prep_max(float v, float *red, int ctid) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((ctid & 31) == 0) red[ctid >> 5] = v;
  consumers_sync<kDecCW>();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kDecCW; ++w) t = fmaxf(t, red[w]);
  return t;
}

enum PrepMode { kPrepPlain, kPrepRms, kPrepAmaxGiven };

// v: the thread's groups (loaded); nw: RMSNorm weights of the same groups
// (read only in kPrepRms mode).
template <int J, int MODE, int JW>
__device__ __forceinline__ void prep_groups(int K, float (&v)[J][8], const float (&nw)[JW][8], float eps,
                                            float amax_given, uint8_t *xb, int8_t *xq_out, float *xs_out, float *red,
                                            int ctid) {
  static_assert(MODE != kPrepRms || JW == J, "RMSNorm weights for every group");
  const int ngroups = K / 8, chunks = K / 32;
  if constexpr (MODE == kPrepRms) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) ss = __fadd_rn(ss, __fmul_rn(v[j][t], v[j][t]));
    ss = prep_sum(ss, red, ctid);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) v[j][t] = __fmul_rn(__fmul_rn(v[j][t], scale), nw[j][t]);
  }
  float amax;
  if constexpr (MODE == kPrepAmaxGiven) {
    amax = amax_given;
  } else {
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) m = fmaxf(m, fabsf(v[j][t]));
    amax = prep_max(m, red + kDecCW, ctid);
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

// ---- ring position, kept incrementally (no division per slot) --------------
struct RingPos {
  int b = 0;           // slot
  uint32_t phase = 0;  // parity of the slot's current use
  __device__ __forceinline__ void next(int nslots) {
    if (++b == nslots) {
      b = 0;
      phase ^= 1u;
    }
  }
};

// This CTA's rows of one stage, computed once per launch (shared memory):
// a contiguous block balanced to one row, and its ring slots.
struct StageRows {
  int r0, n, nblk;
};

// ---- consumers: one matrix of one stage -------------------------------------
template <int NCPL, class Out>
__device__ __forceinline__ void consume_matrix(const DecStage &S, const StageRows &G, const Out &out,
                                               const uint8_t *xb, int gshift, const uint8_t *ring, int slot_bytes,
                                               int nslots, uint64_t *full, uint64_t *empty, RingPos &rp,
                                               int &pair_base, uint32_t &mx, bool &stop, int warp, int lane,
                                               uint32_t *status) {
  using Op = W4A8Op<__half, NCPL, false>;
  const W4A8OpParams op{S.cols / 32, gshift, 1.0f, 0, 0};
  typename Op::Lane L;
  Op::lane_init(op, L, xb, lane);
  const GemvItem none{};
  for (int st = 0, lo = 0; st < G.nblk; ++st, lo += S.rps, rp.next(nslots)) {
    if (stop) continue;  // keeps the ring position in step with the producer
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[rp.b], rp.phase));
    if (!ok) {
      if (lane == 0) set_status(status, kStatusTimeout);
      stop = true;
      continue;
    }
    const int hi = min(lo + S.rps, G.n);
    const uint8_t *base = ring + (size_t)rp.b * slot_bytes;
    const uint8_t *sbase = base + (size_t)S.rps * S.row_bytes;
    // row pairs (lo + 2q, lo + 2q + 1); the pair's running index picks the
    // warp, so consecutive slots start on different warps
    const int pair0 = pair_base + (lo >> 1);  // rps is even
    for (int q = (warp - pair0) & (kDecCW - 1); lo + 2 * q < hi; q += kDecCW) {
      const int li = 2 * q;
      mx = max(mx, Op::rows2(op, L, xb, base + (size_t)li * S.row_bytes, sbase + (size_t)li * S.srow_bytes,
                             base + (size_t)(li + 1) * S.row_bytes, sbase + (size_t)(li + 1) * S.srow_bytes, out,
                             none, (int64_t)G.r0 + lo + li, lo + li + 1 < hi, lane, L));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[rp.b]);
  }
  pair_base += (G.n + 1) >> 1;
}

// NH, NI: 32-element chunks per lane for rows of h and of i columns.
template <int NH, int NI>
__global__ void __launch_bounds__(kDecThreads, 1) decode_layer_kernel(const __grid_constant__ DecParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + P.nslots;
  float *red = reinterpret_cast<float *>(smem + kBarBytes - 128);  // 2 x kDecCW floats (sum, max)
  uint32_t *amax_cta = reinterpret_cast<uint32_t *>(smem + kBarBytes - 192);  // this CTA's max|act| bits
  uint64_t *bar_base = reinterpret_cast<uint64_t *>(smem + kBarBytes - 256);  // the launch's barrier base
  StageRows *geo = reinterpret_cast<StageRows *>(smem + kBarBytes - 512);  // kSegs segments
  uint8_t *xb = smem + kBarBytes;      // inputs of V, Q, K; of gate, up
  uint8_t *xb2 = xb + P.xbuf_bytes;    // inputs of O; of down
  uint8_t *ring = xb2 + P.xbuf2_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < P.nslots; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], kDecCW);
    }
    for (int s = 0; s < kSegs; ++s) {
      const DecStage &S = P.st[s];
      const int r0 = (int)((int64_t)blockIdx.x * S.rows / gridDim.x);
      const int r1 = (int)((int64_t)(blockIdx.x + 1) * S.rows / gridDim.x);
      geo[s] = StageRows{r0, r1 - r0, (r1 - r0 + S.rps - 1) / S.rps};
    }
    *amax_cta = 0u;
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == kDecCW) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      RingPos rp, landed;  // next slot to fill; oldest slot that may still be in flight
      int issued = 0, waited = 0;
      bool stop = false;
      // While the ring is full (the consumers held at a stage boundary), the
      // next l2_ahead slots are prefetched into L2, so HBM keeps streaming
      // through the boundary and the ring refills from L2 after it.  pf
      // counts the slots prefetched or issued; (pl, ps, plo) is slot pf.
      int pf = 0, pl = 0, ps = 0, plo = 0;
      auto pf_skip_empty = [&]() {
        while (pl < P.layers && geo[ps].n == 0) {
          if (++ps == kSegs) {
            ps = 0;
            ++pl;
          }
        }
      };
      auto pf_advance = [&]() {
        plo += P.st[ps].rps;
        if (plo >= geo[ps].n) {
          plo = 0;
          if (++ps == kSegs) {
            ps = 0;
            ++pl;
          }
          pf_skip_empty();
        }
        ++pf;
      };
      pf_skip_empty();
      for (int l = 0; l < P.layers && !stop; ++l) {
        const DecLayer &Ly = P.layer[l];
        for (int s = 0; s < kSegs && !stop; ++s) {
          const DecStage &S = P.st[s];
          const StageRows G = geo[s];
          {
            const uint8_t *wm = Ly.w[S.mat] + (int64_t)(S.row_off + G.r0) * S.row_bytes;
            const uint8_t *sm = Ly.s[S.mat] + (int64_t)(S.row_off + G.r0) * S.srow_bytes;
            for (int lo = 0; lo < G.n; lo += S.rps, ++issued, rp.next(P.nslots)) {
              if (P.l2_ahead > 0 && issued >= P.nslots && !mbar_try_wait(&empty[rp.b], rp.phase ^ 1u)) {
                if (pf < issued) {  // catch the prefetch cursor up with this slot
                  pl = l;
                  ps = s;
                  plo = lo;
                  pf = issued;
                }
                for (; pf < issued + P.l2_ahead && pl < P.layers; pf_advance()) {
                  const DecStage &T = P.st[ps];
                  const int n = min(T.rps, geo[ps].n - plo);
                  const int64_t row = T.row_off + geo[ps].r0 + plo;
                  bulk_prefetch_l2(P.layer[pl].w[T.mat] + row * T.row_bytes, (uint32_t)n * (uint32_t)T.row_bytes);
                  bulk_prefetch_l2(P.layer[pl].s[T.mat] + row * T.srow_bytes, (uint32_t)n * (uint32_t)T.srow_bytes);
                }
              }
              if (issued >= P.nslots && !mbar_wait(&empty[rp.b], rp.phase ^ 1u)) {
                set_status(P.status, kStatusTimeout);
                stop = true;
                break;
              }
              // at most `inflight` slots issued and not yet landed: a shorter
              // memory queue keeps the barrier's and the input loads' latency low
              for (; P.inflight > 0 && issued - waited >= P.inflight; ++waited, landed.next(P.nslots)) {
                if (!mbar_wait(&full[landed.b], landed.phase)) {
                  set_status(P.status, kStatusTimeout);
                  stop = true;
                  break;
                }
              }
              if (stop) break;
              const int n = min(S.rps, G.n - lo);
              const uint32_t wbytes = (uint32_t)n * (uint32_t)S.row_bytes;
              const uint32_t sbytes = (uint32_t)n * (uint32_t)S.srow_bytes;
              uint8_t *dst = ring + (size_t)rp.b * P.slot_bytes;
              mbar_arrive_expect_tx(&full[rp.b], wbytes + sbytes);
              bulk_g2s_hint(dst, wm + (int64_t)lo * S.row_bytes, wbytes, &full[rp.b], pol);
              bulk_g2s(dst + (size_t)S.rps * S.row_bytes, sm + (int64_t)lo * S.srow_bytes, sbytes, &full[rp.b]);
            }
          }
        }
      }
      // every copy issued must land before the CTA may exit: the last
      // min(issued, nslots) slots (the earlier ones were consumed)
      for (; waited < issued - P.nslots; ++waited) landed.next(P.nslots);
      for (; waited < issued; ++waited, landed.next(P.nslots))
        if (!mbar_wait(&full[landed.b], landed.phase)) set_status(P.status, kStatusTimeout);
    }
    return;
  }

  // ------------------------------------------------------------- consumers --
  constexpr int JH = NH / 4, JI = NI / 4;  // 8-element groups per thread (NT = 512)
  const int ctid = threadIdx.x;
  const int64_t h = P.st[kSegO].rows, inter = P.st[kSegGate].rows;
  RingPos rp;
  int pair_base = 0, bk = 0;
  uint32_t mx = 0;
  bool stop = false;
  if (ctid == 0) *bar_base = barrier_base(P.bar_count);
  // RMSNorm weights of this thread's groups for the next RMSNorm (stage 1
  // or 3): each vector is loaded before the grid barrier that precedes its
  // stage, since it does not depend on it, and only one is held at a time
  float nw[JH][8];
  load_groups<JH>(P.layer[0].norm1_w, (int)(h / 8), ctid, nw);

  for (int l = 0; l < P.layers; ++l) {
    // this layer's input and output vectors, computed where used (fewer live registers)
    auto h_in = [&]() -> const float * {
      const int g = P.layer0 + l;
      return g == 0 ? P.h_in : P.hbuf[(g - 1) & 1];
    };
    auto h_out = [&]() -> float * {
      const int g = P.layer0 + l;
      return g == P.total_layers - 1 ? P.h_out : P.hbuf[g & 1];
    };
    // V, then Q: x1 = q(RMSNorm(h_in, norm1)) in xb.  The barrier that
    // publishes V is arrived at before Q and waited for after it.
    if (blockIdx.x == 0 && ctid == 0) atomicExch(P.amax, 0u);
    {
      float v[JH][8];
      load_groups<JH>(h_in(), (int)(h / 8), ctid, v);
      prep_groups<JH, kPrepRms>((int)h, v, nw, P.eps, 0.0f, xb, P.q[0], P.scales + 0, red, ctid);
    }
    consume_matrix<NH>(P.st[kSegV], geo[kSegV], PlainOut{P.qkv + 2 * h}, xb, P.gshift, ring, P.slot_bytes, P.nslots,
                       full, empty, rp, pair_base, mx, stop, warp, lane, P.status);
    grid_arrive(P.bar_count, ctid);
    consume_matrix<NH>(P.st[kSegQ], geo[kSegQ], PlainOut{P.qkv}, xb, P.gshift, ring, P.slot_bytes, P.nslots, full,
                       empty, rp, pair_base, mx, stop, warp, lane, P.status);
    grid_wait(P.bar_count, bar_base, bk++, ctid, P.status);

    // O: h2 = h_in + W_o . q(V), its input in xb2; then K on x1 (still in xb)
    // between arriving at the barrier that publishes h2 and waiting for it
    {
      float v[JH][8];
      load_groups<JH>(P.qkv + 2 * h, (int)(h / 8), ctid, v);
      prep_groups<JH, kPrepPlain>((int)h, v, nw, P.eps, 0.0f, xb2, P.q[1], P.scales + 1, red, ctid);
      consume_matrix<NH>(P.st[kSegO], geo[kSegO], ResidualOut{P.h2, h_in()}, xb2, P.gshift, ring, P.slot_bytes,
                         P.nslots, full, empty, rp, pair_base, mx, stop, warp, lane, P.status);
    }
    load_groups<JH>(P.layer[l].norm2_w, (int)(h / 8), ctid, nw);
    grid_arrive(P.bar_count, ctid);
    consume_matrix<NH>(P.st[kSegK], geo[kSegK], PlainOut{P.qkv + h}, xb, P.gshift, ring, P.slot_bytes, P.nslots,
                       full, empty, rp, pair_base, mx, stop, warp, lane, P.status);
    grid_wait(P.bar_count, bar_base, bk++, ctid, P.status);  // also: every warp is done with x1

    // gate, up = W_g, W_u . q(RMSNorm(h2, norm2)) (input in xb); act = silu(gate) * up
    {
      float v[JH][8];
      load_groups<JH>(P.h2, (int)(h / 8), ctid, v);
      prep_groups<JH, kPrepRms>((int)h, v, nw, P.eps, 0.0f, xb, P.q[2], P.scales + 2, red, ctid);
      consume_matrix<NH>(P.st[kSegGate], geo[kSegGate], PlainOut{P.gate}, xb, P.gshift, ring, P.slot_bytes,
                         P.nslots, full, empty, rp, pair_base, mx, stop, warp, lane, P.status);
      consumers_sync<kDecCW>();  // gate rows (any warp) before the up pass reads them
      consume_matrix<NH>(P.st[kSegUp], geo[kSegUp], SiluMulOut{P.up, P.gate, P.act, amax_cta}, xb, P.gshift, ring,
                         P.slot_bytes, P.nslots, full, empty, rp, pair_base, mx, stop, warp, lane, P.status);
      consumers_sync<kDecCW>();
      if (ctid == 0) {
        atomicMax(P.amax, *amax_cta);
        *amax_cta = 0u;  // the next layer's gate/up starts from zero
      }
    }
    grid_barrier(P.bar_count, bar_base, bk++, ctid, P.status);

    // down: h_out = h2 + W_d . q(act), scale from max|act| (atomics, read from L2), input in xb2
    {
      float v[JI][8];
      const float amax = __uint_as_float(__ldcg(P.amax));
      load_groups<JI>(P.act, (int)(inter / 8), ctid, v);
      prep_groups<JI, kPrepAmaxGiven>((int)inter, v, nw, P.eps, amax, xb2, P.q[3], P.scales + 3, red, ctid);
      consume_matrix<NI>(P.st[kSegDown], geo[kSegDown], ResidualOut{h_out(), P.h2}, xb2, P.gshift, ring,
                         P.slot_bytes, P.nslots, full, empty, rp, pair_base, mx, stop, warp, lane, P.status);
    }
    if (l + 1 < P.layers) {
      load_groups<JH>(P.layer[l + 1].norm1_w, (int)(h / 8), ctid, nw);
      grid_barrier(P.bar_count, bar_base, bk++, ctid, P.status);  // h_out before the next layer's RMSNorm
    }
  }
  // every launch adds kBarriers arrivals per CTA: the ones this launch did not use
  if (ctid == 0 && bk < kBarriers)
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(P.bar_count), "l"((uint64_t)(kBarriers - bk))
                 : "memory");
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

cudaError_t launch_decode_layers_persistent(const DecodeLayersArgs &a, cudaStream_t stream, int device, bool dry) {
  if (env_int("KS_B200_DECODE_PERSISTENT", 1) == 0) return cudaErrorNotSupported;
  if (a.layers < 1) return cudaErrorInvalidValue;
  const int64_t h = a.hidden, i = a.inter, G = a.group;
  const int NH = ncpl_for(h), NI = ncpl_for(i);
  if (!((NH == 4 && (NI == 12 || NI == 16)) || (NH == 8 && NI == 16))) return cudaErrorNotSupported;
  DecParams P{};
  // segments V, Q, O, K, gate, up, down: matrix, first row, rows, columns
  const int mats[kSegs] = {0, 0, 1, 0, 2, 3, 4};
  const int64_t offs[kSegs] = {2 * h, 0, 0, h, 0, 0, 0};
  const int64_t rows[kSegs] = {h, h, h, h, i, i, h}, cols[kSegs] = {h, h, h, h, h, h, i};
  const int target = std::max(8, env_int("KS_B200_DECODE_SLOT_KB", kDecSlotTarget / 1024)) * 1024;
  int slot = 0, xbuf2 = 0;
  const int xbuf = W4A8Op<__half, 4, false>::xbuf_bytes((int)(h / 32));
  for (int s = 0; s < kSegs; ++s) {
    DecStage &S = P.st[s];
    S.mat = mats[s];
    S.row_off = (int32_t)offs[s];
    S.rows = (int32_t)rows[s];
    S.cols = (int32_t)cols[s];
    S.row_bytes = (int32_t)(cols[s] / 2);
    S.srow_bytes = (int32_t)(cols[s] / G * 2);
    if (S.row_bytes % 16 || S.srow_bytes % 16) return cudaErrorNotSupported;  // bulk-copy granularity
    const int rt = S.row_bytes + S.srow_bytes;
    S.rps = std::max(2, (target / rt) & ~1);
    slot = std::max(slot, S.rps * rt);
    xbuf2 = std::max(xbuf2, W4A8Op<__half, 4, false>::xbuf_bytes((int)(cols[s] / 32)));
  }
  // 16-byte vector loads of the inputs, 16-byte bulk copies of the weights
  uintptr_t al = reinterpret_cast<uintptr_t>(a.h_in);
  for (int l = 0; l < a.layers; ++l) {
    const DecodeLayerWeights &lw = a.lw[l];
    al |= reinterpret_cast<uintptr_t>(lw.norm1_w) | reinterpret_cast<uintptr_t>(lw.norm2_w);
    for (int k = 0; k < 5; ++k) al |= reinterpret_cast<uintptr_t>(lw.w[k]) | reinterpret_cast<uintptr_t>(lw.s[k]);
  }
  if (al & 15u) return cudaErrorNotSupported;
  slot = (slot + 127) / 128 * 128;
  const DeviceProps &dp = device_props(device);
  const int nslots = std::min(kDecMaxSlots, (dp.smem_optin - kBarBytes - xbuf - xbuf2) / slot);
  if (nslots < 3) return cudaErrorNotSupported;
  P.nslots = nslots;
  P.slot_bytes = slot;
  P.xbuf_bytes = xbuf;
  P.xbuf2_bytes = xbuf2;
  int gshift = 0;
  while ((int64_t(32) << gshift) < G) ++gshift;
  P.gshift = gshift;
  P.inflight = std::max(0, std::min(env_int("KS_B200_DECODE_INFLIGHT", 0), nslots - 1));
  // measured on B200 (hidden 4096, inter 11008, 32 layers per launch), us per
  // layer: 0 slots 32.36, 1 31.21, 2 30.69, 3 30.49, 4 31.12, 6 31.39, 12 32.94,
  // 24 38.46 (farther prefetches crowd out the ring's own copies)
  P.l2_ahead = std::max(0, std::min(env_int("KS_B200_DECODE_L2_AHEAD", 3), 64));
  P.total_layers = a.layers;
  P.h_in = a.h_in;
  P.h_out = a.h_out;
  P.hbuf[0] = a.hbuf[0];
  P.hbuf[1] = a.hbuf[1];
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
  const size_t smem = (size_t)kBarBytes + xbuf + xbuf2 + (size_t)nslots * slot;
  for (int l0 = 0; l0 < a.layers; l0 += kDecMaxLayers) {
    P.layer0 = l0;
    P.layers = std::min(kDecMaxLayers, a.layers - l0);
    for (int l = 0; l < P.layers; ++l) {
      const DecodeLayerWeights &lw = a.lw[l0 + l];
      for (int k = 0; k < 5; ++k) {
        P.layer[l].w[k] = lw.w[k];
        P.layer[l].s[k] = static_cast<const uint8_t *>(lw.s[k]);
      }
      P.layer[l].norm1_w = lw.norm1_w;
      P.layer[l].norm2_w = lw.norm2_w;
    }
    cudaError_t e;
    if (NH == 4 && NI == 12)
      e = launch_persistent<4, 12>(P, smem, stream, device, dry);
    else if (NH == 4 && NI == 16)
      e = launch_persistent<4, 16>(P, smem, stream, device, dry);
    else
      e = launch_persistent<8, 16>(P, smem, stream, device, dry);
    if (e != cudaSuccess || dry) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_decode_layers_w4a8(const DecodeLayersArgs &a, cudaStream_t stream, int device) {
  {
    const cudaError_t e = launch_decode_layers_persistent(a, stream, device);
    if (e == cudaSuccess) return e;
    if (e != cudaErrorNotSupported && e != cudaErrorCooperativeLaunchTooLarge) return e;
    cudaGetLastError();  // not a sticky error: take four launches per layer below
  }
  for (int l = 0; l < a.layers; ++l) {
    const DecodeLayerWeights &lw = a.lw[l];
    DecodeLayerArgs d{};
    d.h_in = l == 0 ? a.h_in : a.hbuf[(l - 1) & 1];
    d.h_out = l == a.layers - 1 ? a.h_out : a.hbuf[l & 1];
    d.norm1_w = lw.norm1_w;
    d.norm2_w = lw.norm2_w;
    d.eps = a.eps;
    for (int k = 0; k < 5; ++k) {
      d.w[k] = lw.w[k];
      d.s[k] = lw.s[k];
    }
    d.hidden = a.hidden;
    d.inter = a.inter;
    d.group = a.group;
    d.qkv = a.qkv;
    d.h2 = a.h2;
    d.gate = a.gate;
    d.up = a.up;
    d.act = a.act;
    d.scales = a.scales;
    d.amax = a.amax;
    for (int k = 0; k < 4; ++k) d.q[k] = a.q[k];
    d.status = a.status;
    const cudaError_t e = launch_decode_layer_four(d, stream, device);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ksb
