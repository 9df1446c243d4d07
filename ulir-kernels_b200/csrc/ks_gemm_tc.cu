// ks_gemm_tc.cu -- skinny INT8 GEMM with requantisation on 5th-generation
// tensor cores (tcgen05.mma kind::i8, accumulators in TMEM), sm_100a.
//
//   out[m, n] = sat_i8(rne(((f32(acc[m, n]) * a_scale[m]) * w_scale[n]) / out_scale))
//   acc[m, n] = sum_k A[m, k] * W[n, k]          (int32, exact)
//
// A is [M, K] int8 activations (M = 8..256 decode tokens), W is [N, K] int8
// weights in the GEMV layout (row-major, K contiguous).  The contraction is
// "swap-AB": weight rows fill the MMA's 128-row M dimension and the tokens
// its N dimension (padded to a multiple of 16), so a [128 x Mpad] int32 tile
// lives in TMEM while all of K streams through shared memory.
//
// Every SM gets the same share of weight rows: a CTA owns `tile_rows` =
// ceil(N / (waves * SMs * ctas_per_SM)) consecutive rows (at most 128; the
// TMA box height), so the weight stream -- the bound at M <= 64 -- is spread
// over all SMs instead of over ceil(N / 128) CTAs.  The MMA is always
// M = 128; accumulator lanes at and above tile_rows belong to no weight row
// of the CTA and are never stored.
//
// Warp-specialised CTA of 192 threads:
//   warp 0  TMA producer: per 128-byte K block, one 2-D tiled copy of the
//           weight tile [tile_rows x 128 B] and one of the activation tile
//           [Mpad x 128 B], both 128-byte swizzled, into a ring of stages of
//           up to four K blocks each (one barrier pair and one commit per
//           stage: each producer -> MMA -> commit -> producer round trip costs
//           a few hundred cycles of the MMA thread's time, so a stage carries
//           16 MMAs rather than 4).
//           The weight copies of the first stages are issued before
//           griddepcontrol.wait (weights are never written by the kernels of
//           this library that trigger an early launch); the activations only
//           after it.  No multicast anywhere.
//   warp 1  allocates TMEM, issues 4 x tcgen05.mma (K = 32 each) per K block,
//           frees the stage with tcgen05.commit, finally commits to the
//           accumulator barrier; deallocates TMEM at the end.
//   warps 2-5 epilogue: after griddepcontrol.wait, stage the per-token
//           activation scales in shared memory and the row's weight scale in
//           a register while the main loop runs; then tcgen05.ld the
//           accumulator rows (one TMEM lane per weight row), requantise in the
//           order written above with IEEE round-to-nearest operations and
//           store int8.
//
// Every mbarrier wait is bounded (about one second); on a timeout the kernel
// records it in the status word, lets in-flight copies and MMAs drain, frees
// TMEM and returns.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "ks_internal.h"
#include "ks_ptx.cuh"
#include "ks_tc.cuh"

namespace ksb {

namespace {

constexpr int kMmaRows = 128;    // MMA M = TMEM lanes; a CTA stores its first tile_rows
constexpr int kKBlock = 128;     // K bytes per stage (one 128-B swizzle row)
constexpr int kGemmThreads = 192;
constexpr int kEpiThreads = 128;  // warps 2-5
constexpr int kMaxTokens = 256;  // MMA N limit
constexpr int kMaxStages = 12;
constexpr int kWTileBytes = kMmaRows * kKBlock;  // weight region of a stage (MMA reads 128 rows)
constexpr int kBarRegion = 1024;                 // barriers, TMEM slot, abort flag
constexpr int kScaleRegion = kMaxTokens * 4;     // activation scales

// A stage holds `bps` consecutive K blocks: their weight tiles first (one
// 16 KB MMA-A region each), then their activation tiles.  More blocks per
// stage means fewer mbarrier round trips (TMA -> MMA -> commit -> producer)
// per MMA; each round trip, not the MMA instruction, paces a skinny GEMM.
__device__ __forceinline__ uint8_t *stage_w(uint8_t *st, int j) { return st + (size_t)j * kWTileBytes; }
__device__ __forceinline__ uint8_t *stage_a(uint8_t *st, int bps, int b_bytes, int j) {
  return st + (size_t)bps * kWTileBytes + (size_t)j * b_bytes;
}

struct GemmParams {
  const float *sa;
  const float *ws;
  float out_scale;
  float inv_out_scale;  // RN(1 / out_scale), or 0 when that is not finite (then divide)
  int8_t *out;
  int64_t ldo;
  int32_t *acc_out;  // optional
  int32_t m, n, k;
  int32_t mpad;       // tokens padded to a multiple of 16
  int32_t nkb;        // K blocks of 128
  int32_t bps;        // K blocks per stage (one barrier pair and one commit per stage)
  int32_t nks;        // stages per GEMM: nkb / bps, rounded up
  int32_t nst;        // ring stages
  int32_t stage_bytes;
  int32_t b_bytes;    // activation tile bytes per K block
  int32_t tile_rows;  // weight rows per CTA (TMA box height, multiple of 16, <= 128)
  int32_t tma_store;  // 1: the int8 tile leaves through one TMA store (aligned out, ldo)
  uint32_t tmem_cols;
  uint32_t *status;
};

__device__ __forceinline__ void epi_barrier() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }
// AND of `pred` over the epilogue warps (named barrier 1): every epilogue
// thread takes the same branch after it, so none can miss a later barrier.
__device__ __forceinline__ bool epi_all(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kEpiThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ int8_t requant(int32_t acc, float sa, float ws, float out_scale) {
  float t = __fmul_rn((float)acc, sa);
  t = __fmul_rn(t, ws);
  t = __fdiv_rn(t, out_scale);
  t = rintf(t);  // round half to even
  t = fminf(fmaxf(t, -128.0f), 127.0f);
  return (int8_t)(int)t;
}

// Sixteen requant() results without a division per element and without a
// branch per element, so the sixteen chains overlap.  inv = RN(1/out_scale)
// (finite).  q = RN(t * inv) and the correctly rounded quotient RN(t/out_scale)
// both lie within |t/out_scale| * 2^-23 of the exact quotient (two and one
// half-ulp errors), i.e. within 3.1e-5 while |q| < 129; rint() can tell them
// apart only across a half-integer.  q is clamped to [-129, 128] (fmaxf maps
// NaN to -129, like fmaxf(NaN, -128) in requant()); y = RN(q + 1.5 * 2^23)
// holds rint(q) (ties to even) in its low mantissa bits, r = y - 1.5 * 2^23 is
// the same integer as a float, and |q - r| within 2^-14 of 0.5 marks a
// near-tie.  Only near-ties (rare; one warp-uniform test per 16) divide.
__device__ __forceinline__ void requant16(const uint32_t (&v)[16], const float *sv, float ws, float out_scale,
                                          float inv, int (&o)[16]) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr int kMagicBits = 0x4B400000;
  float t[16];
  uint32_t near = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    t[j] = __fmul_rn(__fmul_rn((float)(int32_t)v[j], sv[j]), ws);
    const float q = fminf(fmaxf(__fmul_rn(t[j], inv), -129.0f), 128.0f);
    const float y = __fadd_rn(q, kMagic);
    const float r = __fsub_rn(y, kMagic);
    near |= (__fsub_rn(0.5f, fabsf(__fsub_rn(q, r))) < 0x1p-14f ? 1u : 0u) << j;
    o[j] = __float_as_int(y) - kMagicBits;
  }
  if (__any_sync(0xffffffffu, near != 0)) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if ((near >> j) & 1u) {
        float e = rintf(__fdiv_rn(t[j], out_scale));
        o[j] = (int)fminf(fmaxf(e, -128.0f), 127.0f);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j] = min(max(o[j], -128), 127);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stages = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)p.nst * p.stage_bytes);
  uint64_t *empty = full + p.nst;
  uint64_t *accum = empty + p.nst;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  float *sa_s = reinterpret_cast<float *>(smem + (size_t)p.nst * p.stage_bytes + kBarRegion);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * p.tile_rows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_a);
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t tx_block = (uint32_t)(p.tile_rows * kKBlock + p.b_bytes);
      const int pre = min(p.nst, p.nks);
      // weights of the first stages, before the previous grid has finished
      for (int ks = 0; ks < pre; ++ks) {
        const int nb = min(p.bps, p.nkb - ks * p.bps);
        uint8_t *st = stages + (size_t)ks * p.stage_bytes;
        mbar_arrive_expect_tx(&full[ks], (uint32_t)nb * tx_block);
        for (int j = 0; j < nb; ++j)
          tma_load_2d_hint(stage_w(st, j), &tmap_w, (ks * p.bps + j) * kKBlock, row0, &full[ks], pol);
      }
      pdl_wait();
      pdl_trigger();
      for (int ks = 0; ks < pre; ++ks) {
        const int nb = min(p.bps, p.nkb - ks * p.bps);
        uint8_t *st = stages + (size_t)ks * p.stage_bytes;
        for (int j = 0; j < nb; ++j)
          tma_load_2d(stage_a(st, p.bps, p.b_bytes, j), &tmap_a, (ks * p.bps + j) * kKBlock, 0, &full[ks]);
      }
      int issued = pre;
      for (int ks = pre; ks < p.nks; ++ks) {
        const int s = ks % p.nst;
        if (!mbar_wait(&empty[s], (uint32_t)((ks / p.nst) - 1) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        const int nb = min(p.bps, p.nkb - ks * p.bps);
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)nb * tx_block);
        for (int j = 0; j < nb; ++j) {
          tma_load_2d_hint(stage_w(st, j), &tmap_w, (ks * p.bps + j) * kKBlock, row0, &full[s], pol);
          tma_load_2d(stage_a(st, p.bps, p.b_bytes, j), &tmap_a, (ks * p.bps + j) * kKBlock, 0, &full[s]);
        }
        ++issued;
      }
      for (int ks = max(0, issued - p.nst); ks < issued; ++ks) {
        if (!mbar_wait(&full[ks % p.nst], (uint32_t)(ks / p.nst) & 1u)) set_status(p.status, kStatusTimeout);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = (2u << 4)                         // D: s32
                             | (1u << 7) | (1u << 10)          // A, B: signed int8
                             | ((uint32_t)(p.mpad >> 3) << 17) // N
                             | ((uint32_t)(kMmaRows >> 4) << 24);  // M
      for (int ks = 0; ks < p.nks; ++ks) {
        const int s = ks % p.nst;
        if (!mbar_wait(&full[s], (uint32_t)(ks / p.nst) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        const int nb = min(p.bps, p.nkb - ks * p.bps);
        for (int j = 0; j < nb; ++j) {
          const uint64_t adesc = umma_desc_sw128(stage_w(st, j));
          const uint64_t bdesc = umma_desc_sw128(stage_a(st, p.bps, p.b_bytes, j));
#pragma unroll
          for (int kk = 0; kk < kKBlock / 32; ++kk) {
            // advance the start address by 32 bytes (K = 32 int8) per step
            tc_mma_i8(tmem_d, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                      (ks > 0 || j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc_commit(&empty[s]);
      }
      tc_commit(accum);  // fires once every MMA issued above has completed
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int et = threadIdx.x - 64;  // 0..127
    const int quarter = warp & 3;     // TMEM lanes 32*quarter .. +31
    const int r = quarter * 32 + lane;
    const int n = row0 + r;
    const bool row_ok = r < p.tile_rows && n < p.n;
    // Scales may come from the previous grid; `out` may still be read by it.
    pdl_wait();
    const float *__restrict__ sa = p.sa;
    for (int m = et; m < p.mpad; m += kEpiThreads) sa_s[m] = m < p.m ? sa[m] : 0.0f;
    const float wsn = row_ok ? p.ws[n] : 0.0f;
    epi_barrier();
    const bool ok = epi_all(mbar_wait(accum, 0));
    tc_fence_after();
    const bool aborted = !epi_all(*abort_flag == 0);
    if (!ok) {
      if (et == 0) set_status(p.status, kStatusTimeout);
    } else if (!aborted) {
      int8_t *__restrict__ out = p.out;
      int32_t *__restrict__ acc_out = p.acc_out;
      // int8 tile [mpad][tile_rows] for the TMA store, in the stage ring: every
      // copy into it has landed and every MMA reading it has completed.
      int8_t *tile = reinterpret_cast<int8_t *>(stages);
      const bool via_tma = p.tma_store != 0;
      const uint32_t taddr = tmem_d + ((uint32_t)(quarter * 32) << 16);
      for (int c0 = 0; c0 < p.mpad; c0 += 32) {
        const bool two = c0 + 16 < p.mpad;  // uniform across the CTA
        uint32_t va[16], vb[16];
        tc_ld16_nowait(taddr + (uint32_t)c0, va);
        if (two) tc_ld16_nowait(taddr + (uint32_t)(c0 + 16), vb);
        tc_wait_ld(va, vb);
        int oa[16], ob[16];
        requant16(va, sa_s + c0, wsn, p.out_scale, p.inv_out_scale, oa);
        if (two) requant16(vb, sa_s + c0 + 16, wsn, p.out_scale, p.inv_out_scale, ob);
        for (int h = 0; h < (two ? 2 : 1); ++h) {
          const int cb = c0 + 16 * h;
          const int(&o)[16] = h ? ob : oa;
          const uint32_t(&v)[16] = h ? vb : va;
          if (via_tma) {
            if (r < p.tile_rows) {
#pragma unroll
              for (int j = 0; j < 16; ++j) tile[(cb + j) * p.tile_rows + r] = (int8_t)o[j];
            }
          } else if (row_ok) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb + j < p.m) out[(int64_t)(cb + j) * p.ldo + n] = (int8_t)o[j];
          }
          if (acc_out && row_ok) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb + j < p.m) acc_out[(int64_t)(cb + j) * p.n + n] = (int32_t)v[j];
          }
        }
      }
      if (via_tma) {
        // generic-proxy writes of the tile -> visible to the bulk-copy engine
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        epi_barrier();
        // rows >= m and columns >= n fall outside the tensor and are not written
        if (et == 0) tma_store_2d(&tmap_out, row0, 0, tile);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(p.tmem_cols)
                 : "memory");
  }
}

// ------------------------------------------------------------------------
// Batched form: `count` independent GEMMs of the same shape in one launch.
// Every CTA owns the same tile_rows weight rows of every GEMM and streams
// them GEMM after GEMM through one stage ring, so the ring never drains
// between GEMMs and the launch, ramp-up and tail are paid once per launch
// instead of once per GEMM.  The accumulator is double-buffered in TMEM
// (2 x mpad columns): the epilogue requantises and stores GEMM i from one
// buffer while the MMA warp accumulates GEMM i + 1 into the other.  The
// int8 output tile has its own shared-memory buffer (the ring is still in
// use), stored by one TMA store per GEMM whose shared-memory reads are waited
// for before the next GEMM's tile is written.
constexpr int kMaxGemmItems = 16;
constexpr int kBatchMaxTokens = 64;
constexpr int kBatchTileBytes = kBatchMaxTokens * kMmaRows;  // int8 output tile [mpad x tile_rows]

struct GemmBatchMaps {  // tensor maps live in the kernel's parameter space
  CUtensorMap w[kMaxGemmItems];
  CUtensorMap a[kMaxGemmItems];
  CUtensorMap o[kMaxGemmItems];
};

struct GemmBatchParams {
  const float *sa[kMaxGemmItems];
  const float *ws[kMaxGemmItems];
  int8_t *out[kMaxGemmItems];
  float out_scale;
  float inv_out_scale;
  int64_t ldo;
  int32_t count, m, n, k;
  int32_t mpad, nkb, bps, nks, nst, stage_bytes, b_bytes, tile_rows, tma_store;
  uint32_t tmem_cols;
  uint32_t *status;
};

__device__ __forceinline__ void tma_store_2d_commit(const CUtensorMap *map, int x, int y, const void *src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
               "r"(y), "r"(smem_u32(src))
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_i8_tc_batch_kernel(const __grid_constant__ GemmBatchMaps maps, const GemmBatchParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [ring: nst stages] [int8 output tile] [barriers ...] [activation scales, two buffers]
  uint8_t *stages = smem;
  int8_t *tile = reinterpret_cast<int8_t *>(smem + (size_t)p.nst * p.stage_bytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)p.nst * p.stage_bytes + kBatchTileBytes);
  uint64_t *empty = full + p.nst;
  uint64_t *acc_full = empty + p.nst;  // [2] accumulator buffer complete
  uint64_t *acc_empty = acc_full + 2;  // [2] accumulator buffer read by the epilogue
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  float *sa_buf = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(full) + kBarRegion);  // [2][64]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * p.tile_rows;
  const int total = p.count * p.nks;  // stages over all GEMMs

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiThreads / 32);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      for (int i = 0; i < p.count; ++i) {
        prefetch_tmap(&maps.w[i]);
        prefetch_tmap(&maps.a[i]);
      }
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t tx_block = (uint32_t)(p.tile_rows * kKBlock + p.b_bytes);
      const int pre = min(p.nst, total);
      // weights of the first stages, before the previous grid has finished
      for (int gs = 0; gs < pre; ++gs) {
        const int i = gs / p.nks, ks = gs % p.nks, nb = min(p.bps, p.nkb - ks * p.bps);
        uint8_t *st = stages + (size_t)gs * p.stage_bytes;
        mbar_arrive_expect_tx(&full[gs], (uint32_t)nb * tx_block);
        for (int j = 0; j < nb; ++j)
          tma_load_2d_hint(stage_w(st, j), &maps.w[i], (ks * p.bps + j) * kKBlock, row0, &full[gs], pol);
      }
      pdl_wait();
      pdl_trigger();
      for (int gs = 0; gs < pre; ++gs) {
        const int i = gs / p.nks, ks = gs % p.nks, nb = min(p.bps, p.nkb - ks * p.bps);
        uint8_t *st = stages + (size_t)gs * p.stage_bytes;
        for (int j = 0; j < nb; ++j)
          tma_load_2d(stage_a(st, p.bps, p.b_bytes, j), &maps.a[i], (ks * p.bps + j) * kKBlock, 0, &full[gs]);
      }
      int issued = pre;
      for (int gs = pre; gs < total; ++gs) {
        const int s = gs % p.nst, i = gs / p.nks, ks = gs % p.nks, nb = min(p.bps, p.nkb - ks * p.bps);
        if (!mbar_wait(&empty[s], (uint32_t)((gs / p.nst) - 1) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)nb * tx_block);
        for (int j = 0; j < nb; ++j) {
          tma_load_2d_hint(stage_w(st, j), &maps.w[i], (ks * p.bps + j) * kKBlock, row0, &full[s], pol);
          tma_load_2d(stage_a(st, p.bps, p.b_bytes, j), &maps.a[i], (ks * p.bps + j) * kKBlock, 0, &full[s]);
        }
        ++issued;
      }
      for (int gs = max(0, issued - p.nst); gs < issued; ++gs) {
        if (!mbar_wait(&full[gs % p.nst], (uint32_t)(gs / p.nst) & 1u)) set_status(p.status, kStatusTimeout);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = (2u << 4)                            // D: s32
                             | (1u << 7) | (1u << 10)             // A, B: signed int8
                             | ((uint32_t)(p.mpad >> 3) << 17)    // N
                             | ((uint32_t)(kMmaRows >> 4) << 24);  // M
      int gs = 0;
      bool stop = false;
      for (int i = 0; i < p.count && !stop; ++i) {
        const int b = i & 1;
        // the epilogue has read this buffer's previous GEMM (i - 2)
        if (i >= 2 && !mbar_wait(&acc_empty[b], (uint32_t)((i >> 1) - 1) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_d + (uint32_t)(b * p.mpad);
        for (int ks = 0; ks < p.nks; ++ks, ++gs) {
          const int s = gs % p.nst;
          if (!mbar_wait(&full[s], (uint32_t)(gs / p.nst) & 1u)) {
            set_status(p.status, kStatusTimeout);
            *abort_flag = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          uint8_t *st = stages + (size_t)s * p.stage_bytes;
          const int nb = min(p.bps, p.nkb - ks * p.bps);
          for (int j = 0; j < nb; ++j) {
            const uint64_t adesc = umma_desc_sw128(stage_w(st, j));
            const uint64_t bdesc = umma_desc_sw128(stage_a(st, p.bps, p.b_bytes, j));
#pragma unroll
            for (int kk = 0; kk < kKBlock / 32; ++kk)
              tc_mma_i8(d, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                        (ks > 0 || j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!stop) tc_commit(&acc_full[b]);  // fires once GEMM i's MMAs have completed
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int et = threadIdx.x - 64;  // 0..127
    const int quarter = warp & 3;     // TMEM lanes 32*quarter .. +31
    const int r = quarter * 32 + lane;
    const int n = row0 + r;
    const bool row_ok = r < p.tile_rows && n < p.n;
    const bool via_tma = p.tma_store != 0;
    // Scales may come from the previous grid; outputs may still be read by it.
    pdl_wait();
    const uint32_t taddr0 = tmem_d + ((uint32_t)(quarter * 32) << 16);
    bool stored = false;
    for (int i = 0; i < p.count; ++i) {
      const int b = i & 1;
      float *sa_s = sa_buf + b * kBatchMaxTokens;
      const float *__restrict__ sa = p.sa[i];
      for (int m = et; m < p.mpad; m += kEpiThreads) sa_s[m] = m < p.m ? sa[m] : 0.0f;
      const float wsn = row_ok ? p.ws[i][n] : 0.0f;
      // sa_s is complete, and thread 0 has seen the previous tile's store read
      epi_barrier();
      const bool ok = epi_all(mbar_wait(&acc_full[b], (uint32_t)(i >> 1) & 1u));
      tc_fence_after();
      if (!ok) {
        if (et == 0) set_status(p.status, kStatusTimeout);
        break;
      }
      if (!epi_all(*abort_flag == 0)) break;
      int8_t *__restrict__ out = p.out[i];
      const uint32_t taddr = taddr0 + (uint32_t)(b * p.mpad);
      for (int c0 = 0; c0 < p.mpad; c0 += 32) {
        const bool two = c0 + 16 < p.mpad;  // uniform across the CTA
        uint32_t va[16], vb[16];
        tc_ld16_nowait(taddr + (uint32_t)c0, va);
        if (two) tc_ld16_nowait(taddr + (uint32_t)(c0 + 16), vb);
        tc_wait_ld(va, vb);
        int oa[16], ob[16];
        requant16(va, sa_s + c0, wsn, p.out_scale, p.inv_out_scale, oa);
        if (two) requant16(vb, sa_s + c0 + 16, wsn, p.out_scale, p.inv_out_scale, ob);
        for (int h = 0; h < (two ? 2 : 1); ++h) {
          const int cb = c0 + 16 * h;
          const int(&o)[16] = h ? ob : oa;
          if (via_tma) {
            if (r < p.tile_rows) {
#pragma unroll
              for (int j = 0; j < 16; ++j) tile[(cb + j) * p.tile_rows + r] = (int8_t)o[j];
            }
          } else if (row_ok) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb + j < p.m) out[(int64_t)(cb + j) * p.ldo + n] = (int8_t)o[j];
          }
        }
      }
      // this warp's TMEM loads are complete (tcgen05.wait::ld above): free the buffer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (via_tma) {
        // generic-proxy writes of the tile -> visible to the bulk-copy engine
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        epi_barrier();
        // rows >= m and columns >= n fall outside the tensor and are not written
        if (et == 0) {
          tma_store_2d_commit(&maps.o[i], row0, 0, tile);
          bulk_wait_read_all();  // the tile may be rewritten after the next barrier
          stored = true;
        }
      }
    }
    if (stored) bulk_wait_all();  // every output store has completed before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(p.tmem_cols)
                 : "memory");
  }
}

// Generic fallback (any strides / alignment): one warp per (token, weight row).
__global__ void __launch_bounds__(256)
    gemm_i8_generic_kernel(const int8_t *__restrict__ a, int64_t lda, const int8_t *__restrict__ w, int64_t ldw,
                           const GemmParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)p.m * p.n;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += nwarps) {
    const int m = (int)(i / p.n), n = (int)(i % p.n);
    const int8_t *ar = a + m * lda;
    const int8_t *wr = w + (int64_t)n * ldw;
    uint32_t acc = 0;
    for (int k = lane; k < p.k; k += 32) acc += (uint32_t)((int)ar[k] * (int)wr[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      p.out[m * p.ldo + n] = requant((int32_t)acc, p.sa[m], p.ws[n], p.out_scale);
      if (p.acc_out) p.acc_out[(int64_t)m * p.n + n] = (int32_t)acc;
    }
  }
}

bool tc_shape_ok(const GemmI8Launch &a) {
  const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return a.m >= 1 && a.m <= kMaxTokens && a.n >= 1 && a.n < (int64_t(1) << 31) && a.k >= 1 &&
         a.k < (int64_t(1) << 31) && a.lda % 16 == 0 && a.ldw % 16 == 0 && al16(a.a) && al16(a.w) &&
         encode_fn() != nullptr;
}

}  // namespace

int gemm_i8_path(const GemmI8Launch &a) { return tc_shape_ok(a) ? 1 : 0; }

namespace {
// K blocks per stage: KS_B200_GEMM_BLOCKS (1, 2 or 4), default 4, never more than K has.
// Measured at 14336 x 4096 (batched, M = 8): 14.8 / 10.1 / 8.8 us for 1 / 2 / 4.
int gemm_blocks_per_stage(int nkb) {
  static const int env = env_int("KS_B200_GEMM_BLOCKS", 4);
  const int b = env >= 4 ? 4 : env >= 2 ? 2 : 1;
  return std::max(1, std::min(b, nkb));
}
}  // namespace

cudaError_t launch_gemm_i8(const GemmI8Launch &a, cudaStream_t stream, int device) {
  GemmParams p{};
  p.sa = a.sa;
  p.ws = a.ws;
  p.out_scale = a.out_scale;
  {
    const float inv = 1.0f / a.out_scale;  // IEEE division on the host: RN(1 / out_scale)
    p.inv_out_scale = std::isfinite(inv) ? inv : 0.0f;
  }
  p.out = a.out;
  p.ldo = a.ldo;
  p.acc_out = a.acc_out;
  p.m = (int32_t)a.m;
  p.n = (int32_t)a.n;
  p.k = (int32_t)a.k;
  p.status = a.status;
  const DeviceProps &dp = device_props(device);
  if (!tc_shape_ok(a)) {
    const int64_t warps = a.m * a.n;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, (int64_t)dp.sm_count * 16));
    gemm_i8_generic_kernel<<<grid, 256, 0, stream>>>(a.a, a.lda, a.w, a.ldw, p);
    return cudaGetLastError();
  }
  p.mpad = (int32_t)((a.m + 15) / 16 * 16);
  p.nkb = (int32_t)((a.k + kKBlock - 1) / kKBlock);
  p.b_bytes = p.mpad * kKBlock;
  p.bps = gemm_blocks_per_stage(p.nkb);
  uint32_t cols = 32;
  while (cols < (uint32_t)p.mpad) cols <<= 1;
  p.tmem_cols = cols;
  // Rows per CTA: the same share for every SM, at most the MMA's 128.  Every
  // CTA also reads the whole activation tile (from L2), so a tile is kept at
  // least half as tall as the padded token count (and at least 16 rows).
  const int64_t slots = (int64_t)dp.sm_count;
  const int64_t waves = (a.n + slots * kMmaRows - 1) / (slots * kMmaRows);
  const int64_t even = (a.n + waves * slots - 1) / (waves * slots);
  const int64_t floor_rows = std::min<int64_t>(kMmaRows, std::max<int64_t>(16, p.mpad / 2));
  // multiple of 16 rows: the output tile's TMA store starts at x = row0
  p.tile_rows = (int32_t)std::min<int64_t>(kMmaRows, (std::max(even, floor_rows) + 15) / 16 * 16);
  const int grid = (int)((a.n + p.tile_rows - 1) / p.tile_rows);
  const int reserve = 1024 /* alignment slack */ + kBarRegion + kScaleRegion;
  // at least two stages in flight: fewer blocks per stage for many tokens
  while (p.bps > 1 && (dp.smem_optin - reserve) / (p.bps * (kWTileBytes + p.b_bytes)) < 2) p.bps /= 2;
  p.nks = (p.nkb + p.bps - 1) / p.bps;
  p.stage_bytes = p.bps * (kWTileBytes + p.b_bytes);  // multiple of 1024
  int nst = (dp.smem_optin - reserve) / p.stage_bytes;
  nst = std::min(nst, std::max(1, std::min(kMaxStages, env_int("KS_B200_GEMM_STAGES", 8))));
  nst = std::min(nst, p.nks);
  if (nst < 1) return cudaErrorInvalidValue;
  p.nst = nst;
  CUtensorMap mw, ma, mo;
  if (!make_map(&mw, a.w, a.n, a.k, a.ldw, p.tile_rows) || !make_map(&ma, a.a, a.m, a.k, a.lda, p.mpad))
    return cudaErrorInvalidValue;
  // int8 output [m, n], row stride ldo: one box [mpad x tile_rows] per CTA.
  p.tma_store = (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0 && a.ldo % 16 == 0 &&
                make_store_map(&mo, a.out, a.m, a.n, a.ldo, p.tile_rows, p.mpad);
  if (!p.tma_store) std::memset(&mo, 0, sizeof(mo));
  const size_t smem = (size_t)reserve + (size_t)nst * p.stage_bytes;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[device & 63], [&] {
    attr_err[device & 63] =
        cudaFuncSetAttribute(gemm_i8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dp.smem_optin);
  });
  if (attr_err[device & 63] != cudaSuccess) return attr_err[device & 63];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled(stream)) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemm_i8_tc_kernel, mw, ma, mo, p);
}

cudaError_t launch_gemm_i8_batch(const GemmI8Launch &shape, const GemmI8Batch &b, cudaStream_t stream,
                                 int device) {
  if (b.count <= 0) return cudaSuccess;
  auto item = [&](int i) {
    GemmI8Launch g = shape;
    g.a = b.a[i];
    g.sa = b.sa[i];
    g.w = b.w[i];
    g.ws = b.ws[i];
    g.out = b.out[i];
    g.acc_out = nullptr;
    return g;
  };
  // The batched kernel takes up to 64 tokens with every operand on the
  // tensor-core path; anything else runs one launch per GEMM.
  bool batched = shape.m <= kBatchMaxTokens;
  for (int i = 0; i < b.count && batched; ++i) batched = tc_shape_ok(item(i));
  if (!batched) {
    for (int i = 0; i < b.count; ++i) {
      const cudaError_t e = launch_gemm_i8(item(i), stream, device);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  const DeviceProps &dp = device_props(device);
  GemmBatchParams p{};
  p.out_scale = shape.out_scale;
  {
    const float inv = 1.0f / shape.out_scale;  // IEEE division on the host: RN(1 / out_scale)
    p.inv_out_scale = std::isfinite(inv) ? inv : 0.0f;
  }
  p.ldo = shape.ldo;
  p.m = (int32_t)shape.m;
  p.n = (int32_t)shape.n;
  p.k = (int32_t)shape.k;
  p.status = shape.status;
  p.mpad = (int32_t)((shape.m + 15) / 16 * 16);
  p.nkb = (int32_t)((shape.k + kKBlock - 1) / kKBlock);
  p.b_bytes = p.mpad * kKBlock;
  p.bps = gemm_blocks_per_stage(p.nkb);
  uint32_t cols = 32;
  while (cols < (uint32_t)(2 * p.mpad)) cols <<= 1;
  p.tmem_cols = cols;
  const int64_t slots = (int64_t)dp.sm_count;
  const int64_t waves = (shape.n + slots * kMmaRows - 1) / (slots * kMmaRows);
  const int64_t even = (shape.n + waves * slots - 1) / (waves * slots);
  const int64_t floor_rows = std::min<int64_t>(kMmaRows, std::max<int64_t>(16, p.mpad / 2));
  p.tile_rows = (int32_t)std::min<int64_t>(kMmaRows, (std::max(even, floor_rows) + 15) / 16 * 16);
  const int grid = (int)((shape.n + p.tile_rows - 1) / p.tile_rows);
  const int reserve = 1024 /* alignment slack */ + kBatchTileBytes + kBarRegion + 2 * kBatchMaxTokens * 4;
  // at least two stages in flight
  while (p.bps > 1 && (dp.smem_optin - reserve) / (p.bps * (kWTileBytes + p.b_bytes)) < 2) p.bps /= 2;
  p.nks = (p.nkb + p.bps - 1) / p.bps;
  p.stage_bytes = p.bps * (kWTileBytes + p.b_bytes);
  int nst_cap = (dp.smem_optin - reserve) / p.stage_bytes;
  nst_cap = std::min(nst_cap, std::max(1, std::min(kMaxStages, env_int("KS_B200_GEMM_STAGES", 8))));
  if (nst_cap < 1) return cudaErrorInvalidValue;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[device & 63], [&] {
    attr_err[device & 63] =
        cudaFuncSetAttribute(gemm_i8_tc_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dp.smem_optin);
  });
  if (attr_err[device & 63] != cudaSuccess) return attr_err[device & 63];
  for (int i0 = 0; i0 < b.count; i0 += kMaxGemmItems) {
    const int cnt = std::min(kMaxGemmItems, b.count - i0);
    GemmBatchMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    p.count = cnt;
    p.nst = std::min<int>(nst_cap, cnt * p.nks);
    bool tma_store = shape.ldo % 16 == 0;
    for (int j = 0; j < cnt; ++j) {
      const int i = i0 + j;
      p.sa[j] = b.sa[i];
      p.ws[j] = b.ws[i];
      p.out[j] = b.out[i];
      if (!make_map(&maps.w[j], b.w[i], shape.n, shape.k, shape.ldw, p.tile_rows) ||
          !make_map(&maps.a[j], b.a[i], shape.m, shape.k, shape.lda, p.mpad))
        return cudaErrorInvalidValue;
      tma_store = tma_store && (reinterpret_cast<uintptr_t>(b.out[i]) & 15u) == 0 &&
                  make_store_map(&maps.o[j], b.out[i], shape.m, shape.n, shape.ldo, p.tile_rows, p.mpad);
    }
    p.tma_store = tma_store ? 1 : 0;
    const size_t smem = (size_t)reserve + (size_t)p.nst * p.stage_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl_enabled(stream)) {
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i8_tc_batch_kernel, maps, p);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace ksb
