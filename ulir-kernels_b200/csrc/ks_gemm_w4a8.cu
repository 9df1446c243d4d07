// ks_gemm_w4a8.cu -- batched W4A8 GEMM for decode (M = 1..64 tokens) on 5th-
// generation tensor cores (tcgen05.mma kind::i8, TMEM accumulators), sm_100a.
//
//   y[m, n]      = sx[m] * sum_g f32(acc_g[m, n]) * s[n, g]      (groups in order)
//   acc_g[m, n]  = sum_{k in group g} x[m, k] * w[n, k]           (int32, exact)
//
// x: int8 activations [M, K] with a per-token scale sx[m]; w: the native W4A8
// weights (signed int4, value k in byte k/2, low nibble for even k) [N, K];
// s: f16 or f32 group scales [N, K/G], G in {32, 64, 128}; zero points 0.
// Each token's row of y is ks_matvec_w4a8's result for that token up to the
// order of the f32 sum (the reference sums per element; here per group,
// like the GEMV kernels).
//
// Swap-AB as in the INT8 GEMM: weight rows fill the MMA's M = 128 (TMEM
// lanes), tokens its N (padded to 16).  A CTA owns `tile_rows` weight rows
// (the same share for every SM, a multiple of 16).  K streams in stages of up
// to four 128-K blocks (one barrier round trip per stage in every hand-off;
// each round trip costs the MMA thread a few hundred cycles).  Per block:
//   warp 0    TMA: the packed weight tile [tile_rows x 64 B] (no swizzle),
//             the token tile [Mpad x 128 B] (128-byte swizzle) and, once per
//             one or more stages, a scale box [tile_rows x 16..64 B] into a
//             small ring of its own.  No multicast.
//   warps 2-5 unpack: one weight row each, int4 -> int8 holding 16 x the
//             weight (shift + mask per 4 bytes, PRMT to interleave), written
//             in the UMMA K-major 128-byte-swizzle layout; proxy fence; arrive.
//   warp 1    MMA: per group, tcgen05.mma (K = 32 each, G / 32 of them) into
//             the group's own TMEM column block (fresh accumulate), buffered
//             over as many stages as 512 TMEM columns hold (at least 2, up
//             to 8); one commit per stage frees it, one hands the buffer to
//             the epilogue.
//   warps 6-9 epilogue: tcgen05.ld each group's int32 accumulators (one TMEM
//             lane per weight row), acc[m] += f32(v) * (s[n, g] / 16) in
//             registers,
//             release the TMEM buffer; at the end y = acc * sx.
// Every wait is bounded (about one second); a timeout is recorded in the
// status word, the waiting role stops, and the kernel runs to its end.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "ks_internal.h"
#include "ks_ptx.cuh"
#include "ks_tc.cuh"

namespace ksb {

namespace {

constexpr int kRows = 128;         // MMA M
constexpr int kStageK = 128;       // K elements per stage: one 128-byte int8 swizzle row
constexpr int kPacked = kStageK / 2;  // packed weight bytes per row per stage
constexpr int kThreads = 320;      // 0 producer, 1 MMA, 2-5 unpack, 6-9 epilogue
constexpr int kScaleRing = 4;
constexpr int kMaxStagesW4 = 8;
constexpr int kMaxBufs = 8;
constexpr int kOpBytes = kRows * kStageK;  // int8 weight operand of a stage

struct W4GemmParams {
  float *y;
  int64_t ldy;
  const float *sx;
  int32_t m, n, k;
  int32_t nkb;        // 128-K blocks (K / 128, rounded up)
  int32_t bps;        // blocks per ring stage (one barrier round trip per stage in every ring)
  int32_t nks;        // stages: nkb / bps, rounded up
  int32_t nst;        // ring stages
  int32_t tile_rows;
  int32_t gps;        // groups per block: 128 / G (at least 1)
  int32_t kpg;        // MMAs (K = 32) per group: G / 32
  int32_t sbytes;     // 2 (f16) or 4 (f32)
  int32_t sbox;       // scale bytes per row per box: max(16, bps * gps * sbytes)
  int32_t spb;        // stages per scale box
  int32_t stage_bytes, a_bytes, pk_bytes, sbox_bytes;  // a_bytes, pk_bytes: per block
  int32_t nbuf;       // TMEM accumulator buffers (stages the MMA may run ahead of the epilogue)
  uint32_t tmem_cols;
  uint32_t *status;
};

// 8 signed int4 (value 2b in the low nibble of byte b, 2b + 1 in the high
// nibble) -> 8 int8 in k order, as two words, each byte holding 16 x the
// weight (the nibble moved to the byte's high half: exact and sign-correct).
// The int32 group sums are then 16 x the true sums (at most 128 * 128 * 128
// in magnitude, exact in f32) and the epilogue scales by s / 16 instead of s
// -- a power of two, so every product and sum rounds as with the true sums.
__device__ __forceinline__ void unpack8x16(uint32_t v, uint32_t &lo, uint32_t &hi) {
  const uint32_t te = (v << 4) & 0xF0F0F0F0u;  // values 0, 2, 4, 6
  const uint32_t to = v & 0xF0F0F0F0u;         // values 1, 3, 5, 7
  lo = prmt(te, to, 0x5140);
  hi = prmt(te, to, 0x7362);
}

template <int MPAD>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w4a8_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_s, const W4GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [stage 0 .. nst-1: bps int8 operands (16 KB each) | bps token tiles | bps packed tiles]
  // [scale boxes] [barriers]
  uint8_t *stages = smem;
  uint8_t *sboxes = smem + (size_t)p.nst * p.stage_bytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sboxes + (size_t)kScaleRing * p.sbox_bytes);
  uint64_t *full = bars;                      // [nst]  TMA landed
  uint64_t *unpacked = full + kMaxStagesW4;   // [nst]  int8 operands written
  uint64_t *empty = unpacked + kMaxStagesW4;  // [nst]  MMAs of the stage done
  uint64_t *mma_done = empty + kMaxStagesW4;  // [nbuf] TMEM buffer ready
  uint64_t *tmem_free = mma_done + kMaxBufs;  // [nbuf] TMEM buffer read
  uint64_t *sfull = tmem_free + kMaxBufs;     // [ring] scale box landed
  uint64_t *sempty = sfull + kScaleRing;      // [ring] scale box used
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + kScaleRing);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * p.tile_rows;
  const int tok_off = p.bps * kOpBytes;                  // token tiles of a stage
  const int pk_off = p.bps * (kOpBytes + p.a_bytes);     // packed tiles of a stage
  auto blocks_of = [&](int ks) { return min(p.bps, p.nkb - ks * p.bps); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&unpacked[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < p.nbuf; ++b) {
      mbar_init(&mma_done[b], 1);
      mbar_init(&tmem_free[b], 4);
    }
    for (int b = 0; b < kScaleRing; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], 4);
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
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_a);
      prefetch_tmap(&tmap_s);
      pdl_wait();
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t tx_block = (uint32_t)(p.tile_rows * kPacked + MPAD * kStageK);
      int issued = 0, boxes = 0;
      for (int ks = 0; ks < p.nks; ++ks) {
        const int s = ks % p.nst;
        if (ks >= p.nst && !mbar_wait(&empty[s], (uint32_t)((ks / p.nst) - 1) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        if (ks % p.spb == 0) {
          const int bi = ks / p.spb, sb = bi % kScaleRing;
          if (bi >= kScaleRing && !mbar_wait(&sempty[sb], (uint32_t)((bi / kScaleRing) - 1) & 1u)) {
            set_status(p.status, kStatusTimeout);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&sfull[sb], (uint32_t)(p.tile_rows * p.sbox));
          tma_load_2d(sboxes + (size_t)sb * p.sbox_bytes, &tmap_s, bi * p.sbox, row0, &sfull[sb]);
          ++boxes;
        }
        const int nb = blocks_of(ks);
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)nb * tx_block);
        for (int j = 0; j < nb; ++j) {
          const int kb = ks * p.bps + j;
          tma_load_2d_hint(st + pk_off + j * p.pk_bytes, &tmap_w, kb * kPacked, row0, &full[s], pol);
          tma_load_2d(st + tok_off + j * p.a_bytes, &tmap_a, kb * kStageK, 0, &full[s]);
        }
        ++issued;
      }
      pdl_trigger();
      for (int ks = max(0, issued - p.nst); ks < issued; ++ks)
        if (!mbar_wait(&full[ks % p.nst], (uint32_t)(ks / p.nst) & 1u)) set_status(p.status, kStatusTimeout);
      for (int bi = max(0, boxes - kScaleRing); bi < boxes; ++bi)
        if (!mbar_wait(&sfull[bi % kScaleRing], (uint32_t)(bi / kScaleRing) & 1u))
          set_status(p.status, kStatusTimeout);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA --
    if (lane == 0) {
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MPAD >> 3) << 17) |
                             ((uint32_t)(kRows >> 4) << 24);
      for (int ks = 0; ks < p.nks; ++ks) {
        const int s = ks % p.nst, b = ks % p.nbuf;
        if (!mbar_wait(&unpacked[s], (uint32_t)(ks / p.nst) & 1u) ||
            (ks >= p.nbuf && !mbar_wait(&tmem_free[b], (uint32_t)((ks / p.nbuf) - 1) & 1u))) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        const int nb = blocks_of(ks);
        for (int j = 0; j < nb; ++j) {
          const uint64_t adesc = umma_desc_sw128(st + j * kOpBytes);
          const uint64_t bdesc = umma_desc_sw128(st + tok_off + j * p.a_bytes);
          for (int g = 0; g < p.gps; ++g) {
            const uint32_t d = tmem_d + (uint32_t)(((b * p.bps + j) * p.gps + g) * MPAD);
            for (int kk = 0; kk < p.kpg; ++kk) {
              const int kx = g * p.kpg + kk;  // 32-element step inside the 128-byte row
              tc_mma_i8(d, adesc + (uint64_t)(2 * kx), bdesc + (uint64_t)(2 * kx), idesc, kk > 0 ? 1u : 0u);
            }
          }
        }
        tc_commit(&empty[s]);
        tc_commit(&mma_done[b]);
      }
    }
  } else if (warp < 6) {
    // -------------------------------------------------------------- unpack --
    const int r = threadIdx.x - 64;  // weight row of the tile
    for (int ks = 0; ks < p.nks; ++ks) {
      const int s = ks % p.nst;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (uint32_t)(ks / p.nst) & 1u))) {
        if (lane == 0) set_status(p.status, kStatusTimeout);
        break;
      }
      uint8_t *st = stages + (size_t)s * p.stage_bytes;
      const int nb = blocks_of(ks);
      if (r < p.tile_rows) {
        for (int j = 0; j < nb; ++j) {
          const uint8_t *src = st + pk_off + j * p.pk_bytes + (size_t)r * kPacked;
          uint8_t *dst = st + j * kOpBytes + (size_t)r * kStageK;
          // 16 packed bytes = 32 weights = two 16-byte output chunks.  The
          // chunk order rotates with lane / 8: packed rows are 64 bytes apart,
          // so the 32 lanes reading chunk q together would hit 8 of the 32
          // banks (16-way conflicts); rotated they cover all banks, and each
          // group of 8 rows keeps one chunk, so the swizzled 16-byte stores
          // below stay conflict-free too.
#pragma unroll
          for (int q0 = 0; q0 < 4; ++q0) {
            const int q = (q0 + (lane >> 3)) & 3;
            const uint4 v = lds128(src + 16 * q);
            uint32_t o[8];
            unpack8x16(v.x, o[0], o[1]);
            unpack8x16(v.y, o[2], o[3]);
            unpack8x16(v.z, o[4], o[5]);
            unpack8x16(v.w, o[6], o[7]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int c = 2 * q + h;  // 16-byte chunk of the 128-byte row, swizzled by the row within its 8
              *reinterpret_cast<uint4 *>(dst + ((c ^ (r & 7)) << 4)) =
                  make_uint4(o[4 * h], o[4 * h + 1], o[4 * h + 2], o[4 * h + 3]);
            }
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA operand reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&unpacked[s]);
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int n = row0 + r;
    const bool row_ok = r < p.tile_rows && n < p.n;
    pdl_wait();
    float acc[MPAD];
#pragma unroll
    for (int t = 0; t < MPAD; ++t) acc[t] = 0.0f;
    bool stop = false;
    const uint32_t lane_base = tmem_d + ((uint32_t)(quarter * 32) << 16);
    const int gst = p.bps * p.gps;  // group accumulators per full stage
    for (int ks = 0; ks < p.nks && !stop; ++ks) {
      const int b = ks % p.nbuf;
      const int bi = ks / p.spb, sb = bi % kScaleRing;
      bool ok = true;
      if (ks % p.spb == 0) ok = mbar_wait(&sfull[sb], (uint32_t)(bi / kScaleRing) & 1u);
      ok = ok && mbar_wait(&mma_done[b], (uint32_t)(ks / p.nbuf) & 1u);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) set_status(p.status, kStatusTimeout);
        stop = true;
        break;
      }
      tc_fence_after();
      const uint8_t *srow = sboxes + (size_t)sb * p.sbox_bytes + (size_t)r * p.sbox;
      const int gbase = (ks % p.spb) * gst;  // this stage's first group inside the box row
      const int ng = blocks_of(ks) * p.gps;  // groups computed in this stage
      // The stage's group accumulators are contiguous TMEM columns
      // ((b * bps + j) * gps + g) * MPAD: up to 64 of them are loaded before one wait.
      constexpr int GPC = MPAD >= 48 ? 1 : 64 / MPAD;  // groups per load batch
      for (int g0 = 0; g0 < ng; g0 += GPC) {
        const int nvals = min(GPC, ng - g0) * MPAD;
        const uint32_t col = lane_base + (uint32_t)((b * gst + g0) * MPAD);
        uint32_t v0[16], v1[16], v2[16], v3[16];
        tc_ld16_nowait(col, v0);
        if (16 < nvals) tc_ld16_nowait(col + 16u, v1);
        if (32 < nvals) tc_ld16_nowait(col + 32u, v2);
        if (48 < nvals) tc_ld16_nowait(col + 48u, v3);
        tc_wait_ld(v0, v1);
        tc_wait_ld(v2, v3);  // nothing left to wait for: passes v2, v3 through the wait
        float sc[GPC];
        // the box holds tile_rows rows: lanes at and above them have no weight row
        const int gi0 = gbase + g0;  // first scale index of the batch inside the box row
        if (r < p.tile_rows && g0 + GPC <= ng && gi0 % GPC == 0 && (gi0 + GPC) * p.sbytes <= p.sbox) {
          // the batch's scales in one vector load (rows are sbox bytes apart:
          // one load per batch instead of GPC conflicting 2- or 4-byte loads)
          if (p.sbytes == 2) {
            uint32_t h[(GPC + 1) / 2];
            if constexpr (GPC == 4) {
              const uint2 t = *reinterpret_cast<const uint2 *>(srow + 2 * gi0);
              h[0] = t.x;
              h[1] = t.y;
            } else if constexpr (GPC == 2) {
              h[0] = *reinterpret_cast<const uint32_t *>(srow + 2 * gi0);
            } else {
              h[0] = *reinterpret_cast<const uint16_t *>(srow + 2 * gi0);
            }
#pragma unroll
            for (int gg = 0; gg < GPC; ++gg)
              sc[gg] = __half2float(__ushort_as_half((unsigned short)(h[gg / 2] >> (16 * (gg & 1)))));
          } else {
            if constexpr (GPC == 4) {
              const float4 t = *reinterpret_cast<const float4 *>(srow + 4 * gi0);
              sc[0] = t.x;
              sc[1] = t.y;
              sc[2] = t.z;
              sc[3] = t.w;
            } else if constexpr (GPC == 2) {
              const float2 t = *reinterpret_cast<const float2 *>(srow + 4 * gi0);
              sc[0] = t.x;
              sc[1] = t.y;
            } else {
              sc[0] = *reinterpret_cast<const float *>(srow + 4 * gi0);
            }
          }
        } else {
#pragma unroll
          for (int gg = 0; gg < GPC; ++gg) {
            const int gi = gi0 + gg;
            sc[gg] = 0.0f;
            if (r < p.tile_rows && g0 + gg < ng)
              sc[gg] = p.sbytes == 2 ? __half2float(*reinterpret_cast<const __half *>(srow + 2 * gi))
                                     : *reinterpret_cast<const float *>(srow + 4 * gi);
          }
        }
#pragma unroll
        for (int gg = 0; gg < GPC; ++gg) sc[gg] = __fmul_rn(sc[gg], 0.0625f);  // the operand holds 16 x the weights
#pragma unroll
        for (int f = 0; f < GPC * MPAD && f < 64; ++f) {
          const uint32_t u = f < 16 ? v0[f & 15] : f < 32 ? v1[f & 15] : f < 48 ? v2[f & 15] : v3[f & 15];
          acc[f % MPAD] = fmaf((float)(int32_t)u, sc[f / MPAD], acc[f % MPAD]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tmem_free[b]);
        if (ks % p.spb == p.spb - 1 || ks == p.nks - 1) mbar_arrive(&sempty[sb]);
      }
    }
    if (!stop && row_ok) {
      const float *__restrict__ sx = p.sx;
#pragma unroll
      for (int t = 0; t < MPAD; ++t)
        if (t < p.m) p.y[(int64_t)t * p.ldy + n] = __fmul_rn(acc[t], sx[t]);
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

// u8 2-D tensor map over `rows` rows of `row_bytes` bytes (stride ld), box [box_cols x box_rows], no swizzle
bool make_plain_map(CUtensorMap *map, const void *base, int64_t rows, int64_t row_bytes, int64_t ld, int box_cols,
                    int box_rows) {
  return make_map(map, base, rows, row_bytes, ld, box_rows, box_cols, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int MPAD>
cudaError_t launch_mpad(const CUtensorMap &mw, const CUtensorMap &ma, const CUtensorMap &ms, const W4GemmParams &p,
                        int grid, size_t smem, cudaStream_t stream, int device) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  std::call_once(once[device & 63], [&] {
    err[device & 63] = cudaFuncSetAttribute(gemm_w4a8_tc_kernel<MPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            device_props(device).smem_optin);
  });
  if (err[device & 63] != cudaSuccess) return err[device & 63];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled(stream)) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemm_w4a8_tc_kernel<MPAD>, mw, ma, ms, p);
}

}  // namespace

bool gemm_w4a8_supported(const GemmW4A8Launch &a) {
  const auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const int sbytes = a.stype == kScaleF16 ? 2 : 4;
  return a.m >= 1 && a.m <= 64 && a.n >= 1 && a.n < (int64_t(1) << 31) && a.k >= 32 && a.k % 32 == 0 &&
         (a.group == 32 || a.group == 64 || a.group == 128) && a.k % a.group == 0 && a.lda % 16 == 0 &&
         a.wstride % 16 == 0 && (a.sstride * sbytes) % 16 == 0 && al16(a.a) && al16(a.w) && al16(a.s) &&
         encode_fn() != nullptr;
}

cudaError_t launch_gemm_w4a8(const GemmW4A8Launch &a, cudaStream_t stream, int device) {
  if (!gemm_w4a8_supported(a)) return cudaErrorNotSupported;
  const DeviceProps &dp = device_props(device);
  W4GemmParams p{};
  p.y = a.y;
  p.ldy = a.ldy;
  p.sx = a.sx;
  p.m = (int32_t)a.m;
  p.n = (int32_t)a.n;
  p.k = (int32_t)a.k;
  p.status = a.status;
  const int mpad = (int)((a.m + 15) / 16 * 16);
  p.nkb = (int32_t)((a.k + kStageK - 1) / kStageK);
  p.gps = (int32_t)(kStageK / a.group) > 0 ? (int32_t)(kStageK / a.group) : 1;
  p.kpg = (int32_t)(a.group / 32);
  p.sbytes = a.stype == kScaleF16 ? 2 : 4;
  const int64_t slots = dp.sm_count;
  const int64_t waves = (a.n + slots * kRows - 1) / (slots * kRows);
  const int64_t even = (a.n + waves * slots - 1) / (waves * slots);
  p.tile_rows = (int32_t)std::min<int64_t>(kRows, (std::max<int64_t>(even, 16) + 15) / 16 * 16);
  const int grid = (int)((a.n + p.tile_rows - 1) / p.tile_rows);
  p.a_bytes = mpad * kStageK;  // multiple of 2048
  p.pk_bytes = (p.tile_rows * kPacked + 1023) / 1024 * 1024;
  // Blocks per stage: KS_B200_W4GEMM_BLOCKS (1, 2 or 4), default 4, halved
  // until TMEM holds two stages of group accumulators and shared memory two
  // stages (fewer barrier round trips per MMA; each costs the MMA thread a
  // few hundred cycles).
  static const int env_bps = env_int("KS_B200_W4GEMM_BLOCKS", 4);
  int bps = env_bps >= 4 ? 4 : env_bps >= 2 ? 2 : 1;
  // a power of two, so the scale bytes per stage are too (TMA boxes and their
  // x coordinates must be multiples of 16 bytes)
  while (bps > p.nkb) bps /= 2;
  auto sbox_of = [&](int bb) { return std::max(16, bb * p.gps * p.sbytes); };
  auto sbox_bytes_of = [&](int bb) { return (p.tile_rows * sbox_of(bb) + 127) / 128 * 128; };
  auto fixed_of = [&](int bb) { return 1024 /* alignment */ + kScaleRing * sbox_bytes_of(bb) + 512 /* barriers */; };
  auto stage_of = [&](int bb) { return bb * (kOpBytes + p.a_bytes + p.pk_bytes); };
  while (bps > 1 && (512 / (bps * p.gps * mpad) < 2 || (dp.smem_optin - fixed_of(bps)) / stage_of(bps) < 2)) bps /= 2;
  p.bps = bps;
  p.nks = (p.nkb + bps - 1) / bps;
  p.sbox = sbox_of(bps);
  p.spb = p.sbox / (bps * p.gps * p.sbytes);
  p.sbox_bytes = sbox_bytes_of(bps);
  p.stage_bytes = stage_of(bps);
  const int per_buf = bps * p.gps * mpad;  // TMEM columns of one stage's group accumulators
  p.nbuf = std::min(kMaxBufs, 512 / per_buf);
  if (p.nbuf < 2) return cudaErrorNotSupported;
  uint32_t cols = 32;
  while (cols < (uint32_t)(p.nbuf * per_buf)) cols <<= 1;
  p.tmem_cols = cols;
  const int fixed = fixed_of(bps);
  int nst = std::min({kMaxStagesW4, (dp.smem_optin - fixed) / p.stage_bytes, p.nks,
                      std::max(1, env_int("KS_B200_W4GEMM_STAGES", kMaxStagesW4))});
  if (nst < 1) return cudaErrorNotSupported;
  p.nst = nst;
  CUtensorMap mw, ma, ms;
  if (!make_plain_map(&mw, a.w, a.n, a.k / 2, a.wstride, kPacked, p.tile_rows) ||
      !make_map(&ma, a.a, a.m, a.k, a.lda, mpad) ||
      !make_plain_map(&ms, a.s, a.n, a.k / a.group * p.sbytes, a.sstride * p.sbytes, p.sbox, p.tile_rows))
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)fixed + (size_t)nst * p.stage_bytes;
  switch (mpad) {
    case 16: return launch_mpad<16>(mw, ma, ms, p, grid, smem, stream, device);
    case 32: return launch_mpad<32>(mw, ma, ms, p, grid, smem, stream, device);
    case 48: return launch_mpad<48>(mw, ma, ms, p, grid, smem, stream, device);
    default: return launch_mpad<64>(mw, ma, ms, p, grid, smem, stream, device);
  }
}

}  // namespace ksb
