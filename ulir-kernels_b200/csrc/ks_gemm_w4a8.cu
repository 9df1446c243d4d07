// ks_gemm_w4a8.cu -- batched W4A8 GEMM for decode (M = 1..64 tokens) on 5th-
// generation tensor cores (tcgen05.mma kind::i8, TMEM operands), sm_100a.
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
// Swap-AB: weight rows fill the MMA's M = 128 (TMEM lanes), tokens its N
// (padded to 16).  A CTA owns `tile_rows` weight rows (the same share for
// every SM, a multiple of 16).  K runs in 128-element blocks (four MMAs of
// K = 32), four blocks per ring stage, handed between the roles one or two
// blocks at a time (Shape).  The int4 weights are widened to int8 by the CUDA
// cores and written straight into tensor memory, which the MMA reads as its
// A operand, so shared memory holds only what TMA brings in (packed weights
// and tokens: about 40 KB per stage at M <= 16, five stages in flight).
// Roles:
//   warp 0      TMA: per stage two packed-weight boxes [tile_rows x 128 B]
//               (128-byte swizzle: the unpack reads are conflict-free), four
//               token tiles [Mpad x 128 B] (128-byte swizzle, the MMA's B
//               operand) and, once per one or more stages, a scale box
//               [tile_rows x 16..64 B] into a ring of its own.  No multicast.
//   warps 2-9   unpack, two sets of four (one warp per TMEM lane quarter;
//               even and odd blocks): one weight row per lane, int4 -> int8
//               holding 16 x the weight (shift and mask; even k in one word,
//               odd k in the next, the token tiles rewritten into the same k
//               order), tcgen05.st of the row's 32 columns into an A slot,
//               tcgen05.wait::st, arrive.
//   warps 1, 18 MMA: one or two issuers (alternate hand-offs, each with its
//               own accumulator units): per block four tcgen05.mma (A from
//               the slot, B the token tile) into the groups' accumulator
//               columns, loops unrolled with compile-time accumulate flags; a
//               commit per hand-off frees the A slot and hands the
//               accumulators on, one per stage frees the stage (its tokens).
//   warps 10-17 epilogue, two sets of four: tcgen05.ld of a unit's group
//               accumulators (one TMEM lane per weight row), acc[m] +=
//               f32(v) * (s[n, g] / 16), release the columns; at the end
//               y = acc * sx.  Each set takes half of the tokens, or, at most
//               8 tokens (paired accumulators, Shape), half of the groups,
//               the two partial sums added at the end.
// Every barrier has one waiting role that takes its phases in order (a
// parity wait is only sound while the barrier is at most one phase ahead of
// or behind the waiter); tests/test_w4a8_gemm_barrier_model.py restates the
// protocol and checks it under random interleavings.
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

constexpr int kRows = 128;                     // MMA M = TMEM lanes
constexpr int kBlockK = 128;                   // K per block: 32 TMEM columns of int8, four MMAs
constexpr int kBlockPacked = kBlockK / 2;      // packed bytes per row per block
constexpr int kSB = 4;                         // blocks per ring stage (two 128-byte packed boxes)
constexpr int kUnpackWarps = 8;                // two sets of four: even and odd blocks
constexpr int kEpiWarp0 = 2 + kUnpackWarps;    // first epilogue warp
constexpr int kNA = 8;                         // A blocks in TMEM (32 columns each), where the accumulators allow
constexpr int kTmemCols = 512;
constexpr int kMaxStages = 8;
constexpr int kMaxAcc = 8;
constexpr int kMD = 16;  // "MMAs of hand-off h done" barriers: h % kMD (more than the MMA can run ahead of any waiter)
constexpr int kScaleRing = 4;

struct W4GemmParams {
  float *y;
  int64_t ldy;
  const float *sx;
  int32_t m, n, k;
  int32_t nkb;         // 128-K blocks (K / 128, rounded up)
  int32_t nks;         // ring stages: nkb / kSB, rounded up
  int32_t nst;         // ring depth
  int32_t tile_rows;
  int32_t box_bytes;   // one packed box: tile_rows x 128 B
  int32_t tok_off;     // token tiles of a stage, after its two packed boxes
  int32_t stage_bytes;
  int32_t sbytes;      // 2 (f16) or 4 (f32)
  int32_t sbox;        // scale bytes per row per box: max(16, kSB * groups per block * sbytes)
  int32_t spb;         // stages per scale box
  int32_t sbox_bytes;
  uint32_t *status;
};

// 8 signed int4 (value 2b in the low nibble of byte b, 2b + 1 in the high
// nibble) -> 8 int8 as two words, each byte holding 16 x the weight (the
// nibble moved to the byte's high half: exact and sign-correct): even k
// (0, 2, 4, 6) in the first word, odd k in the second.  The MMA only pairs
// A[k] with B[k], so the token tiles are put in the same order (each 8-byte
// group of k as x0 x2 x4 x6 x1 x3 x5 x7) and the weights need no byte
// shuffle.  The int32 group sums are 16 x the true sums (at most 2^21 in
// magnitude) and the epilogue scales by s / 16 instead of s -- a power of
// two, so every product and sum rounds as with the true sums.
__device__ __forceinline__ void unpack8x16(uint32_t v, uint32_t &even, uint32_t &odd) {
  even = (v << 4) & 0xF0F0F0F0u;
  odd = v & 0xF0F0F0F0u;
}

// int32 -> f32, exact for every group sum here (|v| <= 2^21).  The plain
// conversion measured faster than two full-rate operations on the bits of
// 1.5 * 2^23 (an integer add, then subtracting 1.5 * 2^23): 45.9 against
// 52.1 us per GEMM at M = 64, 25.9 against 28.2 at M = 32.
__device__ __forceinline__ float i2f_small(uint32_t v) { return __int2float_rn((int)v); }

// Compile-time shape of one hand-off between the roles: HB blocks (two while
// three accumulator units of two blocks fit in TMEM beside the A slots, else
// one), UPH accumulator units of UG groups (UCOLS columns) per hand-off, NACC
// units after the A slots, NAS A slots of HB blocks.  Fewer, larger hand-offs
// matter: every barrier wait and commit of the MMA thread costs about a
// hundred cycles while the unpack and epilogue warps share its scheduler.
//
// PK (at most 8 tokens): two groups share one 16-column accumulator.  The
// even group's MMAs read the token tile with the tokens in rows 0-7 (rows
// 8-15 zero) and start fresh; the odd group's accumulate with the tokens
// moved to rows 8-15 (rows 0-7 zero), so they fill columns 8-15 and add zero
// to columns 0-7: 8 columns per group instead of 16, and a unit's groups in
// consecutive columns.
template <int MPAD, int KPG, bool PK>
struct Shape {
  static constexpr int GPS = 4 / KPG;  // groups per block
  static constexpr int HB = PK ? 4 : GPS * MPAD <= 64 ? 2 : 1;
  static constexpr int GPH = HB * GPS;
  static constexpr int GCOLS = PK ? 8 : MPAD;  // accumulator columns per group
  static constexpr int UPH = GPH * GCOLS <= 192 ? 1 : 2;
  static constexpr int UG = GPH / UPH;
  static constexpr int UCOLS = UG * GCOLS;
  static constexpr int NA = (kTmemCols - kNA * 32) / UCOLS >= 2 ? kNA : 4;  // A blocks
  static constexpr int NAS = NA / HB;
  static constexpr int ACC0 = NA * 32;  // accumulator columns start after the A slots
  static constexpr int NACC = (kTmemCols - ACC0) / UCOLS < kMaxAcc ? (kTmemCols - ACC0) / UCOLS : kMaxAcc;
  // MMA issuers: two (alternate hand-offs) when each can own NPI >= UPH
  // accumulator units and the A slots split by hand-off parity; else one.
  // Every barrier then has one waiting role that takes its phases in order
  // (a parity wait is only sound while the barrier is at most one phase
  // ahead of or behind the waiter).
  // SPLIT (16-column tokens, hand-offs of 2 or 4 blocks): both issuers take
  // every hand-off, issuer i the i-th half of its blocks, sharing one ring
  // of accumulator units (every waiter still takes every phase in order)
  static constexpr bool SPLIT = MPAD == 16 && HB >= 2;
  static constexpr int ISS = SPLIT ? 2 : NACC >= 2 * UPH && NAS % 2 == 0 ? 2 : 1;
  static constexpr int NPI = SPLIT ? NACC : NACC / ISS;  // units per ring (one ring per issuer unless SPLIT)
  static_assert(NACC >= 2 && kSB % HB == 0, "two accumulator units at least; whole hand-offs per stage");
  static_assert(!PK || (MPAD == 16 && HB == 4 && UPH == 1 && UG % 2 == 0), "pairs of groups per unit");
  // token tile in shared memory: PK keeps 8 zero rows before the box, so the
  // tile at row 8 has the tokens first and the tile at row 0 has them last
  static constexpr int TOKB = (PK ? 24 : MPAD) * kBlockK;  // bytes per block
  static constexpr int TOFF = PK ? 8 * kBlockK : 0;        // where TMA puts the box
};

// Epilogue warps -- two sets of four, each set half of the tokens -- and the
// warp of the second MMA issuer after them (on the third scheduler).
template <int MR>
struct Roles {
  static constexpr int EW = 8;
  static constexpr int MMA2 = kEpiWarp0 + EW;
  static constexpr int THREADS = 32 * (MMA2 + 1);
};

// A ring position kept incrementally: slot and the parity of its current use.
struct Ring {
  int i = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int n) {
    if (++i == n) {
      i = 0;
      ph ^= 1u;
    }
  }
};

// UG consecutive group scales of one row of a scale box, times 1/16 (the
// operand holds 16 x the weights); one or two vector loads.
template <int UG>
__device__ __forceinline__ void load_scales(const uint8_t *srow, int gi0, int sbytes, bool live, float (&sc)[UG]) {
#pragma unroll
  for (int g = 0; g < UG; ++g) sc[g] = 0.0f;
  if (live) {
    if (sbytes == 2) {
      uint32_t h[(UG + 1) / 2];
      const uint8_t *q = srow + 2 * gi0;
      if constexpr (UG == 8) {
        const uint4 t = *reinterpret_cast<const uint4 *>(q);
        h[0] = t.x;
        h[1] = t.y;
        h[2] = t.z;
        h[3] = t.w;
      } else if constexpr (UG == 4) {
        const uint2 t = *reinterpret_cast<const uint2 *>(q);
        h[0] = t.x;
        h[1] = t.y;
      } else if constexpr (UG == 2) {
        h[0] = *reinterpret_cast<const uint32_t *>(q);
      } else {
        h[0] = *reinterpret_cast<const uint16_t *>(q);
      }
#pragma unroll
      for (int g = 0; g < UG; ++g)
        sc[g] = __half2float(__ushort_as_half((unsigned short)(h[g / 2] >> (16 * (g & 1)))));
    } else {
      const float *q = reinterpret_cast<const float *>(srow + 4 * gi0);
      if constexpr (UG >= 4) {
#pragma unroll
        for (int v = 0; v < UG / 4; ++v) {
          const float4 t = reinterpret_cast<const float4 *>(q)[v];
          sc[4 * v] = t.x;
          sc[4 * v + 1] = t.y;
          sc[4 * v + 2] = t.z;
          sc[4 * v + 3] = t.w;
        }
      } else if constexpr (UG == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(q);
        sc[0] = t.x;
        sc[1] = t.y;
      } else {
        sc[0] = q[0];
      }
    }
  }
#pragma unroll
  for (int g = 0; g < UG; ++g) sc[g] = __fmul_rn(sc[g], 0.0625f);
}

template <int MPAD, int MR, int KPG>
__global__ void __launch_bounds__(Roles<MR>::THREADS, 1)
    gemm_w4a8_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_s, const W4GemmParams p) {
  using SH = Shape<MPAD, KPG, (MR <= 8)>;
  constexpr bool PK = MR <= 8;
  constexpr int TOKB = SH::TOKB, TOFF = SH::TOFF;
  constexpr int GPS = SH::GPS, HB = SH::HB, UPH = SH::UPH, UG = SH::UG, UCOLS = SH::UCOLS, NAS = SH::NAS,
                NACC = SH::NACC, ISS = SH::ISS, NPI = SH::NPI;
  constexpr int TOK_BYTES = MPAD * kBlockK;  // one token box
  constexpr int EW = Roles<MR>::EW;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [stage 0 .. nst-1: two packed boxes | kSB token tiles] [scale boxes] [barriers]
  uint8_t *stages = smem;
  uint8_t *sboxes = smem + (size_t)p.nst * p.stage_bytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sboxes + (size_t)kScaleRing * p.sbox_bytes);
  uint64_t *full = bars;                        // [nst]  TMA landed
  uint64_t *empty = full + kMaxStages;          // [nst]  unpacked by all eight warps and its MMAs done
  uint64_t *afull = empty + kMaxStages;         // [NAS]  A slot written
  uint64_t *mdone = afull + 8;                // [kMD]  MMAs of a hand-off done: A slot free, accumulators ready
  uint64_t *accempty = mdone + kMD;             // [NACC] accumulator unit read
  uint64_t *sfull = accempty + kMaxAcc;         // [ring] scale box landed
  uint64_t *sempty = sfull + kScaleRing;        // [ring] scale box used
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + kScaleRing);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * p.tile_rows;
  const int nh = (p.nkb + HB - 1) / HB;  // hand-offs
  auto blocks_of = [&](int ks) { return min(kSB, p.nkb - ks * kSB); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kUnpackWarps + ISS);  // eight unpack warps, one commit per MMA issuer
    }
    for (int a = 0; a < NAS; ++a) mbar_init(&afull[a], HB >= 2 ? 8 : 4);  // the warps writing the slot's blocks
    for (int b = 0; b < kMD; ++b) mbar_init(&mdone[b], SH::SPLIT ? 2 : 1);  // one commit per issuer of the hand-off
    for (int b = 0; b < NACC; ++b) mbar_init(&accempty[b], EW);
    for (int b = 0; b < kScaleRing; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], EW);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  // ---------------------------------------------------------------- producer --
  const uint64_t pol = l2_policy_evict_first();
  int issued = 0, boxes = 0;
  auto issue_stage = [&](int ks) -> bool {
    const int s = ks % p.nst;
    if (ks >= p.nst && !mbar_wait(&empty[s], (uint32_t)((ks / p.nst) - 1) & 1u)) return false;
    if (ks % p.spb == 0) {
      const int bi = ks / p.spb, sb = bi % kScaleRing;
      if (bi >= kScaleRing && !mbar_wait(&sempty[sb], (uint32_t)((bi / kScaleRing) - 1) & 1u)) return false;
      mbar_arrive_expect_tx(&sfull[sb], (uint32_t)(p.tile_rows * p.sbox));
      tma_load_2d(sboxes + (size_t)sb * p.sbox_bytes, &tmap_s, bi * p.sbox, row0, &sfull[sb]);
      ++boxes;
    }
    const int nb = blocks_of(ks), npk = (nb + 1) / 2;
    uint8_t *st = stages + (size_t)s * p.stage_bytes;
    mbar_arrive_expect_tx(&full[s], (uint32_t)(npk * p.box_bytes + nb * TOK_BYTES));
    for (int b = 0; b < npk; ++b)
      tma_load_2d_hint(st + b * p.box_bytes, &tmap_w, (ks * kSB + 2 * b) * kBlockPacked, row0, &full[s], pol);
    for (int j = 0; j < nb; ++j)
      tma_load_2d(st + p.tok_off + j * TOKB + TOFF, &tmap_a, (ks * kSB + j) * kBlockK, 0, &full[s]);
    ++issued;
    return true;
  };
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if constexpr (PK) {
    // the 8 zero rows before every token box, written once (TMA never does)
    for (int i = threadIdx.x; i < p.nst * kSB * (TOFF / 16); i += blockDim.x) {
      const int blk = i / (TOFF / 16), w = i % (TOFF / 16);
      uint8_t *reg = stages + (size_t)(blk / kSB) * p.stage_bytes + p.tok_off + (blk % kSB) * TOKB;
      reinterpret_cast<uint4 *>(reg)[w] = make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_a);
      prefetch_tmap(&tmap_s);
      pdl_wait();
      for (int ks = 0; ks < p.nks; ++ks) {
        if (!issue_stage(ks)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
      }
      pdl_trigger();
      for (int ks = max(0, issued - p.nst); ks < issued; ++ks)
        if (!mbar_wait(&full[ks % p.nst], (uint32_t)(ks / p.nst) & 1u)) set_status(p.status, kStatusTimeout);
      for (int bi = max(0, boxes - kScaleRing); bi < boxes; ++bi)
        if (!mbar_wait(&sfull[bi % kScaleRing], (uint32_t)(bi / kScaleRing) & 1u))
          set_status(p.status, kStatusTimeout);
    }
  } else if (warp == 1 || warp == Roles<MR>::MMA2) {
    // ----------------------------------------------------------------- MMA --
    // Two issuing threads on different schedulers take alternate hand-offs
    // (each MMA instruction costs its thread tens of cycles of issue while
    // the unpack and epilogue warps share the scheduler); their hand-offs use
    // different A slots and accumulator columns, and each commits its own.
    const int mine = warp == 1 ? 0 : 1;
    if (lane == 0 && mine < ISS) {
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MPAD >> 3) << 17) |
                             ((uint32_t)(kRows >> 4) << 24);
      Ring st, as, ac;  // stage, A slot, this issuer's next accumulator unit (of its own NPI)
      int j0 = 0;       // first block of the hand-off within its stage
      for (int h = 0; h < nh; ++h) {
        const int kb0 = h * HB, nbh = min(HB, p.nkb - kb0);
        const bool issue = SH::SPLIT || (h % ISS) == mine;
        bool ok = true;
        if (issue) {
          ok = mbar_wait(&full[st.i], st.ph);  // the stage's token tiles
          ok = ok && mbar_wait(&afull[as.i], as.ph);
          Ring u = ac;
          const int k0 = (SH::SPLIT ? h : h / ISS) * UPH;  // this ring's units so far
          const int rbase = SH::SPLIT ? 0 : mine * NPI;   // this issuer's ring
#pragma unroll
          for (int k = 0; k < UPH; ++k, u.next(NPI))
            if (k0 + k >= NPI) ok = ok && mbar_wait(&accempty[rbase + u.i], u.ph ^ 1u);
        }
        if (!ok) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        if (issue) {
          tc_fence_after();
          const uint8_t *tok = stages + (size_t)st.i * p.stage_bytes + p.tok_off + j0 * TOKB;
          const uint32_t at = tmem + (uint32_t)(as.i * HB * 32);
          // accumulator units of this hand-off: the ring's ac.i, ac.i + 1 (mod NPI)
          const int rbase2 = SH::SPLIT ? 0 : mine * NPI;
          const uint32_t d0 = tmem + (uint32_t)(SH::ACC0 + (rbase2 + ac.i) * UCOLS);
          const uint32_t d1 = tmem + (uint32_t)(SH::ACC0 + (rbase2 + (ac.i + 1 == NPI ? 0 : ac.i + 1)) * UCOLS);
#pragma unroll
          for (int blk = 0; blk < HB; ++blk) {
            // SPLIT: this issuer's half of the blocks only
            if (blk < nbh && (!SH::SPLIT || blk / (HB >= 2 ? HB / 2 : 1) == mine)) {
              const uint8_t *reg = tok + blk * TOKB;
              const uint64_t bdesc = umma_desc_sw128(reg + TOFF);  // tokens in the first rows
              const uint64_t bodd = umma_desc_sw128(reg);          // PK: tokens in rows 8-15
#pragma unroll
              for (int kx = 0; kx < 4; ++kx) {  // K = 32 each: 8 A columns, 32 bytes of the token rows
                const int g = blk * GPS + kx / KPG, u = g / UG, gi = g % UG;
                const uint32_t a = at + (uint32_t)(blk * 32 + 8 * kx);
                if constexpr (PK) {
                  // groups 2q and 2q + 1 share the 16 columns at 16q
                  const uint32_t d = (u == 0 ? d0 : d1) + (uint32_t)((gi / 2) * 16);
                  if ((gi & 1) == 0 && kx % KPG == 0)
                    tc_mma_i8_ts<false>(d, a, bdesc + (uint64_t)(2 * kx), idesc);
                  else if ((gi & 1) == 0)
                    tc_mma_i8_ts<true>(d, a, bdesc + (uint64_t)(2 * kx), idesc);
                  else
                    tc_mma_i8_ts<true>(d, a, bodd + (uint64_t)(2 * kx), idesc);
                } else {
                  const uint32_t d = (u == 0 ? d0 : d1) + (uint32_t)(gi * MPAD);
                  if (kx % KPG == 0)
                    tc_mma_i8_ts<false>(d, a, bdesc + (uint64_t)(2 * kx), idesc);
                  else
                    tc_mma_i8_ts<true>(d, a, bdesc + (uint64_t)(2 * kx), idesc);
                }
              }
            }
          }
          tc_commit(&mdone[h % kMD]);  // frees the A slot and hands the accumulators on
#pragma unroll
          for (int k = 0; k < UPH; ++k) ac.next(NPI);
        }
        as.next(NAS);
        j0 += HB;
        if (j0 == kSB || h == nh - 1) {
          tc_commit(&empty[st.i]);  // each issuer once per stage (after its own MMAs of it, if any)
          st.next(p.nst);
          j0 = 0;
        }
      }
    }
  } else if (warp < kEpiWarp0) {
    // -------------------------------------------------------------- unpack --
    const int set = (warp - 2) >> 2;  // 0: even blocks, 1: odd blocks
    const int quarter = warp & 3;     // TMEM lanes 32 * quarter ..
    const int r = quarter * 32 + lane;  // weight row of the tile
    const bool live = r < p.tile_rows;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    bool stop = false;
    Ring st;
    for (int ks = 0; ks < p.nks && !stop; ++ks, st.next(p.nst)) {
      if (!__all_sync(0xffffffffu, mbar_wait(&full[st.i], st.ph))) {
        if (lane == 0) set_status(p.status, kStatusTimeout);
        break;
      }
      uint8_t *stg = stages + (size_t)st.i * p.stage_bytes;
      const int nb = blocks_of(ks);
      // HB >= 2: both sets write the hand-off's blocks into one slot (set s
      // the blocks j0 + s, j0 + s + 2, ...) and both arrive, even where the
      // last hand-off has fewer blocks; HB = 1: each set its own blocks
      for (int j0 = (HB >= 2 ? 0 : set); j0 < nb; j0 += (HB >= 2 ? HB : 2)) {
        const int h = (ks * kSB + j0) / HB;     // hand-off: its A slot h % NAS, used for the (h / NAS)-th time
        const int slot = h % NAS;
        // the slot's previous hand-off (h - NAS) must have been read by its MMAs
        if (h >= NAS &&
            !__all_sync(0xffffffffu, mbar_wait(&mdone[(h - NAS) % kMD], (uint32_t)((h - NAS) / kMD) & 1u))) {
          if (lane == 0) set_status(p.status, kStatusTimeout);
          stop = true;
          break;
        }
#pragma unroll
        for (int jj = (HB >= 2 ? set : 0); jj < (HB >= 2 ? HB : 1); jj += 2) {
        const int j = j0 + jj;  // this warp's block of the stage
        if (j < nb) {
          // this block's token tile into the A operand's k order (its MMAs
          // wait for this set's arrival below), generic stores made visible
          // to the tensor core's reads
          uint8_t *tok = stg + p.tok_off + j * TOKB + TOFF;
          constexpr int TROWS = PK ? 8 : MPAD;  // rows that can hold tokens
#pragma unroll
          for (int q = 0; q < TROWS * kBlockK / 8 / 128; ++q) {
            uint2 *u = reinterpret_cast<uint2 *>(tok) + quarter * 32 + lane + 128 * q;
            const uint2 x = *u;
            *u = make_uint2(prmt(x.x, x.y, 0x6420), prmt(x.x, x.y, 0x7531));
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc_fence_after();
          uint32_t o[32];
          if (live) {
            // block j is half (j & 1) of packed box j / 2: logical 16-byte
            // chunks 4(j & 1) .. +3 of the row, stored at chunk ^ (row & 7)
            const uint8_t *rowp = stg + (j >> 1) * p.box_bytes + r * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int c = (j & 1) * 4 + q;
              const uint4 v = lds128(rowp + ((c ^ (r & 7)) << 4));
              unpack8x16(v.x, o[8 * q + 0], o[8 * q + 1]);
              unpack8x16(v.y, o[8 * q + 2], o[8 * q + 3]);
              unpack8x16(v.z, o[8 * q + 4], o[8 * q + 5]);
              unpack8x16(v.w, o[8 * q + 6], o[8 * q + 7]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
          }
          // column c of the block holds k = 4c .. 4c + 3
          tc_st32(lane_base + (uint32_t)(slot * HB * 32 + jj * 32), o);
          tc_wait_st();
          tc_fence_before();
        }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[slot]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st.i]);  // this warp is done with the stage's packed boxes
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    if constexpr (PK) {
      // Two sets of four warps (one per TMEM lane quarter), each for half of
      // a unit's groups: one load of its consecutive columns (8 tokens per
      // group).  The two partial sums of a row are added once at the end.
      const int quarter = warp & 3;
      const int set = (warp - kEpiWarp0) >> 2;
      const int r = quarter * 32 + lane;
      const int n = row0 + r;
      const bool row_ok = r < p.tile_rows && n < p.n;
      constexpr int HG = UG / 2;    // groups of this set per unit
      constexpr int CN = HG * 8;    // their columns
      constexpr int NL = CN > 32 ? CN / 32 : 1;  // loads (and waits) of up to 32 columns
      constexpr int LC = CN / NL;
      constexpr int GPL = LC / 8;                // groups per load
      static_assert(CN % NL == 0 && (LC == 8 || LC == 16 || LC == 32), "column split");
      pdl_wait();
      float acc[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
      bool stop = false;
      const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(SH::ACC0 + set * CN);
      Ring er[ISS], sr;  // each issuer's accumulator units (in hand-off order); scale box ring
      int j0 = 0, sk = 0;
      for (int h = 0; h < nh && !stop; ++h) {
        const int nbh = min(HB, p.nkb - h * HB);
        bool ok = true;
        if (j0 == 0 && sk == 0) ok = mbar_wait(&sfull[sr.i], sr.ph);
        ok = ok && mbar_wait(&mdone[h % kMD], (uint32_t)(h / kMD) & 1u);
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) set_status(p.status, kStatusTimeout);
          stop = true;
          break;
        }
        tc_fence_after();
        const int iss = (ISS == 2 && !SH::SPLIT) ? (h & 1) : 0;  // the ring of this hand-off's units
        Ring &ac = er[iss];
        const int slot = iss * NPI + ac.i;
        const int ng = nbh * GPS - set * HG;  // this set's groups that exist (the last hand-off may have one block)
        const uint32_t col = lane_base + (uint32_t)(slot * UCOLS);
        const uint8_t *srow = sboxes + (size_t)sr.i * p.sbox_bytes + (size_t)r * p.sbox;
        float sc[HG];
#pragma unroll
        for (int l = 0; l < NL; ++l) {
          if (l * GPL < ng) {
            uint32_t v[LC];
            if constexpr (LC == 32)
              tc_ld32_nowait(col + (uint32_t)(l * LC), v);
            else if constexpr (LC == 16)
              tc_ld16_nowait(col + (uint32_t)(l * LC), v);
            else
              tc_ld8_nowait(col + (uint32_t)(l * LC), v);
            // the set's scales, loaded while the first load is in flight
            if (l == 0) load_scales<HG>(srow, sk * (kSB * GPS) + j0 * GPS + set * HG, p.sbytes, r < p.tile_rows, sc);
            tc_wait_ld_n<LC>(v);
#pragma unroll
            for (int gg = 0; gg < GPL; ++gg) {
              const int g = l * GPL + gg;
              if (g < ng) {
#pragma unroll
                for (int t = 0; t < 8; ++t) acc[t] = fmaf(i2f_small(v[gg * 8 + t]), sc[g], acc[t]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[slot]);
        ac.next(NPI);
        j0 += HB;
        if (j0 == kSB || h == nh - 1) {  // end of a stage
          j0 = 0;
          if (++sk == p.spb || h == nh - 1) {  // end of a scale box
            if (lane == 0) mbar_arrive(&sempty[sr.i]);
            sr.next(kScaleRing);
            sk = 0;
          }
        }
      }
      // set 1's partial sums -> shared memory (the first ring stage: free
      // once both sets have seen every hand-off's MMAs done) -> set 0 adds
      // them and stores; both barriers are reached on every path
      float *part = reinterpret_cast<float *>(stages);  // [8][128]
      asm volatile("bar.sync 1, %0;" ::"n"(8 * 32) : "memory");
      if (set == 1) {
#pragma unroll
        for (int t = 0; t < 8; ++t) part[t * kRows + r] = acc[t];
      }
      asm volatile("bar.sync 1, %0;" ::"n"(8 * 32) : "memory");
      if (set == 0 && !stop && row_ok) {
        const float *__restrict__ sx = p.sx;
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (t < p.m) p.y[(int64_t)t * p.ldy + n] = __fmul_rn(__fadd_rn(acc[t], part[t * kRows + r]), sx[t]);
      }
    } else {
    // EW / 4 sets of four warps (one per TMEM lane quarter), each for its
    // share of the tokens: per token the groups are summed in order either way
    const int quarter = warp & 3;
    const int half = (warp - kEpiWarp0) >> 2;  // token set
    const int r = quarter * 32 + lane;
    const int n = row0 + r;
    const bool row_ok = r < p.tile_rows && n < p.n;
    constexpr int TPW = MR / (EW / 4);  // tokens of this warp: half * TPW ..
    constexpr int PIECE = TPW % 16 == 0 ? 16 : TPW % 8 == 0 ? 8 : 4;  // accumulator columns per tcgen05.ld
    constexpr int PPG = TPW / PIECE;                                  // loads per group
    constexpr int NPC = UG * PPG;                                     // loads per unit
    constexpr int CAP = TPW >= 16 ? 32 : 64;                          // registers of loads in flight
    constexpr int BP = NPC * PIECE <= CAP ? NPC : CAP / PIECE;        // loads per wait
    pdl_wait();
    float acc[TPW];
#pragma unroll
    for (int t = 0; t < TPW; ++t) acc[t] = 0.0f;
    bool stop = false;
    const uint32_t lane_base =
        tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(SH::ACC0 + half * TPW);
    Ring er[ISS], sr;  // each issuer's accumulator units (taken in hand-off order); scale box ring
    int j0 = 0, sk = 0;  // first block of the hand-off in its stage; stage within the scale box
    for (int h = 0; h < nh && !stop; ++h) {
      const int nbh = min(HB, p.nkb - h * HB);
      bool ok = true;
      if (j0 == 0 && sk == 0) ok = mbar_wait(&sfull[sr.i], sr.ph);
      ok = ok && mbar_wait(&mdone[h % kMD], (uint32_t)(h / kMD) & 1u);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) set_status(p.status, kStatusTimeout);
        stop = true;
        break;
      }
      tc_fence_after();
      const uint8_t *srow = sboxes + (size_t)sr.i * p.sbox_bytes + (size_t)r * p.sbox;
      Ring &ac = er[(ISS == 2 && !SH::SPLIT) ? (h & 1) : 0];
      const int abase = ((ISS == 2 && !SH::SPLIT) ? (h & 1) : 0) * NPI;
#pragma unroll
      for (int u = 0; u < UPH; ++u) {
        const int ng = nbh * GPS - u * UG;  // groups of the unit that exist (the last hand-off may have one block)
        const int slot = abase + ac.i;
        const uint32_t col = lane_base + (uint32_t)(slot * UCOLS);
#pragma unroll
        for (int b0 = 0; b0 < NPC; b0 += BP) {
          uint32_t v[BP][PIECE];
#pragma unroll
          for (int b = 0; b < BP; ++b) {
            const int pc = b0 + b, g = pc / PPG, t0 = (pc % PPG) * PIECE;
            if (pc < NPC && g < ng) {
              if constexpr (PIECE == 4)
                tc_ld4_nowait(col + (uint32_t)(g * MPAD + t0), v[b]);
              else if constexpr (PIECE == 8)
                tc_ld8_nowait(col + (uint32_t)(g * MPAD + t0), v[b]);
              else
                tc_ld16_nowait(col + (uint32_t)(g * MPAD + t0), v[b]);
            }
          }
          // the unit's UG scales lie together in the box row (the box holds
          // tile_rows rows: lanes at and above them read none); loaded while
          // the accumulator loads are in flight
          float sc[UG];
          load_scales<UG>(srow, sk * (kSB * GPS) + j0 * GPS + u * UG, p.sbytes, r < p.tile_rows, sc);
#pragma unroll
          for (int b = 0; b < BP; ++b)
            if (b0 + b < NPC && (b0 + b) / PPG < ng) tc_wait_ld_n<PIECE>(v[b]);
#pragma unroll
          for (int b = 0; b < BP; ++b) {
            const int pc = b0 + b, g = pc / PPG, t0 = (pc % PPG) * PIECE;
            if (pc < NPC && g < ng) {
#pragma unroll
              for (int i = 0; i < PIECE; ++i) acc[t0 + i] = fmaf(i2f_small(v[b][i]), sc[g], acc[t0 + i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[slot]);
        ac.next(NPI);
      }
      j0 += HB;
      if (j0 == kSB || h == nh - 1) {  // end of a stage
        j0 = 0;
        if (++sk == p.spb || h == nh - 1) {  // end of a scale box
          if (lane == 0) mbar_arrive(&sempty[sr.i]);
          sr.next(kScaleRing);
          sk = 0;
        }
      }
    }
    if (!stop && row_ok) {
      const float *__restrict__ sx = p.sx;
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        const int tt = half * TPW + t;
        if (tt < p.m) p.y[(int64_t)tt * p.ldy + n] = __fmul_rn(acc[t], sx[tt]);
      }
    }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// u8 2-D tensor map over `rows` rows of `row_bytes` bytes (stride ld), box [box_cols x box_rows], no swizzle
bool make_plain_map(CUtensorMap *map, const void *base, int64_t rows, int64_t row_bytes, int64_t ld, int box_cols,
                    int box_rows) {
  return make_map(map, base, rows, row_bytes, ld, box_rows, box_cols, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int MPAD, int MR, int KPG>
cudaError_t launch_one(const CUtensorMap &mw, const CUtensorMap &ma, const CUtensorMap &ms, const W4GemmParams &p,
                       int grid, size_t smem, cudaStream_t stream, int device) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  std::call_once(once[device & 63], [&] {
    err[device & 63] = cudaFuncSetAttribute(gemm_w4a8_tc_kernel<MPAD, MR, KPG>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            device_props(device).smem_optin);
  });
  if (err[device & 63] != cudaSuccess) return err[device & 63];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(Roles<MR>::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled(stream)) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemm_w4a8_tc_kernel<MPAD, MR, KPG>, mw, ma, ms, p);
}

template <int KPG>
cudaError_t launch_kpg(int mpad, int mr, const CUtensorMap &mw, const CUtensorMap &ma, const CUtensorMap &ms,
                       const W4GemmParams &p, int grid, size_t smem, cudaStream_t stream, int device) {
  switch (mpad) {
    case 16:
      return mr <= 8 ? launch_one<16, 8, KPG>(mw, ma, ms, p, grid, smem, stream, device)
                     : launch_one<16, 16, KPG>(mw, ma, ms, p, grid, smem, stream, device);
    case 32: return launch_one<32, 32, KPG>(mw, ma, ms, p, grid, smem, stream, device);
    case 48: return launch_one<48, 48, KPG>(mw, ma, ms, p, grid, smem, stream, device);
    default: return launch_one<64, 64, KPG>(mw, ma, ms, p, grid, smem, stream, device);
  }
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
  const int mr = a.m <= 8 ? 8 : mpad;
  const int kpg = (int)(a.group / 32);
  const int gps = 4 / kpg;
  p.nkb = (int32_t)((a.k + kBlockK - 1) / kBlockK);
  p.nks = (p.nkb + kSB - 1) / kSB;
  p.sbytes = a.stype == kScaleF16 ? 2 : 4;
  const int64_t slots = dp.sm_count;
  const int64_t waves = (a.n + slots * kRows - 1) / (slots * kRows);
  const int64_t even = (a.n + waves * slots - 1) / (waves * slots);
  p.tile_rows = (int32_t)std::min<int64_t>(kRows, (std::max<int64_t>(even, 16) + 15) / 16 * 16);
  const int grid = (int)((a.n + p.tile_rows - 1) / p.tile_rows);
  p.box_bytes = p.tile_rows * 128;  // a multiple of 2048: every box and token tile stays 1024-aligned
  p.tok_off = 2 * p.box_bytes;
  // token tiles: at most 8 tokens keep 8 zero rows before the box (paired accumulators)
  p.stage_bytes = p.tok_off + kSB * (mr <= 8 ? 24 : mpad) * kBlockK;
  // scale boxes: a power of two bytes per row, at least 16 (TMA boxes and
  // their x coordinates are multiples of 16 bytes)
  p.sbox = std::max(16, kSB * gps * p.sbytes);
  p.spb = p.sbox / (kSB * gps * p.sbytes);
  p.sbox_bytes = (p.tile_rows * p.sbox + 127) / 128 * 128;
  const int fixed = 1024 /* alignment */ + kScaleRing * p.sbox_bytes + 512 /* barriers */;
  const int nst = std::min({kMaxStages, (dp.smem_optin - fixed) / p.stage_bytes, (int)p.nks,
                            std::max(1, env_int("KS_B200_W4GEMM_STAGES", kMaxStages))});
  if (nst < 1) return cudaErrorNotSupported;
  p.nst = nst;
  CUtensorMap mw, ma, ms;
  if (!make_map(&mw, a.w, a.n, a.k / 2, a.wstride, p.tile_rows, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&ma, a.a, a.m, a.k, a.lda, mpad) ||
      !make_plain_map(&ms, a.s, a.n, a.k / a.group * p.sbytes, a.sstride * p.sbytes, p.sbox, p.tile_rows))
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)fixed + (size_t)nst * p.stage_bytes;
  switch (kpg) {
    case 1: return launch_kpg<1>(mpad, mr, mw, ma, ms, p, grid, smem, stream, device);
    case 2: return launch_kpg<2>(mpad, mr, mw, ma, ms, p, grid, smem, stream, device);
    default: return launch_kpg<4>(mpad, mr, mw, ma, ms, p, grid, smem, stream, device);
  }
}

}  // namespace ksb
