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
// One CTA per 128 weight rows, warp-specialised:
//   warp 0  TMA producer: per 128-byte K block, one 2-D tiled copy of the
//           weight tile [128 x 128 B] and one of the activation tile
//           [Mpad x 128 B], both 128-byte swizzled, into a ring of stages.
//           No multicast anywhere.
//   warp 1  allocates TMEM, issues 4 x tcgen05.mma (K = 32 each) per stage,
//           frees the stage with tcgen05.commit, finally commits to the
//           accumulator barrier; deallocates TMEM at the end.
//   warps 2-5 epilogue: tcgen05.ld the accumulator rows (one TMEM lane per
//           weight row), requantise in the order written above with IEEE
//           round-to-nearest operations and store int8.
//
// Every mbarrier wait is bounded (about one second); on a timeout the kernel
// records it in the status word, lets in-flight copies and MMAs drain, frees
// TMEM and returns.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "ks_internal.h"
#include "ks_ptx.cuh"

namespace ksb {

namespace {

constexpr int kTileRows = 128;   // weight rows per CTA (MMA M)
constexpr int kKBlock = 128;     // K bytes per stage (one 128-B swizzle row)
constexpr int kGemmThreads = 192;
constexpr int kMaxTokens = 256;  // MMA N limit

struct GemmParams {
  const float *sa;
  const float *ws;
  float out_scale;
  int8_t *out;
  int64_t ldo;
  int32_t *acc_out;  // optional
  int32_t m, n, k;
  int32_t mpad;      // tokens padded to a multiple of 16
  int32_t nkb;       // K blocks
  int32_t nst;       // stages
  int32_t stage_bytes;
  int32_t b_bytes;   // activation tile bytes per stage
  uint32_t tmem_cols;
  uint32_t *status;
};

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, int x, int y,
                                                 uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// K-major, 128-byte swizzled operand tile: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(const void *smem_tile) {
  const uint64_t addr = smem_u32(smem_tile);
  return ((addr >> 4) & 0x3FFFull)   // start address
         | (1ull << 16)              // leading byte offset (unused for swizzled K-major)
         | (64ull << 32)             // stride byte offset: 1024 B >> 4
         | (1ull << 46)              // descriptor version (sm_100)
         | (2ull << 61);             // layout: 128-byte swizzle
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ int8_t requant(int32_t acc, float sa, float ws, float out_scale) {
  float t = __fmul_rn((float)acc, sa);
  t = __fmul_rn(t, ws);
  t = __fdiv_rn(t, out_scale);
  t = rintf(t);  // round half to even
  t = fminf(fmaxf(t, -128.0f), 127.0f);
  return (int8_t)(int)t;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                      const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *stages = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)p.nst * p.stage_bytes);
  uint64_t *empty = full + p.nst;
  uint64_t *accum = empty + p.nst;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kTileRows;

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
      const uint32_t tx = (uint32_t)(kTileRows * kKBlock + p.b_bytes);
      int issued = 0;
      for (int kb = 0; kb < p.nkb; ++kb) {
        const int s = kb % p.nst;
        if (kb >= p.nst && !mbar_wait(&empty[s], (uint32_t)((kb / p.nst) - 1) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        tma_load_2d_hint(st, &tmap_w, kb * kKBlock, row0, &full[s], pol);
        tma_load_2d(st + kTileRows * kKBlock, &tmap_a, kb * kKBlock, 0, &full[s]);
        ++issued;
      }
      for (int kb = max(0, issued - p.nst); kb < issued; ++kb) {
        if (!mbar_wait(&full[kb % p.nst], (uint32_t)(kb / p.nst) & 1u)) set_status(p.status, kStatusTimeout);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      const uint32_t idesc = (2u << 4)                         // D: s32
                             | (1u << 7) | (1u << 10)          // A, B: signed int8
                             | ((uint32_t)(p.mpad >> 3) << 17) // N
                             | ((uint32_t)(kTileRows >> 4) << 24);  // M
      for (int kb = 0; kb < p.nkb; ++kb) {
        const int s = kb % p.nst;
        if (!mbar_wait(&full[s], (uint32_t)(kb / p.nst) & 1u)) {
          set_status(p.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint8_t *st = stages + (size_t)s * p.stage_bytes;
        const uint64_t adesc = umma_desc_sw128(st);
        const uint64_t bdesc = umma_desc_sw128(st + kTileRows * kKBlock);
#pragma unroll
        for (int kk = 0; kk < kKBlock / 32; ++kk) {
          // advance the start address by 32 bytes (K = 32 int8) per step
          tc_mma_i8(tmem_d, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2), idesc,
                    (kb > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(accum);  // fires once every MMA issued above has completed
    }
  } else {
    // ---------------------------------------------------------- epilogue --
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int r = quarter * 32 + lane;
    const int n = row0 + r;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(accum, 0));
    tc_fence_after();
    const bool aborted = __shfl_sync(0xffffffffu, *abort_flag, 0) != 0;
    if (!ok) {
      if (lane == 0) set_status(p.status, kStatusTimeout);
    } else if (!aborted) {
      const float wsn = n < p.n ? __ldg(p.ws + n) : 0.0f;
      for (int c0 = 0; c0 < p.mpad; c0 += 16) {
        uint32_t v[16];
        tc_ld16(tmem_d + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, v);
        if (n < p.n) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = c0 + j;
            if (m < p.m) {
              const int32_t acc = (int32_t)v[j];
              p.out[(int64_t)m * p.ldo + n] = requant(acc, __ldg(p.sa + m), wsn, p.out_scale);
              if (p.acc_out) p.acc_out[(int64_t)m * p.n + n] = acc;
            }
          }
        }
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

// ------------------------------------------------------------- host side --
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// int8 matrix [rows, cols] with row stride ld bytes; box [box_rows, 128 B].
bool make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {(cuuint32_t)kKBlock, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_shape_ok(const GemmI8Launch &a) {
  const auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return a.m >= 1 && a.m <= kMaxTokens && a.n >= 1 && a.n < (int64_t(1) << 31) && a.k >= 1 &&
         a.k < (int64_t(1) << 31) && a.lda % 16 == 0 && a.ldw % 16 == 0 && al16(a.a) && al16(a.w) &&
         encode_fn() != nullptr;
}

}  // namespace

int gemm_i8_path(const GemmI8Launch &a) { return tc_shape_ok(a) ? 1 : 0; }

cudaError_t launch_gemm_i8(const GemmI8Launch &a, cudaStream_t stream, int device) {
  GemmParams p{};
  p.sa = a.sa;
  p.ws = a.ws;
  p.out_scale = a.out_scale;
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
  p.stage_bytes = kTileRows * kKBlock + p.b_bytes;  // multiple of 1024
  uint32_t cols = 32;
  while (cols < (uint32_t)p.mpad) cols <<= 1;
  p.tmem_cols = cols;
  const int reserve = 1024 /* alignment slack */ + 1024 /* barriers */;
  int nst = (dp.smem_optin - reserve) / p.stage_bytes;
  nst = std::min(nst, 8);
  nst = std::min(nst, p.nkb);
  if (nst < 1) return cudaErrorInvalidValue;
  p.nst = nst;
  CUtensorMap mw, ma;
  if (!make_map(&mw, a.w, a.n, a.k, a.ldw, kTileRows) || !make_map(&ma, a.a, a.m, a.k, a.lda, p.mpad))
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)reserve + (size_t)nst * p.stage_bytes;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[device & 63], [&] {
    attr_err[device & 63] =
        cudaFuncSetAttribute(gemm_i8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dp.smem_optin);
  });
  if (attr_err[device & 63] != cudaSuccess) return attr_err[device & 63];
  const int grid = (int)((a.n + kTileRows - 1) / kTileRows);
  gemm_i8_tc_kernel<<<grid, kGemmThreads, smem, stream>>>(mw, ma, p);
  return cudaGetLastError();
}

}  // namespace ksb
