// ks_import.cu -- GGML Q4_0 weights -> the native W4A8 layout, on the GPU.
//
// The conversion is the reference's offline GGML -> native path
// (docs/design/DES-015-quantized-layout-abi-and-integration-conversion-paths.md:148-179):
// decode every Q4_0 block to f32, then requantise each native group with a
// positive scale:
//
//   block (18 bytes): f16 d, then 16 bytes qs; element j (0..15) is
//                     (qs[j] & 0x0F) - 8, element j + 16 is (qs[j] >> 4) - 8,
//                     both times d
//   group g:          lo = min, hi = max of the decoded values
//                     scale = max(hi / 7, -lo / 8), or 1 if that is 0
//                     q = clamp(rne(v / scale), -8, 7)
//   native layout:    value k in byte k/2, low nibble for even k
//
// Every step is exact or one IEEE round-to-nearest operation (the decoded
// value (q - 8) * d has at most 15 significant bits; hi / 7 and v / scale are
// single divisions; -lo / 8 is exact), so the result is bit-identical to the
// same steps in f32 on a CPU.  "round" is round half to even, the reference's
// quantisation convention.  With f16 scales the f32 scale is rounded to f16
// first (and kept positive and finite) and the values are quantised with the
// f16 value, so dequantisation uses exactly the scale the codes were made with.
//
// One thread per native group.  Each block is read once (nine 16-bit loads:
// blocks are 18 bytes apart, so 2-byte aligned) and kept in registers.  A
// block's 32 values are (n - 8) * d for its 16 possible nibbles n, so the
// codes are computed once per nibble value (16 per block) and the 32 nibbles
// are mapped through that table; the code for value v is rint(v / scale)
// clamped, computed as rint(v * RN(1 / scale)) except within 2^-14 of a
// rounding tie, where the division is taken (both round to the same integer
// otherwise: they lie within |v / scale| * 2^-23 <= 2.4e-6 of the quotient
// for |v / scale| <= 8.5; beyond that both clamp).  Packed bytes leave as
// 16-byte stores.  HBM-bound: 18 bytes read and 16 + 4 (or 2) written per
// 32 weights.

#include <cuda_fp16.h>

#include <cstdint>

#include "ks_internal.h"

namespace ksb {

namespace {

constexpr int kQ4Block = 18;  // bytes per 32-element Q4_0 block

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }

// rint(v / s) clamped to [-8, 7], as a nibble; inv = RN(1 / s) (0: divide)
__device__ __forceinline__ uint32_t code_of(float v, float s, float inv) {
  float q;
  if (inv != 0.0f) {
    q = rintf(__fmul_rn(v, inv));
    const float t = __fmul_rn(v, inv);
    const float r = __fsub_rn(t, floorf(t));  // in [0, 1)
    if (fabsf(__fsub_rn(r, 0.5f)) < 0x1p-14f) q = rintf(__fdiv_rn(v, s));
  } else {
    q = rintf(__fdiv_rn(v, s));
  }
  q = fminf(fmaxf(q, -8.0f), 7.0f);
  return (uint32_t)((int)q) & 0xFu;
}

template <int NB>  // Q4_0 blocks per native group (group_size / 32)
__global__ void __launch_bounds__(256)
    import_q4_0_kernel(const uint8_t *__restrict__ src, int64_t src_stride, int64_t rows, int64_t groups,
                       uint8_t *__restrict__ packed, int64_t packed_stride, void *scales, int scale_type,
                       int64_t scale_stride) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= rows * groups) return;
  const int64_t r = gid / groups, g = gid % groups;
  const uint8_t *blk0 = src + r * src_stride + g * NB * kQ4Block;
  uint32_t qs[NB][4];  // the 16 nibble bytes of each block
  float d[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const uint8_t *blk = blk0 + b * kQ4Block;
    d[b] = __half2float(__ushort_as_half(ld_u16(blk)));
#pragma unroll
    for (int w = 0; w < 4; ++w)
      qs[b][w] = (uint32_t)ld_u16(blk + 2 + 4 * w) | ((uint32_t)ld_u16(blk + 4 + 4 * w) << 16);
  }
  // lo / hi of the decoded values: (n - 8) * d over each block's nibbles
  float lo = 0.0f, hi = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    int nmin = 15, nmax = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int n = (int)((qs[b][w] >> (4 * k)) & 0xFu);
        nmin = min(nmin, n);
        nmax = max(nmax, n);
      }
    const float a = __fmul_rn((float)(nmin - 8), d[b]), c = __fmul_rn((float)(nmax - 8), d[b]);
    const float blo = fminf(a, c), bhi = fmaxf(a, c);
    lo = b == 0 ? blo : fminf(lo, blo);
    hi = b == 0 ? bhi : fmaxf(hi, bhi);
  }
  float scale = fmaxf(__fdiv_rn(hi, 7.0f), __fmul_rn(-lo, 0.125f));
  if (scale == 0.0f) scale = 1.0f;
  if (scale_type == kScaleF16) {
    float hs = __half2float(__float2half_rn(scale));
    if (!(hs > 0.0f)) hs = __half2float(__ushort_as_half((unsigned short)0x0001));  // smallest positive f16
    if (isinf(hs)) hs = 65504.0f;                                               // largest finite f16
    scale = hs;
    reinterpret_cast<__half *>(scales)[r * scale_stride + g] = __float2half_rn(hs);
  } else {
    reinterpret_cast<float *>(scales)[r * scale_stride + g] = scale;
  }
  const float recip = __fdiv_rn(1.0f, scale);
  const float inv = isfinite(recip) ? recip : 0.0f;
  uint8_t *dst = packed + r * packed_stride + g * NB * 16;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    // code of each nibble value n: 16 x 4 bits
    uint64_t tbl = 0;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      tbl |= (uint64_t)code_of(__fmul_rn((float)(n - 8), d[b]), scale, inv) << (4 * n);
    // block element e: nibble (qs byte e) low for e < 16, (qs byte e - 16) high
    // for e >= 16; native position e: word e / 8, nibble e % 8
    uint32_t out[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int byte = e & 15;
      const uint32_t nib = (qs[b][byte >> 2] >> (8 * (byte & 3) + (e >= 16 ? 4 : 0))) & 0xFu;
      out[e >> 3] |= (uint32_t)((tbl >> (4 * nib)) & 0xFu) << (4 * (e & 7));
    }
    reinterpret_cast<uint4 *>(dst)[b] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

}  // namespace

cudaError_t launch_import_q4_0(const ImportQ4Launch &a, cudaStream_t stream) {
  const int64_t groups = a.cols / a.group;
  const int64_t total = a.rows * groups;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const unsigned grid = (unsigned)((total + threads - 1) / threads);
  switch (a.group / 32) {
#define KS_IMPORT_CASE(NB)                                                                                   \
  case NB:                                                                                                   \
    import_q4_0_kernel<NB><<<grid, threads, 0, stream>>>(a.src, a.src_stride, a.rows, groups, a.packed,     \
                                                         a.packed_stride, a.scales, a.scale_type,           \
                                                         a.scale_stride);                                   \
    break;
    KS_IMPORT_CASE(1)
    KS_IMPORT_CASE(2)
    KS_IMPORT_CASE(4)
    KS_IMPORT_CASE(8)
#undef KS_IMPORT_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace ksb
