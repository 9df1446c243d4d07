// ks_quant.cu -- per-token int8 quantisation of f32 activations.
//
// The activation quantisation the W4A8 path assumes (zero point 0): for each
// token (row of x), s = max|x| / 127 (one IEEE division; 1 when the row is all
// zeros) and q = sat_i8(round_half_even(x / s)), the same rule as the decode
// kernels' input preparation and the oracle's quantize_per_token.  One CTA
// per token: a max reduction, then one exact division per element.  Small
// (tokens x cols bytes); used ahead of the batched W4A8 GEMM.

#include <cstdint>

#include "ks_internal.h"
#include "ks_stream.cuh"

namespace ksb {

namespace {

constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads) quantize_tokens_kernel(const float *__restrict__ x, int64_t ldx,
                                                                        int64_t cols, int8_t *__restrict__ q,
                                                                        int64_t ldq, float *__restrict__ scales) {
  __shared__ float red[kQuantThreads / 32];
  const float *xr = x + (int64_t)blockIdx.x * ldx;
  float m = 0.0f;
  for (int64_t i = threadIdx.x; i < cols; i += kQuantThreads) m = fmaxf(m, fabsf(xr[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = 0.0f;
#pragma unroll
  for (int w = 0; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  int8_t *qr = q + (int64_t)blockIdx.x * ldq;
  for (int64_t i = threadIdx.x; i < cols; i += kQuantThreads) qr[i] = (int8_t)quant_rne_byte(xr[i], s);
  if (threadIdx.x == 0) scales[blockIdx.x] = s;
}

}  // namespace

cudaError_t launch_quantize_tokens(const float *x, int64_t ldx, int64_t n, int64_t cols, int8_t *q, int64_t ldq,
                                   float *scales, cudaStream_t stream) {
  if (n <= 0 || cols <= 0) return cudaSuccess;
  if (n > 0x7FFFFFFF) return cudaErrorInvalidValue;
  quantize_tokens_kernel<<<(unsigned)n, kQuantThreads, 0, stream>>>(x, ldx, cols, q, ldq, scales);
  return cudaGetLastError();
}

}  // namespace ksb
