// ks_stream.cuh -- device building blocks shared by the streaming GEMV
// kernels (ks_gemv.cu) and the persistent decode-layer kernel (ks_decode.cu):
// work-item and epilogue descriptors, the W4A8 and INT8 per-row operators
// (weights and scale rows staged in shared memory, activations prepared once
// per CTA), consumer-warp barriers and reductions, and the f32-activation
// prologue (RMSNorm / per-token quantisation).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "ks_internal.h"
#include "ks_ptx.cuh"

namespace ksb {

constexpr int kMaxStages = 16;
constexpr int kBarBytes = 1024;      // barrier area at the start of shared memory
constexpr int kMaxItems = 64;        // matrices per launch
constexpr int kSmemSingle = 108 * 1024;  // two CTAs per SM (228 KB, 1 KB reserved each)
constexpr int kSmemBatch = 220 * 1024;   // one CTA per SM
constexpr int kMaxStreamChunks = 512;    // W4A8 rows up to 16384 columns, INT8 up to 8192

struct GemvItem {
  const int8_t *x;
  const uint8_t *w;
  const uint8_t *s;  // scales (W4A8) or per-channel dequant scales (INT8 f32 out)
  void *y;
};
constexpr int kMaxPeers = 8;
// Per-launch matrix list.  When npeers > 0 the launch is a sharded GEMV whose
// outputs are gathered by peer stores: the output of row r of matrix m goes to
// peer_y[p][m * mstride + row_offset + r] of every rank p (this rank
// included).  A CTA collects its rows of a matrix in shared memory and, once
// the matrix is done, its consumer threads write that contiguous slice to
// every rank with coalesced stores (a warp writes 128 consecutive bytes of
// one rank's buffer per instruction, instead of one 4-byte NVLink write per
// row and rank).  After its last store each CTA adds 1 to peer_cnt[p] for
// every rank p (system scope, after a system-scope fence); peer_cnt[p] is
// the word of rank p's counter array that counts this rank's arrivals.
struct GemvItems {
  GemvItem it[kMaxItems];
  float *peer_y[kMaxPeers];
  uint32_t *peer_cnt[kMaxPeers];
  int64_t mstride;
  int64_t row_offset;
  int32_t npeers;
};

// Decode-layer fusion: where a launch's activations come from and what its
// epilogue does.  The zero-initialised value is the plain GEMV.
enum XMode : int32_t {
  kXInt8 = 0,     // int8 activations, scale from the arguments
  kXF32 = 1,      // f32 activations, quantised per token (max |x| / 127, RNE)
  kXRmsNorm = 2,  // f32 activations, RMSNorm (weight norm_w, eps), then quantised
  kXF32Amax = 3,  // f32 activations quantised with the max |x| in *amax_in
};
enum EpiMode : int32_t {
  kEpiPlain = 0,
  kEpiResidual = 1,  // y[r] = v + res[r]
  kEpiSiluMul = 2,   // matrix 1 of the launch: act[r] = silu(gate[r]) * v, max |act| into *amax_out
};
struct LayerExt {
  int32_t xmode;
  int32_t epi;
  const float *xf;
  const float *norm_w;
  float eps;
  const uint32_t *amax_in;
  const float *res;
  const float *gate;
  float *act_out;
  uint32_t *amax_out;
  uint32_t *reset_amax;  // CTA 0 sets it to 0 after the wait (first launch of a layer)
  int8_t *xq_out;        // optional: the quantised activations (written by CTA 0)
  float *xs_out;         // optional: their scale
};

// Where a row's result goes.
struct OutRef {
  void *y;               // local output (npeers == 0)
  const GemvItems *items;
  int64_t peer_off;      // m * mstride + row_offset
  const LayerExt *ext;
  int m;
  float *ostage;         // npeers > 0: this CTA's rows of matrix m, in shared memory
  int64_t r0;            // first row of this CTA
  // the epilogue's global operand for row r (residual or gate value), loaded
  // before the row's dot product
  struct Pre {
    float v;
  };
  __device__ __forceinline__ Pre pre(int64_t r, bool ok) const;
  __device__ __forceinline__ void store(int64_t r, float v, Pre p) const;
};

__device__ __forceinline__ OutRef::Pre OutRef::pre(int64_t r, bool ok) const {
  if (!ok || items->npeers != 0) return {0.0f};
  if (ext->epi == kEpiResidual) return {ext->res[r]};
  if (ext->epi == kEpiSiluMul && m == 1) return {ext->gate[r]};
  return {0.0f};
}

__device__ __forceinline__ void store_f32(const OutRef &o, int64_t r, float v, OutRef::Pre p) {
  const int np = o.items->npeers;
  if (np == 0) {
    const LayerExt &e = *o.ext;
    float out = v;
    if (e.epi == kEpiResidual) {
      out = __fadd_rn(v, p.v);
    } else if (e.epi == kEpiSiluMul && o.m == 1) {
      const float g = p.v;
      const float a = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), v);
      e.act_out[r] = a;
      atomicMax(e.amax_out, __float_as_uint(fabsf(a)));
    }
    reinterpret_cast<float *>(o.y)[r] = out;
  } else {
    o.ostage[r - o.r0] = v;  // written to the ranks by flush_peer_rows
  }
}

// Write this CTA's staged rows [r0, r0 + n) of one matrix to every rank's
// gathered buffer: consecutive threads take consecutive rows of one rank, so
// each warp store instruction covers up to 128 contiguous bytes.  Every
// consumer thread calls it after the consumer barrier that follows the
// matrix's last row.
template <int CW>
__device__ __forceinline__ void flush_peer_rows(const GemvItems &items, const float *ostage, int64_t off, int n,
                                                int ctid) {
  const int total = n * items.npeers;
  for (int i = ctid; i < total; i += CW * 32) {
    const int p = i / n;
    const int e = i - p * n;
    items.peer_y[p][off + e] = ostage[e];
  }
}

__device__ __forceinline__ void OutRef::store(int64_t r, float v, Pre p) const { store_f32(*this, r, v, p); }

// Geometry of the streamed weight blocks, shared by all stream kernels.
struct StreamGeom {
  int64_t wstride;      // bytes between weight rows
  int64_t sstride;      // bytes between side rows
  int64_t rows;
  int32_t count;        // matrices in this launch
  int32_t n_cta;
  int32_t rps;          // rows per stage (even)
  int32_t nst;          // stages in the ring
  int32_t row_bytes;    // streamed bytes per weight row
  int32_t srow_bytes;   // streamed bytes per side row (0: none)
  int32_t stage_bytes;
  int32_t xbuf_bytes;   // one prepared-activation buffer
  int32_t ostage_bytes; // one output staging buffer (peer-gather launches; else 0)
  int32_t w_contig;     // wstride == row_bytes: one copy per stage
  int32_t s_contig;
  int32_t x_al16;       // every activation vector 16-byte aligned
  int32_t l2_ahead;     // stages prefetched into L2 ahead of the ring
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
  // 0 < bits < +inf; negative values, zero, inf and nan fail.  Kernels
  // keep max(bits - 1) over the scales they read and test it once.
  static constexpr uint32_t kBadFrom = 0x7F7FFFFFu;
  __device__ __forceinline__ static bool bad(uint32_t b) { return (b - 1u) >= kBadFrom; }
  __device__ __forceinline__ static float f32(uint32_t b) { return __uint_as_float(b); }
};
template <>
struct ScaleBits<__half> {
  static constexpr int kBytes = 2;
  __device__ __forceinline__ static uint32_t load(const uint8_t *p) { return lds_u16(p); }
  __device__ __forceinline__ static uint32_t gload(const __half *p) {
    return __half_as_ushort(__ldg(p));
  }
  static constexpr uint32_t kBadFrom = 0x7BFFu;
  __device__ __forceinline__ static bool bad(uint32_t b) { return (b - 1u) >= kBadFrom; }
  __device__ __forceinline__ static float f32(uint32_t b) {
    return __half2float(__ushort_as_half((unsigned short)b));
  }
};

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two partial sums of the same warp reduced together: after the first
// exchange lanes 0-15 hold a's partials and lanes 16-31 b's, so the rest of
// the butterfly carries one value.  Lane 0 ends with sum(a), lane 16 with
// sum(b).  Fixed order: bitwise reproducible.
template <typename T>
__device__ __forceinline__ T warp_sum_pair(T a, T b, int lane) {
  const bool upper = (lane & 16) != 0;
  T keep = upper ? b : a;
  const T give = upper ? a : b;
  keep += __shfl_xor_sync(0xffffffffu, give, 16);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
  return keep;
}

template <int WORDS>
__device__ __forceinline__ void load_words(const int8_t *p, bool al16, uint32_t (&X)[WORDS]) {
  if (al16) {
#pragma unroll
    for (int i = 0; i < WORDS; i += 4) {
      const uint4 a = __ldg(reinterpret_cast<const uint4 *>(p) + i / 4);
      X[i] = a.x; X[i + 1] = a.y; X[i + 2] = a.z; X[i + 3] = a.w;
    }
  } else {
    const uint8_t *q = reinterpret_cast<const uint8_t *>(p);
#pragma unroll
    for (int i = 0; i < WORDS; ++i)
      X[i] = (uint32_t)q[4 * i] | ((uint32_t)q[4 * i + 1] << 8) | ((uint32_t)q[4 * i + 2] << 16) |
             ((uint32_t)q[4 * i + 3] << 24);
  }
}

// ---------------------------------------------------------------- W4A8 op --
struct W4A8OpParams {
  int32_t chunks;  // 32-element chunks per row (cols / 32)
  int32_t gshift;  // log2(group / 32)
  float sx;
  int32_t zx, zw;
};

// int32 dot of one 32-element chunk (packed word v) against prepared x.
template <bool ZX>
__device__ __forceinline__ int w4a8_chunk_dot(const uint4 v, const uint4 xe, const uint4 xo, int kc, int zx) {
  const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
  const uint32_t e[4] = {xe.x, xe.y, xe.z, xe.w};
  const uint32_t o[4] = {xo.x, xo.y, xo.z, xo.w};
  int lo = 0, hi = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    lo = dp4a_us(and_xor(vw[q], 0x0F0F0F0Fu, 0x08080808u), e[q], lo);
    hi = dp4a_us(and_xor(vw[q], 0xF0F0F0F0u, 0x80808080u), o[q], hi);
  }
  int acc = lo + (hi >> 4) - kc;
  if (ZX) {
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

// Prepared activations, per 32-element chunk c: at xb + 16c the even-k bytes
// of the chunk's four packed words, at xb + 16*chunks + 16c the odd-k bytes,
// and at xb + 32*chunks + 4c the constant kc = (8 + zw) * sum(x - zx).  Lanes
// read consecutive chunks, so both byte planes are read without bank
// conflicts (16 contiguous bytes per lane).
// ZX: input zero point != 0.
template <typename ST, int NCPL, bool ZX>
struct W4A8Op {
  using Params = W4A8OpParams;
  using SB = ScaleBits<ST>;
  static constexpr int kRawWords = 8;  // 32 activation bytes per chunk
  static constexpr int kChunkK = 32;
  __device__ __forceinline__ static void set_sx(const Params &p, uint8_t *xb, float sx) {
    *reinterpret_cast<float *>(xb + 36 * p.chunks) = sx;
  }
  __device__ __forceinline__ static float default_sx(const Params &p) { return p.sx; }
  struct Lane {
    float sx;  // activation scale of the current matrix (from the prepared buffer)
  };

  // 36 bytes per chunk, then the activation scale
  static int xbuf_bytes(int chunks) { return ((chunks * 36 + 4 + 127) / 128) * 128; }


  __device__ __forceinline__ static void load_raw(const int8_t *x, int c, bool al16, uint32_t (&raw)[8]) {
    load_words<8>(x + 32 * c, al16, raw);
  }

  __device__ __forceinline__ static void store_prep(const Params &p, const uint32_t (&X)[8], int c, uint8_t *xb) {
    uint32_t e[4], o[4];
    int sumx = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      e[q] = prmt(X[2 * q], X[2 * q + 1], 0x6420);
      o[q] = prmt(X[2 * q], X[2 * q + 1], 0x7531);
      sumx = dp4a_ss(X[2 * q], 0x01010101u, sumx);
      sumx = dp4a_ss(X[2 * q + 1], 0x01010101u, sumx);
    }
    *reinterpret_cast<uint4 *>(xb + 16 * c) = make_uint4(e[0], e[1], e[2], e[3]);
    *reinterpret_cast<uint4 *>(xb + 16 * p.chunks + 16 * c) = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<int *>(xb + 32 * p.chunks)[c] = (8 + p.zw) * (sumx - 32 * p.zx);
  }

  __device__ __forceinline__ static void lane_init(const Params &p, Lane &L, const uint8_t *xb, int) {
    L.sx = *reinterpret_cast<const float *>(xb + 36 * p.chunks);
  }

  // Two rows (b valid if has_b) whose weights and scale rows are in shared
  // memory -> out.store(row, value).  Returns max(scale bits - 1) over the
  // scales read.
  template <class Out>
  __device__ __forceinline__ static uint32_t rows2(const Params &p, const Lane &, const uint8_t *xb,
                                                   const uint8_t *wa, const uint8_t *sa, const uint8_t *wb,
                                                   const uint8_t *sb, const Out &out, const GemvItem &, int64_t ga,
                                                   bool has_b, int lane, const Lane &Lx) {
    // lane 0 writes row a, lane 16 row b; the epilogue's own global loads
    // (a residual, a gate value) are issued now and land during the dot product
    const int64_t mine = ga + (lane == 16 ? 1 : 0);
    const bool writes = lane == 0 || (lane == 16 && has_b);
    const typename Out::Pre pre = out.pre(mine, writes);
    float pa = 0.0f, pb = 0.0f;
    uint32_t mx = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) {
        const uint4 xe = lds128(xb + 16 * c);
        const uint4 xo = lds128(xb + 16 * p.chunks + 16 * c);
        const int kc = (int)lds_u32(xb + 32 * p.chunks + 4 * c);
        const int g = c >> p.gshift;
        const uint4 va = lds128(wa + 16 * c);
        const uint4 vb = lds128(wb + 16 * c);
        const uint32_t ba = SB::load(sa + g * SB::kBytes);
        const uint32_t bb = has_b ? SB::load(sb + g * SB::kBytes) : 1u;
        const int acc_a = w4a8_chunk_dot<ZX>(va, xe, xo, kc, p.zx);
        const int acc_b = w4a8_chunk_dot<ZX>(vb, xe, xo, kc, p.zx);
        mx = max(mx, max(ba - 1u, bb - 1u));
        pa = fmaf((float)acc_a, SB::f32(ba), pa);
        pb = fmaf((float)acc_b, SB::f32(bb), pb);
      }
    }
    const float t = warp_sum_pair(pa, pb, lane);
    if (writes) out.store(mine, t * Lx.sx, pre);
    return mx;
  }

  __device__ __forceinline__ static bool bad(uint32_t mx) { return mx >= SB::kBadFrom; }
};

// ---------------------------------------------------------------- INT8 op --
struct I8OpParams {
  float sa;
  int32_t chunks;  // 16-element chunks per row (cols / 16)
  int32_t zx, zw;
};

// Prepared activations, per 16-element chunk c: the 16 bytes at xb + 16c and
// the constant zw*sum(x) - 16*zx*zw at xb + 16*chunks + 4c.
template <int NCPL, bool OUT_F32, bool ZX>
struct I8Op {
  using Params = I8OpParams;
  static constexpr int kRawWords = 4;
  static constexpr int kChunkK = 16;
  __device__ __forceinline__ static void set_sx(const Params &, uint8_t *, float) {}
  __device__ __forceinline__ static float default_sx(const Params &p) { return p.sa; }
  struct Lane {
    int kl;  // sum of the chunk constants over this lane's chunks
  };

  static int xbuf_bytes(int chunks) { return ((chunks * 20 + 127) / 128) * 128; }

  __device__ __forceinline__ static void load_raw(const int8_t *x, int c, bool al16, uint32_t (&raw)[4]) {
    load_words<4>(x + 16 * c, al16, raw);
  }

  __device__ __forceinline__ static void store_prep(const Params &p, const uint32_t (&X)[4], int c, uint8_t *xb) {
    int sumx = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) sumx = dp4a_ss(X[q], 0x01010101u, sumx);
    reinterpret_cast<uint4 *>(xb)[c] = make_uint4(X[0], X[1], X[2], X[3]);
    reinterpret_cast<uint32_t *>(xb + 16 * p.chunks)[c] =
        (uint32_t)p.zw * (uint32_t)sumx - 16u * (uint32_t)p.zx * (uint32_t)p.zw;
  }

  __device__ __forceinline__ static void lane_init(const Params &p, Lane &L, const uint8_t *xb, int lane) {
    uint32_t kl = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) kl += lds_u32(xb + 16 * p.chunks + 4 * c);
    }
    L.kl = (int)kl;
  }

  __device__ __forceinline__ static uint32_t rows2(const Params &p, const Lane &L, const uint8_t *xb,
                                                   const uint8_t *wa, const uint8_t *, const uint8_t *wb,
                                                   const uint8_t *, const OutRef &, const GemvItem &it, int64_t ga,
                                                   bool has_b, int lane, const Lane &) {
    const float *ws = reinterpret_cast<const float *>(it.s);
    float wsa = 0.0f, wsb = 0.0f;
    if (OUT_F32) {  // issue the per-channel scale loads early
      if (lane == 0) wsa = __ldg(ws + ga);
      if (lane == 16 && has_b) wsb = __ldg(ws + ga + 1);
    }
    int acc_a = 0, acc_b = 0, sw_a = 0, sw_b = 0;
#pragma unroll
    for (int j = 0; j < NCPL; ++j) {
      const int c = lane + 32 * j;
      if (c < p.chunks) {
        const uint4 xr = lds128(xb + 16 * c);
        const uint4 va = lds128(wa + 16 * c);
        const uint4 vb = lds128(wb + 16 * c);
        acc_a = dp4a_ss(va.x, xr.x, acc_a);
        acc_b = dp4a_ss(vb.x, xr.x, acc_b);
        acc_a = dp4a_ss(va.y, xr.y, acc_a);
        acc_b = dp4a_ss(vb.y, xr.y, acc_b);
        acc_a = dp4a_ss(va.z, xr.z, acc_a);
        acc_b = dp4a_ss(vb.z, xr.z, acc_b);
        acc_a = dp4a_ss(va.w, xr.w, acc_a);
        acc_b = dp4a_ss(vb.w, xr.w, acc_b);
        if (ZX) {
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
    const uint32_t ta = (uint32_t)acc_a - (uint32_t)p.zx * (uint32_t)sw_a - (uint32_t)L.kl;
    const uint32_t tb = (uint32_t)acc_b - (uint32_t)p.zx * (uint32_t)sw_b - (uint32_t)L.kl;
    const uint32_t t = warp_sum_pair(ta, tb, lane);
    if (OUT_F32) {
      float *y = reinterpret_cast<float *>(it.y);
      if (lane == 0) y[ga] = __fmul_rn(__fmul_rn((float)(int)t, wsa), p.sa);
      if (lane == 16 && has_b) y[ga + 1] = __fmul_rn(__fmul_rn((float)(int)t, wsb), p.sa);
    } else {
      int32_t *y = reinterpret_cast<int32_t *>(it.y);
      if (lane == 0) y[ga] = (int32_t)t;
      if (lane == 16 && has_b) y[ga + 1] = (int32_t)t;
    }
    return 0;
  }

  __device__ __forceinline__ static bool bad(uint32_t) { return false; }
};

// ------------------------------------------------------ streaming skeleton --
template <int CW>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
}

// Reductions over the consumer threads, in a fixed order (bitwise
// reproducible).  `red` is CW floats of shared memory.
template <int CW>
__device__ __forceinline__ float consumers_sum(float v, float *red, int ctid) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((ctid & 31) == 0) red[ctid >> 5] = v;
  consumers_sync<CW>();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < CW; ++w) t += red[w];
  consumers_sync<CW>();
  return t;
}

template <int CW>
__device__ __forceinline__ float consumers_max(float v, float *red, int ctid) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((ctid & 31) == 0) red[ctid >> 5] = v;
  consumers_sync<CW>();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < CW; ++w) t = fmaxf(t, red[w]);
  consumers_sync<CW>();
  return t;
}

__device__ __forceinline__ uint32_t quant_rne_byte(float v, float s) {
  float q = rintf(__fdiv_rn(v, s));  // ties to even
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return (uint32_t)((int)q) & 0xFFu;
}

// sat_i8(rint(v / s)) without the division, given inv = RN(1/s) finite:
// q = RN(v * inv) and RN(v / s) both lie within |v/s| * 2^-23 of v/s (3.1e-5
// while |q| < 129), so rint() can differ between them only across a
// half-integer.  q is clamped to [-129, 128] (NaN -> -129, as fmaxf does in
// quant_rne_byte), rounded to an integer by adding 1.5 * 2^23 (ties to even);
// `near` is set when q lies within 2^-14 of a half-integer, and the caller
// then takes quant_rne_byte() instead.
__device__ __forceinline__ uint32_t quant_rne_byte_inv(float v, float inv, bool &near) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float q = fminf(fmaxf(__fmul_rn(v, inv), -129.0f), 128.0f);
  const float y = __fadd_rn(q, kMagic);
  near = __fsub_rn(0.5f, fabsf(__fsub_rn(q, __fsub_rn(y, kMagic)))) < 0x1p-14f;
  const int i = min(max(__float_as_int(y) - 0x4B400000, -128), 127);
  return (uint32_t)i & 0xFFu;
}

// Four consecutive f32 (16-byte load when the vector is 16-byte aligned).
// The chunk loops below are unrolled, so a chunk's loads are independent and
// cost about one memory latency together, not one each.
__device__ __forceinline__ float4 load4_f32(const float *p, bool al16) {
  if (al16) return *reinterpret_cast<const float4 *>(p);
  return make_float4(p[0], p[1], p[2], p[3]);
}

// Prepare matrix m's activations into buffer xb.  For f32 inputs every CTA
// computes the same normalisation / scale from the whole vector, so no extra
// kernel or global round trip is needed; the quantisation is
//   s = max|v| / 127 (1 if the vector is all zero),  q = sat_i8(rne(v / s))
// with v = x, or v = (x * rsqrt-scale) * norm_w for RMSNorm, where
// rsqrt-scale = 1 / sqrtf(sum(x^2) / K + eps).  Each consumer thread owns the
// chunks c = ctid, ctid + NT, ... in all passes (sum of squares, max, quantise)
// and sums its chunks in order before the fixed-order CTA reduction, so every
// CTA computes the same scale.  Contains consumer barriers: every consumer
// warp must call it.
template <class Op, int CW>
__device__ void prep_x_f32(const typename Op::Params &op, const LayerExt &e, uint8_t *xb, float *red, int ctid) {
  constexpr int NT = CW * 32;
  constexpr int KC = Op::kChunkK;
  const int chunks = op.chunks;
  const int K = chunks * KC;
  const bool rms = e.xmode == kXRmsNorm;
  const bool al16 =
      ((reinterpret_cast<uintptr_t>(e.xf) | (rms ? reinterpret_cast<uintptr_t>(e.norm_w) : 0)) & 15u) == 0;
  float scale = 1.0f;
  if (rms) {
    float ss = 0.0f;
    for (int c = ctid; c < chunks; c += NT) {
#pragma unroll
      for (int g = 0; g < KC / 4; ++g) {
        const float4 x = load4_f32(e.xf + (size_t)c * KC + 4 * g, al16);
        ss = __fadd_rn(ss, __fmul_rn(x.x, x.x));
        ss = __fadd_rn(ss, __fmul_rn(x.y, x.y));
        ss = __fadd_rn(ss, __fmul_rn(x.z, x.z));
        ss = __fadd_rn(ss, __fmul_rn(x.w, x.w));
      }
    }
    ss = consumers_sum<CW>(ss, red, ctid);
    scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), e.eps)));
  }
  // v[k .. k+3], k = c * KC + 4 * g
  auto vals4 = [&](int c, int g) -> float4 {
    const size_t k = (size_t)c * KC + 4 * g;
    float4 v = load4_f32(e.xf + k, al16);
    if (rms) {
      const float4 w = load4_f32(e.norm_w + k, al16);
      v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
      v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
      v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
      v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
    }
    return v;
  };
  float amax;
  if (e.xmode == kXF32Amax) {
    amax = __uint_as_float(__ldcg(e.amax_in));  // written by atomics in L2
  } else {
    float m = 0.0f;
    for (int c = ctid; c < chunks; c += NT) {
#pragma unroll
      for (int g = 0; g < KC / 4; ++g) {
        const float4 v = vals4(c, g);
        m = fmaxf(fmaxf(fmaxf(m, fabsf(v.x)), fmaxf(fabsf(v.y), fabsf(v.z))), fabsf(v.w));
      }
    }
    amax = consumers_max<CW>(m, red, ctid);
  }
  const float s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, s);
  const bool fast = isfinite(inv);
  for (int c = ctid; c < chunks; c += NT) {
    // all of the chunk's loads first (no branch between them), then the
    // branch-free quantisation, then at most one branch for near-ties
    float4 v[Op::kRawWords];
#pragma unroll
    for (int w = 0; w < Op::kRawWords; ++w) v[w] = vals4(c, w);
    uint32_t raw[Op::kRawWords];
    bool any_near = !fast;
#pragma unroll
    for (int w = 0; w < Op::kRawWords; ++w) {
      bool n0, n1, n2, n3;
      raw[w] = quant_rne_byte_inv(v[w].x, inv, n0) | (quant_rne_byte_inv(v[w].y, inv, n1) << 8) |
               (quant_rne_byte_inv(v[w].z, inv, n2) << 16) | (quant_rne_byte_inv(v[w].w, inv, n3) << 24);
      any_near = any_near || n0 || n1 || n2 || n3;
    }
    if (any_near) {  // rare: a value near a rounding tie (or no usable reciprocal): divide
#pragma unroll
      for (int w = 0; w < Op::kRawWords; ++w)
        raw[w] = quant_rne_byte(v[w].x, s) | (quant_rne_byte(v[w].y, s) << 8) | (quant_rne_byte(v[w].z, s) << 16) |
                 (quant_rne_byte(v[w].w, s) << 24);
    }
    Op::store_prep(op, raw, c, xb);
    if (e.xq_out && blockIdx.x == 0) {
#pragma unroll
      for (int w = 0; w < Op::kRawWords; ++w)
        reinterpret_cast<uint32_t *>(e.xq_out + (size_t)c * Op::kChunkK)[w] = raw[w];
    }
  }
  if (ctid == 0) {
    Op::set_sx(op, xb, s);
    if (e.xs_out && blockIdx.x == 0) *e.xs_out = s;
  }
}

}  // namespace ksb
