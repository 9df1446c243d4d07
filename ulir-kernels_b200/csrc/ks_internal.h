// ks_internal.h -- host-side declarations shared by the libkernelsmith (B200)
// translation units: kernel launchers, device properties, error text.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

namespace ksb {

enum ScaleType : int { kScaleF32 = 0, kScaleF16 = 1 };

// Status words written by kernels (plain stores of 1, never atomics, so the
// words may live in mapped host memory).  status[0]: a weight scale was <= 0,
// inf or nan.  status[1]: a device-side wait hit its time limit.
constexpr int kStatusBadScale = 0;
constexpr int kStatusTimeout = 1;
constexpr int kStatusWords = 2;

struct W4A8Launch {
  const int8_t *x;
  const uint8_t *w;
  int64_t wstride;  // bytes between packed rows
  const void *s;    // f32 or f16 group scales
  int64_t sstride;  // scale elements between rows
  int stype;        // ScaleType
  float *y;
  int64_t rows, cols, group;
  float sx;
  int32_t zx, zw;
  uint32_t *status;  // kStatusWords words, may be null
};

struct I8Launch {
  const int8_t *x;
  const int8_t *w;
  int64_t wstride;  // bytes between rows
  void *y;          // int32_t[rows] or float[rows]
  int64_t rows, cols;
  int32_t zx, zw;
  const float *ws;  // per-row dequant scale (f32 output only)
  float sa;         // activation scale (f32 output only)
  int out_f32;
  uint32_t *status;
};

struct GemmI8Launch {
  const int8_t *a;   // [m, k], row stride lda
  int64_t lda;
  const float *sa;   // [m]
  const int8_t *w;   // [n, k], row stride ldw
  int64_t ldw;
  const float *ws;   // [n]
  float out_scale;
  int8_t *out;       // [m, n], row stride ldo
  int64_t ldo;
  int64_t m, n, k;
  int32_t *acc_out;  // optional [m, n] int32 accumulators (tests), may be null
  uint32_t *status;
};

struct DeviceProps {
  int sm_count = 0;
  int smem_optin = 0;  // max dynamic shared memory per block
  int cc_major = 0, cc_minor = 0;
};
const DeviceProps &device_props(int device);

// Integer environment knob (tuning only; the default when unset or empty).
int env_int(const char *name, int dflt);
// Programmatic dependent launch on this stream: on unless KS_B200_PDL=0, never
// on the legacy or per-thread default stream.
bool pdl_enabled(cudaStream_t stream);

cudaError_t launch_w4a8(const W4A8Launch &a, cudaStream_t stream, int device);
cudaError_t launch_i8(const I8Launch &a, cudaStream_t stream, int device);

// A batch of independent GEMVs of one shape: per-matrix activation, weight,
// scale (W4A8 group scales or INT8 per-channel dequant scales) and output
// pointers, host arrays of `count` entries.  Launched as one streaming pass
// per SM; the shape fields of the W4A8Launch / I8Launch are used, their
// pointer fields are not.
struct GemvBatch {
  int count;
  const int8_t *const *x;
  const void *const *w;
  const void *const *s;
  void *const *y;
};
cudaError_t launch_w4a8_batch(const W4A8Launch &shape, const GemvBatch &b, cudaStream_t stream, int device);
// f32 activations quantised per token in the kernel; a.x is unused.
cudaError_t launch_w4a8_f32in(const W4A8Launch &a, const float *xf, int8_t *xq_out, float *xs_out,
                              cudaStream_t stream, int device);
// Per-token int8 quantisation of n rows of f32 (s = max|x| / 127, 1 if 0;
// q = sat_i8(rne(x / s))).
cudaError_t launch_quantize_tokens(const float *x, int64_t ldx, int64_t n, int64_t cols, int8_t *q, int64_t ldq,
                                   float *scales, cudaStream_t stream);
cudaError_t launch_i8_batch(const I8Launch &shape, const GemvBatch &b, cudaStream_t stream, int device);

// Sharded W4A8 batch whose outputs are gathered by peer stores (see the
// kernel's GemvItems): the output of row r of matrix m is stored at
// peer_y[p][m * mstride + row_offset + r] for every rank p, and every CTA of
// every launch adds 1 to every rank's arrival counter.  signals_per_rank
// receives how many arrivals this call sends to each rank.
struct PeerGather {
  int npeers;
  float *const *peer_y;
  uint32_t *const *peer_cnt;
  int64_t mstride;
  int64_t row_offset;
};
cudaError_t launch_w4a8_batch_gather(const W4A8Launch &shape, const GemvBatch &b, const PeerGather &pg,
                                     cudaStream_t stream, int device, uint32_t *signals_per_rank);
// One quantised decode layer (see launch_decode_layer_w4a8 in ks_gemv.cu).
// w/s: qkv [3h x h], o [h x h], gate [i x h], up [i x h], down [h x i], W4A8
// with f16 group scales, dense strides.  The other pointers are the caller's
// workspace regions (ks_b200_decode_layer_workspace).
struct DecodeLayerArgs {
  const float *h_in;
  float *h_out;
  const float *norm1_w, *norm2_w;
  float eps;
  const uint8_t *w[5];
  const void *s[5];
  int64_t hidden, inter, group;
  float *qkv, *h2, *gate, *up, *act, *scales;
  uint32_t *amax;
  int8_t *q[4];
  uint32_t *status;
};
cudaError_t launch_decode_layer_w4a8(const DecodeLayerArgs &a, cudaStream_t stream, int device);
// The same layer as four chained GEMV launches (the fallback of the
// persistent kernel).
cudaError_t launch_decode_layer_four(const DecodeLayerArgs &a, cudaStream_t stream, int device);

// A chain of decode layers: layer g reads the previous layer's output and
// writes its own, h_in -> hbuf[0] -> hbuf[1] -> hbuf[0] ... -> h_out (layer g
// writes hbuf[g & 1] unless it is the last).  Per layer: the five weight
// matrices (qkv, o, gate, up, down) with f16 scales, and the two RMSNorm
// weight vectors.  The workspace regions are those of DecodeLayerArgs,
// reused by every layer.
struct DecodeLayerWeights {
  const uint8_t *w[5];
  const void *s[5];
  const float *norm1_w, *norm2_w;
};
struct DecodeLayersArgs {
  int layers;
  const DecodeLayerWeights *lw;  // host array of `layers` entries
  const float *h_in;
  float *h_out;
  float *hbuf[2];
  float eps;
  int64_t hidden, inter, group;
  float *qkv, *h2, *gate, *up, *act, *scales;
  uint32_t *amax;
  int8_t *q[4];
  uint32_t *status;
};
cudaError_t launch_decode_layers_w4a8(const DecodeLayersArgs &a, cudaStream_t stream, int device);
// The chain as cooperative persistent launches of up to 32 layers each;
// cudaErrorNotSupported when the shape, the alignment or the device does not
// allow it (the caller then uses four launches per layer).
// dry: every check (shape, alignment, occupancy), no launch
cudaError_t launch_decode_layers_persistent(const DecodeLayersArgs &a, cudaStream_t stream, int device,
                                            bool dry = false);

// Wait (bounded by limit_ns) until each of counters[0 .. ncounters) reaches
// expected[0] + arrivals; expected[0] then holds the new target.
cudaError_t launch_peer_wait(const uint32_t *counters, int ncounters, uint32_t *expected, uint32_t arrivals,
                             uint64_t limit_ns, uint32_t *status, cudaStream_t stream);
// First row r (of `rows`) whose scale row holds a scale <= 0, inf or nan,
// into *first_bad (atomicMin; the caller sets it to ~0 first).
cudaError_t launch_w4a8_first_bad_row(const void *s, int stype, int64_t sstride, int64_t rows, int64_t groups,
                                      unsigned long long *first_bad, cudaStream_t stream);
cudaError_t launch_gemm_i8(const GemmI8Launch &a, cudaStream_t stream, int device);

// Independent GEMMs of one shape (m, n, k, strides and out_scale from the
// GemmI8Launch; its pointers are unused): host arrays of device pointers.
struct GemmI8Batch {
  int count;
  const int8_t *const *a;
  const float *const *sa;
  const int8_t *const *w;
  const float *const *ws;
  int8_t *const *out;
};
cudaError_t launch_gemm_i8_batch(const GemmI8Launch &shape, const GemmI8Batch &b, cudaStream_t stream,
                                 int device);

// Batched W4A8 GEMM (tokens x native int4 weights, group scales) on tcgen05.
struct GemmW4A8Launch {
  const int8_t *a;      // [m, k] int8, row stride lda
  int64_t lda;
  const float *sx;      // [m] per-token activation scales
  const uint8_t *w;     // [n, k/2] packed int4, row stride wstride bytes
  int64_t wstride;
  const void *s;        // [n, k/group] f32 or f16, row stride sstride elements
  int64_t sstride;
  int stype;            // ScaleType
  float *y;             // [m, n], row stride ldy
  int64_t ldy;
  int64_t m, n, k, group;
  uint32_t *status;
};
bool gemm_w4a8_supported(const GemmW4A8Launch &a);
cudaError_t launch_gemm_w4a8(const GemmW4A8Launch &a, cudaStream_t stream, int device);

// GGML Q4_0 blocks -> native W4A8 (packed int4 + positive group scales).
struct ImportQ4Launch {
  const uint8_t *src;     // rows x (cols / 32) blocks of 18 bytes
  int64_t src_stride;     // bytes between rows of blocks
  int64_t rows, cols, group;
  uint8_t *packed;        // [rows][packed_stride], 16-byte aligned rows
  int64_t packed_stride;
  void *scales;           // f32 or f16 [rows][scale_stride]
  int scale_type;         // ScaleType
  int64_t scale_stride;   // elements
};
cudaError_t launch_import_q4_0(const ImportQ4Launch &a, cudaStream_t stream);

// Which kernel family launch_w4a8 / launch_i8 picked for a shape (tests and
// benchmarks report it): 0 = generic per-element path, 1 = TMA-staged path.
int w4a8_path(const W4A8Launch &a);
int i8_path(const I8Launch &a);
int gemm_i8_path(const GemmI8Launch &a);

void set_last_error(const std::string &msg);

}  // namespace ksb
