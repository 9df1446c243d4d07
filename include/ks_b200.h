/*
 * ks_b200.h -- B200 extensions to the libkernelsmith quantized C API.
 *
 * The reference library (pkp124/ulir-kernels) has no counterpart for any
 * declaration in this file; each one composes reference semantics that the
 * comment names.  The reference entry points themselves are declared,
 * unchanged, in kernelsmith/ks_quantized.h and kernelsmith/ks_common.h, which
 * this header includes.
 *
 * Two calling conventions:
 *   synchronous  (no suffix)   same as ks_quantized.h: device, managed or
 *                              host pointers; returns when the output is
 *                              written; bad scales reported as
 *                              KS_ERR_INVALID_ARG with the reference's
 *                              output contents (rows before the first row
 *                              with a bad scale written, that row and the
 *                              later ones left as they were).
 *   asynchronous (_async)      device (or managed) pointers only; the kernel
 *                              is queued on `stream` (a cudaStream_t, NULL for
 *                              the legacy default stream) and the call
 *                              returns at once.  Host-side argument checks
 *                              still return KS_ERR_INVALID_ARG.  Device-side
 *                              findings are written to `status` (device-
 *                              accessible memory holding
 *                              KS_B200_STATUS_WORDS uint32 words, cleared by
 *                              the caller; NULL to skip): word 0 becomes 1 if a
 *                              weight scale is <= 0, inf or nan, word 1 if a
 *                              device-side wait hit its one-second limit.
 *                              Nothing is allocated; the calls can be captured
 *                              in a CUDA graph.
 */

#ifndef KS_B200_H
#define KS_B200_H

#include <stddef.h>
#include <stdint.h>

#include "kernelsmith/ks_common.h"
#include "kernelsmith/ks_quantized.h"

#ifdef __cplusplus
extern "C" {
#endif

/* A CUDA error or a device-side timeout.  ks_b200_last_error() says which. */
#define KS_ERR_DEVICE (-4)

/* Scale element types for the *_async W4A8 entry points. */
#define KS_B200_SCALE_F32 0
#define KS_B200_SCALE_F16 1

#define KS_B200_STATUS_WORDS 2
#define KS_B200_STATUS_BAD_SCALE 0
#define KS_B200_STATUS_TIMEOUT 1

/* "major.minor.patch+sm_100a" of this build. */
const char *ks_b200_version(void);

/* Message of the last failing call made by this thread ("" if none). */
const char *ks_b200_last_error(void);

/* Number of CUDA devices visible to the process (0 without a GPU). */
int ks_b200_device_count(void);

/*
 * ks_matvec_w4a8 with IEEE binary16 group scales (the raw 16-bit patterns).
 * Each half widens exactly to f32, then the contract of ks_matvec_w4a8
 * applies unchanged, validation included.  Halves the scale traffic of the
 * f32 form.  Composes reference ks_quantized.c:94-159 with an exact
 * f16 -> f32 conversion.
 */
int ks_b200_matvec_w4a8_f16(const int8_t *input, const uint8_t *packed_weights,
                            size_t packed_stride_bytes,
                            const uint16_t *weight_scales_f16,
                            size_t scale_stride, float *output, size_t rows,
                            size_t cols, size_t group_size, float input_scale,
                            int32_t input_zero_point,
                            int32_t weight_zero_point);

/*
 * ks_b200_matvec_w4a8_f16 for callers that must not let a library allocate
 * memory.  This entry point has no counterpart in the reference library.
 *
 * The other synchronous entry points allocate their scratch (staging copies
 * of host buffers, status words) on first use.  Callers that reserve all
 * device memory up front, hand device memory out through their own
 * allocator, or run on threads where an allocation is not allowed use this
 * one instead: it calls no cudaMalloc, cudaFree or other allocating routine.
 * Its scratch is a fixed 540,928-byte array in device memory that every GPU
 * which loads the library holds until the process exits.
 *
 * Same arguments, checks and results as ks_b200_matvec_w4a8_f16 (it runs the
 * same kernels: outputs are bitwise equal; on a bad scale the rows from the
 * first bad one keep their contents), with these limits:
 *   - rows <= 131072 and cols <= 16384, else KS_ERR_UNSUPPORTED (valid
 *     arguments this entry point cannot serve; invalid ones still return
 *     KS_ERR_INVALID_ARG);
 *   - packed_weights and weight_scales_f16 must be device memory (they are
 *     not staged), else KS_ERR_UNSUPPORTED; input and output may be host
 *     memory (staged through the array) or device memory on the weights'
 *     GPU (used in place; another GPU is KS_ERR_INVALID_ARG);
 *   - the first call on a device looks up the scratch array's device address
 *     for that device, so make it before any stream capture; the address is
 *     cached, so no call may follow a cudaDeviceReset;
 *   - every call uses the same scratch array: calls whose work overlaps on
 *     the GPU (from several host threads) race and must be serialised.
 * The caller's current device is the same after the call as before it.
 */
int ks_b200_matvec_w4a8_f16_noalloc(const int8_t *input,
                                    const uint8_t *packed_weights,
                                    size_t packed_stride_bytes,
                                    const uint16_t *weight_scales_f16,
                                    size_t scale_stride, float *output,
                                    size_t rows, size_t cols,
                                    size_t group_size, float input_scale,
                                    int32_t input_zero_point,
                                    int32_t weight_zero_point);

/*
 * INT8 GEMV with a per-output-channel dequant epilogue:
 *   output[r] = (f32(acc[r]) * weight_scales[r]) * input_scale
 * where acc[r] is exactly ks_matvec_i8's int32 result; each product is one
 * IEEE round-to-nearest multiply in the order written (no fused multiply-add),
 * so results are bit-exact against the same expression on the CPU.
 * Argument checks are ks_matvec_i8's plus weight_scales != NULL.
 */
int ks_b200_matvec_i8_dequant(const int8_t *input, const int8_t *weights,
                              size_t weight_stride, const float *weight_scales,
                              float input_scale, float *output, size_t rows,
                              size_t cols, int32_t input_zero_point,
                              int32_t weight_zero_point);

/* Asynchronous forms (device pointers, caller's stream, no allocation). */
int ks_b200_matvec_w4a8_async(const int8_t *input,
                              const uint8_t *packed_weights,
                              size_t packed_stride_bytes,
                              const void *weight_scales, int scale_type,
                              size_t scale_stride, float *output, size_t rows,
                              size_t cols, size_t group_size,
                              float input_scale, int32_t input_zero_point,
                              int32_t weight_zero_point, uint32_t *status,
                              void *stream);

int ks_b200_matvec_i8_async(const int8_t *input, const int8_t *weights,
                            size_t weight_stride, int32_t *output, size_t rows,
                            size_t cols, int32_t input_zero_point,
                            int32_t weight_zero_point, void *stream);

int ks_b200_matvec_i8_dequant_async(const int8_t *input, const int8_t *weights,
                                    size_t weight_stride,
                                    const float *weight_scales,
                                    float input_scale, float *output,
                                    size_t rows, size_t cols,
                                    int32_t input_zero_point,
                                    int32_t weight_zero_point, void *stream);

/*
 * A batch of independent GEMVs of one shape in one launch: matrix i computes
 * outputs[i] from inputs[i], packed_weights[i] and weight_scales[i] exactly
 * as ks_b200_matvec_w4a8_async would (bitwise the same results), but every SM
 * streams its rows of all the matrices back to back through one deep shared-
 * memory ring, so there is no gap between matrices.  For projections that
 * share a shape and run together (Q/K/V or gate/up of a decode step, the
 * experts of a mixture-of-experts layer, the layers of a batch of
 * independent requests).  The pointer arrays are host memory with `count`
 * entries; the buffers they point to are device memory.  Argument checks are
 * ks_matvec_w4a8's, per matrix.  Batches beyond 64 matrices are split into
 * launches of at most 64.
 */
int ks_b200_matvec_w4a8_batch_async(int count, const int8_t *const *inputs,
                                    const uint8_t *const *packed_weights,
                                    const void *const *weight_scales,
                                    float *const *outputs,
                                    size_t packed_stride_bytes, int scale_type,
                                    size_t scale_stride, size_t rows,
                                    size_t cols, size_t group_size,
                                    float input_scale,
                                    int32_t input_zero_point,
                                    int32_t weight_zero_point,
                                    uint32_t *status, void *stream);

/* INT8 batch: int32 outputs (ks_matvec_i8) when weight_scales is NULL,
 * else f32 outputs with the per-channel dequant epilogue of
 * ks_b200_matvec_i8_dequant (outputs are float* then). */
int ks_b200_matvec_i8_batch_async(int count, const int8_t *const *inputs,
                                  const int8_t *const *weights,
                                  const float *const *weight_scales,
                                  void *const *outputs, size_t weight_stride,
                                  size_t rows, size_t cols,
                                  int32_t input_zero_point,
                                  int32_t weight_zero_point, float input_scale,
                                  void *stream);

/*
 * Multi-GPU row sharding (one process per GPU).  A weight matrix is split
 * into contiguous row blocks, one per rank; each rank computes its rows and
 * stores every output element straight into the gathered output buffer of
 * every rank (peer memory over NVLink: plain stores, no multicast).  No
 * collective library runs on the data path.
 *
 * ks_b200_ipc_get_handle / ks_b200_ipc_open_handle exchange device buffers
 * between processes (CUDA IPC; `handle` is KS_B200_IPC_HANDLE_BYTES bytes,
 * `offset` locates the buffer inside its allocation).
 */
#define KS_B200_IPC_HANDLE_BYTES 64
int ks_b200_ipc_get_handle(const void *dev_ptr, unsigned char *handle,
                           size_t *offset);
int ks_b200_ipc_open_handle(const unsigned char *handle, size_t offset,
                            void **peer_ptr);
int ks_b200_ipc_close_handle(void *peer_ptr, size_t offset);

/*
 * Sharded batch: this rank's row block of `count` W4A8 matrices (rows x cols
 * each, the shape of ks_b200_matvec_w4a8_batch_async).  The output of row r
 * of matrix m is stored at rank_outputs[p][m * matrix_stride + row_offset + r]
 * for every rank p (rank_outputs[p] is that rank's gathered buffer, opened
 * with ks_b200_ipc_open_handle; this rank's own buffer included).  Each CTA
 * collects its rows of a matrix in shared memory and writes them to every
 * rank as one contiguous run of coalesced stores once the matrix is done.
 * After its last store each CTA adds 1 to rank_counters[p] for every rank p,
 * behind a system-scope fence; give each rank an array of nranks counter
 * words and pass, as rank_counters[p], the word of rank p's array that
 * counts this rank's arrivals (see ks_b200_peer_arrival_wait_ranks_async).
 * *signals_per_rank receives how many arrivals this call sends to each rank.
 * Needs the streaming kernel's shape rules (else KS_ERR_UNSUPPORTED).
 */
int ks_b200_matvec_w4a8_batch_gather_async(
    int count, const int8_t *const *inputs,
    const uint8_t *const *packed_weights, const void *const *weight_scales,
    int nranks, float *const *rank_outputs, uint32_t *const *rank_counters,
    size_t matrix_stride, size_t row_offset, size_t packed_stride_bytes,
    int scale_type, size_t scale_stride, size_t rows, size_t cols,
    size_t group_size, float input_scale, int32_t input_zero_point,
    int32_t weight_zero_point, uint32_t *signals_per_rank, uint32_t *status,
    void *stream);

/*
 * Queue a wait, on `stream`, until this rank's arrival counter has received
 * `arrivals` more signals than at the previous wait (the running target is
 * kept in expected[0], device memory initialised to 0 with the counter).
 * With arrivals = nranks * signals_per_rank of the preceding sharded calls,
 * the gathered outputs of all ranks are complete and visible once the wait
 * returns.  The wait gives up after one second and sets status word 1.
 */
int ks_b200_peer_arrival_wait_async(const uint32_t *counter,
                                    uint32_t *expected, uint32_t arrivals,
                                    uint32_t *status, void *stream);

/*
 * The same wait over one counter word per source rank: counters[s] (device
 * memory on this rank, zero-initialised with expected[0]) counts the
 * arrivals from rank s.  The wait ends once every counters[s] has received
 * arrivals_per_rank more signals than at the previous wait, so arrivals a
 * fast rank sends for its next run cannot stand in for those of a slow rank.
 * It gives up after timeout_ns nanoseconds (0: one second; at most 10 s),
 * sets status word 1 and returns; expected[0] advances either way.
 */
int ks_b200_peer_arrival_wait_ranks_async(const uint32_t *counters, int nranks,
                                          uint32_t *expected,
                                          uint32_t arrivals_per_rank,
                                          uint64_t timeout_ns, uint32_t *status,
                                          void *stream);

/*
 * Synchronise `stream` and turn the status words an asynchronous call wrote
 * (device, managed or mapped memory) into the synchronous calls' codes:
 * KS_ERR_DEVICE if a device-side wait timed out, KS_ERR_INVALID_ARG if a
 * weight scale was <= 0, inf or nan, else KS_OK.  Allocates nothing.
 */
int ks_b200_status_check(const uint32_t *status, void *stream);

/*
 * One quantised Llama-style decode layer at batch 1 (no counterpart in the
 * reference; it composes the reference's f32 RMSNorm, SiLU and multiply --
 * ks_normalization.c:13-36, ks_activations.c:39-49, ks_elementwise.c:22-30 --
 * with per-token int8 activation quantisation and four W4A8 GEMVs):
 *   x1 = RMSNorm(h_in, norm1_w, eps)        q1, s1 = quantise(x1)
 *   qkv = W_qkv [3h x h] . q1 * s1
 *   v = qkv[2h : 3h]  (attention over one position returns V)
 *                                           q2, s2 = quantise(v)
 *   h2 = h_in + W_o [h x h] . q2 * s2
 *   x3 = RMSNorm(h2, norm2_w, eps)          q3, s3 = quantise(x3)
 *   gate = W_gate [i x h] . q3 * s3,  up = W_up [i x h] . q3 * s3
 *   act = silu(gate) * up                   q4, s4 = quantise(act)
 *   h_out = h2 + W_down [h x i] . q4 * s4
 * quantise(v): s = max|v| / 127 (1 if v is all zero), q = sat_i8(rne(v / s)).
 * weights[5] / scales_f16[5] are qkv, o, gate, up, down: packed int4 (row
 * stride cols/2 bytes) with f16 group scales (row stride cols/group_size).
 * The whole layer is one cooperative persistent kernel (one CTA per SM: a
 * producer warp streams all five weight matrices back to back, the consumer
 * warps run the four stages with a grid barrier between them) when the shape
 * allows it (hidden <= 8192, inter <= 16384, 16-byte aligned vectors, weights
 * and scales, scale rows a multiple of 16 bytes); otherwise four GEMV
 * launches with the same fused preparation and epilogues, chained with
 * programmatic dependent launch.  KS_B200_DECODE_PERSISTENT=0 forces the
 * four launches.  `workspace` (device memory, ks_b200_decode_layer_workspace
 * bytes, zero-filled before its first use, not shared by calls that may run
 * at the same time) receives the intermediates, in this order, each region
 * starting on a 256-byte boundary (ks_b200_decode_layer_offsets gives the 11
 * offsets and the total): f32 qkv[3h], h2[h], gate[i], up[i], act[i],
 * s1..s4[4], u32 max|act| bits (bytes 128..135 of that 256-byte region hold
 * the persistent kernel's grid-barrier counter), int8 q1[h], q2[h], q3[h],
 * q4[i].  After a call whose status reports a timeout, zero the workspace
 * again before reusing it.
 */
size_t ks_b200_decode_layer_workspace(size_t hidden, size_t inter);
/* Kernel launches one ks_b200_decode_layer_w4a8_async call of this shape
 * makes on the current device (16-byte aligned operands): 1 for the
 * persistent kernel, 4 for the chained fallback, 0 for an invalid shape. */
int ks_b200_decode_layer_launches(size_t hidden, size_t inter, size_t group_size);
int ks_b200_decode_layer_offsets(size_t hidden, size_t inter, size_t *offsets);
int ks_b200_decode_layer_w4a8_async(const float *h_in, float *h_out,
                                    const float *norm1_w, const float *norm2_w,
                                    float eps, const uint8_t *const *weights,
                                    const uint16_t *const *scales_f16,
                                    size_t hidden, size_t inter,
                                    size_t group_size, void *workspace,
                                    size_t workspace_bytes, uint32_t *status,
                                    void *stream);

/*
 * A chain of n_layers such layers (no counterpart in the reference): layer l
 * takes the previous layer's output (h_in for layer 0) and the last layer
 * writes h_out.  Per layer l: norm1_w[l], norm2_w[l], and the five matrices
 * weights[5 * l + k] / scales_f16[5 * l + k] in the order qkv, o, gate, up,
 * down (host arrays of device pointers).  Every layer's results are bitwise
 * those of ks_b200_decode_layer_w4a8_async on the same input.  Up to 32
 * layers run in one cooperative persistent launch: the producer warp
 * streams the next layer's weights while the current layer finishes, so the
 * launch and the drain of the weight ring are paid once per 32 layers, not
 * per layer.  workspace: ks_b200_decode_layers_workspace bytes (the
 * single-layer regions at the offsets ks_b200_decode_layer_offsets gives,
 * then two f32[hidden] vectors for the outputs of the inner layers; after
 * the call they hold those of the last two layers before the final one),
 * zero-filled before its first use; it may not be shared by calls that
 * can run at the same time.  The intermediates left in it are the last
 * layer's.  Shape rules, fallback and status as for the single layer.
 */
size_t ks_b200_decode_layers_workspace(size_t hidden, size_t inter);
int ks_b200_decode_layers_w4a8_async(size_t n_layers, const float *h_in,
                                     float *h_out, const float *const *norm1_w,
                                     const float *const *norm2_w, float eps,
                                     const uint8_t *const *weights,
                                     const uint16_t *const *scales_f16,
                                     size_t hidden, size_t inter,
                                     size_t group_size, void *workspace,
                                     size_t workspace_bytes, uint32_t *status,
                                     void *stream);

/*
 * Skinny INT8 GEMM with requantisation (batched decode, M = 1..256 tokens):
 *   acc[m, n] = sum_k a[m, k] * w[n, k]                       (int32, exact)
 *   out[m, n] = sat_i8(rne(((f32(acc) * a_scales[m]) * w_scales[n]) / out_scale))
 * a is [m, k] with row stride lda bytes, w is [n, k] with row stride ldw
 * bytes (the INT8 GEMV weight layout), out is [m, n] with row stride ldo
 * bytes; only the m x n output bytes are written.  Each step of the
 * epilogue is one IEEE round-to-nearest operation in the order written, the
 * rounding to integer is ties-to-even and the result saturates to
 * [-128, 127], so outputs are bit-exact against the same expression on the
 * CPU.  Zero points are 0; scales must be finite.  The reference has no
 * requantising entry point (its quantisation spec leaves requantisation out
 * of the first ABI); this composes reference ks_dot_i8 (ks_quantized.c:44-65)
 * per output with the spec's round-to-nearest-even quantise rule.
 * Runs on tcgen05 tensor cores (kind::i8, TMEM accumulators) when lda and
 * ldw are multiples of 16 and a, w are 16-byte aligned and m <= 256;
 * otherwise on a generic kernel.
 */
int ks_b200_gemm_i8_requant(const int8_t *a, size_t lda, const float *a_scales,
                            const int8_t *w, size_t ldw,
                            const float *w_scales, float out_scale,
                            int8_t *out, size_t ldo, size_t m, size_t n,
                            size_t k);

/* Asynchronous form; acc_out (optional, [m, n] int32, row stride n) receives
 * the raw accumulators. */
int ks_b200_gemm_i8_requant_async(const int8_t *a, size_t lda,
                                  const float *a_scales, const int8_t *w,
                                  size_t ldw, const float *w_scales,
                                  float out_scale, int8_t *out, size_t ldo,
                                  size_t m, size_t n, size_t k,
                                  int32_t *acc_out, uint32_t *status,
                                  void *stream);

/*
 * Batched form of ks_b200_gemm_i8_requant_async (no counterpart in the
 * reference): `count` independent GEMMs of one shape, out_i = requant(a_i x
 * w_i^T) with a_scales[i], w_scales[i] and the shared out_scale, each output
 * bit-identical to the single call.  The pointer arrays are host memory
 * holding device pointers.  With m <= 64 and every operand on the tensor-core
 * path, up to 16 GEMMs run in one persistent launch: each SM streams its rows
 * of every weight matrix back to back, and a GEMM's requantising epilogue
 * overlaps the next GEMM's main loop; otherwise one launch per GEMM.  No
 * allocation, capturable in a CUDA graph.
 */
int ks_b200_gemm_i8_requant_batch_async(int count, const int8_t *const *a,
                                        size_t lda,
                                        const float *const *a_scales,
                                        const int8_t *const *w, size_t ldw,
                                        const float *const *w_scales,
                                        float out_scale, int8_t *const *out,
                                        size_t ldo, size_t m, size_t n,
                                        size_t k, uint32_t *status,
                                        void *stream);

/*
 * Which kernel family a W4A8 / INT8 call with these arguments runs on the
 * current device: 1 = TMA-staged streaming kernel, 0 = generic per-element
 * kernel (any stride, alignment, odd cols, any group size), negative = the
 * arguments would be rejected.  For tests and benchmarks.
 */
int ks_b200_w4a8_kernel_path(const void *input, const void *packed_weights,
                             size_t packed_stride_bytes,
                             const void *weight_scales, int scale_type,
                             size_t scale_stride, size_t rows, size_t cols,
                             size_t group_size);
int ks_b200_i8_kernel_path(const void *input, const void *weights,
                           size_t weight_stride, size_t rows, size_t cols);
/* 1 = tcgen05 tensor-core kernel, 0 = generic kernel, negative = rejected. */
int ks_b200_gemm_i8_kernel_path(const void *a, size_t lda, const void *w,
                                size_t ldw, size_t m, size_t n, size_t k);

/*
 * Batched W4A8 GEMM for decode (M = 1..64 tokens; no counterpart in the
 * reference): for every token m and weight row n
 *   out[m, n] = a_scales[m] * sum_g f32(acc_g) * scale[n, g],
 *   acc_g = sum_{k in group g} a[m, k] * w[n, k]      (int32, exact)
 * a: int8 [m, k] (row stride lda), a_scales: f32 [m]; w: the native packed
 * int4 rows (ks_matvec_w4a8's layout) with f32 or f16 group scales
 * (scale_type, row stride scale_stride); zero points 0; out: f32 [m, n]
 * (row stride ldo).  Each token's row equals ks_matvec_w4a8 for that token up
 * to the order of the f32 sum.  Runs on the tensor cores (tcgen05.mma
 * kind::i8 on int4 weights unpacked to int8 in shared memory); needs
 * m <= 64, k a multiple of 32 and of group_size in {32, 64, 128}, 16-byte
 * aligned a / weights / scales with lda, packed_stride_bytes and scale-row
 * bytes multiples of 16, else KS_ERR_UNSUPPORTED.  Device pointers, queued on
 * `stream`; `status` as for the other asynchronous calls.
 */
int ks_b200_gemm_w4a8_async(const int8_t *a, size_t lda, const float *a_scales,
                            const uint8_t *packed_weights, size_t packed_stride_bytes,
                            const void *weight_scales, int scale_type, size_t scale_stride,
                            float *out, size_t ldo, size_t m, size_t n, size_t k,
                            size_t group_size, uint32_t *status, void *stream);

/*
 * W4A8 GEMV on f32 activations (no counterpart in the reference): the input
 * is quantised per token on the device, s = max|input| / 127 (1 if all zero),
 * q = sat_i8(round_half_even(input / s)), then
 *   output[r] = s * sum_g f32(acc_g) * scale[r, g]
 * exactly as ks_matvec_w4a8 / ks_b200_matvec_w4a8_async with that q and
 * input_scale = s (zero points 0).  quantized_input (int8 [cols]) and
 * input_scale (one float) receive q and s when not NULL.  Streaming kernel
 * only: cols a multiple of 32, group_size a power-of-two multiple of 32,
 * scale-row bytes a multiple of 16, 16-byte aligned input / weights / scales
 * with strides multiples of 16, else KS_ERR_UNSUPPORTED.  Device pointers,
 * queued on `stream`; `status` as for the other asynchronous calls.
 */
int ks_b200_matvec_w4a8_f32in_async(const float *input, const uint8_t *packed_weights,
                                    size_t packed_stride_bytes, const void *weight_scales,
                                    int scale_type, size_t scale_stride, float *output,
                                    size_t rows, size_t cols, size_t group_size,
                                    int8_t *quantized_input, float *input_scale,
                                    uint32_t *status, void *stream);

/*
 * Per-token activation quantisation (the rule above) of n_tokens rows of f32
 * x (row stride ldx elements) into int8 q (row stride ldq) and f32 scales
 * [n_tokens]: the a / a_scales operands of ks_b200_gemm_w4a8_async.  Device
 * pointers, queued on `stream`.
 */
int ks_b200_quantize_per_token_async(const float *x, size_t ldx, size_t n_tokens,
                                     size_t cols, int8_t *q, size_t ldq, float *scales,
                                     void *stream);

/*
 * Native quantized layout version (no counterpart in the reference's headers;
 * the reference's design proposes it for its target profiles,
 * docs/design/DES-015-quantized-layout-abi-and-integration-conversion-paths.md:195-198).
 * Version 1: W4A8 signed int4, value k in byte k/2 (low nibble for even k),
 * rows independent, group scales row-major with element k using group
 * k / group_size; INT8 row-major.  Every kernel and the importer below read or
 * write this layout; ks_b200_quant_layout_version() returns the value the
 * library was built with.
 */
#define KS_QUANT_LAYOUT_VERSION 1
int ks_b200_quant_layout_version(void);

/*
 * Resident W4A8 weights (no counterpart in the reference, whose calls read
 * the weights from the caller's memory every time): upload rows
 * [row_begin, row_begin + row_count) of a packed matrix -- all of it, or one
 * rank's row shard -- to the current device once and run GEMVs on them.
 * The rows are copied byte for byte in the ABI layout; only the row strides
 * grow to multiples of 16 bytes (zero padding, never read).  The source may
 * be host or device memory.  layout_version must be KS_QUANT_LAYOUT_VERSION
 * (the layout the caller's converter wrote; DES-015:195-198 proposes the
 * macro), else KS_ERR_UNSUPPORTED; other argument checks as for
 * ks_matvec_w4a8, plus row_begin + row_count <= rows, else
 * KS_ERR_INVALID_ARG.  Allocates device memory, freed by
 * ks_b200_w4a8_release.
 */
typedef struct ks_b200_w4a8_weights ks_b200_w4a8_weights;
int ks_b200_w4a8_register(const uint8_t *packed_weights,
                          size_t packed_stride_bytes, const void *weight_scales,
                          int scale_type, size_t scale_stride, size_t rows,
                          size_t cols, size_t group_size, size_t row_begin,
                          size_t row_count, int layout_version,
                          ks_b200_w4a8_weights **out);
/* The device copy: pointers, strides (bytes / elements), rows held and the
 * first source row (any output pointer may be NULL). */
int ks_b200_w4a8_weights_info(const ks_b200_w4a8_weights *weights,
                              const uint8_t **packed_weights,
                              size_t *packed_stride_bytes,
                              const void **weight_scales, size_t *scale_stride,
                              size_t *rows, size_t *row_begin);
/* ks_b200_matvec_w4a8_async over the registered rows (output[r] for row
 * row_begin + r), with the registration's device current. */
int ks_b200_w4a8_matvec_registered_async(const ks_b200_w4a8_weights *weights,
                                         const int8_t *input, float input_scale,
                                         int32_t input_zero_point,
                                         int32_t weight_zero_point,
                                         float *output, uint32_t *status,
                                         void *stream);
int ks_b200_w4a8_release(ks_b200_w4a8_weights *weights);

/*
 * GGML Q4_0 weights -> native W4A8, on the GPU (the reference's offline
 * conversion, DES-015:148-179; no counterpart function in the reference).
 * blocks: rows x (cols/32) Q4_0 blocks of 18 bytes (f16 d, then 16 bytes:
 * element j in the low nibble of byte j, element j + 16 in its high nibble,
 * value (nibble - 8) * d), 2-byte aligned, row stride block_row_stride bytes
 * (even).  Each native
 * group of group_size (32..256) is requantised with a positive scale:
 *   scale = max(max(v) / 7, -min(v) / 8), 1 if that is 0;
 *   q = clamp(round_half_even(v / scale), -8, 7)
 * (with KS_B200_SCALE_F16 the scale is rounded to f16 first and the codes are
 * made with that value).  Output: packed int4 rows (16-byte aligned, stride a
 * multiple of 16) and scales, ready for ks_matvec_w4a8 / ks_b200_*_w4a8*.
 * Device pointers, queued on `stream`; not byte-exact to GGML (the reference's
 * design says so), bit-exact to the same f32 steps on a CPU.
 */
int ks_b200_import_ggml_q4_0_async(const void *blocks, size_t block_row_stride,
                                   size_t rows, size_t cols, size_t group_size,
                                   uint8_t *packed_weights, size_t packed_stride_bytes,
                                   void *weight_scales, int scale_type,
                                   size_t scale_stride, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KS_B200_H */
