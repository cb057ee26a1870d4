/* xq_kernels.h: kernel-level C ABI of libxqwen35.so.
 *
 * The reference exposes its kernels as C++ functions over xq::kernels::QuantizedMatrix
 * (customlib/kernels/kernels.hpp:11-53). A host binding them through an FFI needs plain C,
 * so each entry point below takes plain pointers and sizes. Pointers named *_dev are CUDA
 * device pointers; `stream` is a cudaStream_t passed as void* (NULL = the legacy default
 * stream). Entry points return 0 on success and a negative xq_status value on error;
 * xqk_last_error() returns the message of the last failure on the calling thread.
 */
#ifndef XQ_KERNELS_H_
#define XQ_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XQK_API __attribute__((visibility("default")))

/* A W4A16 matrix resident in device memory in the B200 row layout: each row is its
 * nibbles (reference order) followed by that row's group metadata, 16-byte aligned, so one
 * contiguous bulk copy moves a block of rows with their scales. */
typedef struct xqk_matrix xqk_matrix;

XQK_API const char* xqk_last_error(void);

/* Upload a matrix given in the reference's QuantizedMatrix fields (kernels.hpp:11-21,
 * XQ4 payload order custom_model.cpp:218-262): packed rows*ceil(cols/2) bytes (even column
 * in the low nibble), fp32 scales and zeros rows*ceil(cols/group) each; version 1 means
 * (code - zero) * scale, version 2 means code * scale + zero. Host pointers. */
XQK_API int xqk_matrix_create(const uint8_t* packed, const float* scales, const float* zeros, int rows,
                              int cols, int group_size, int version, int device, xqk_matrix** out);
XQK_API void xqk_matrix_destroy(xqk_matrix* m);
/* rows, cols, device bytes, row stride, layout kind (0 fp16 scale with zero 8, 1 fp32
 * scale/offset pairs, 2 generic), and whether the fused fast kernel serves this shape. */
XQK_API int xqk_matrix_info(const xqk_matrix* m, int* rows, int* cols, size_t* device_bytes, int* row_stride,
                            int* layout_kind, int* fast_path);

/* y = W x, fp32 in/out, device pointers (gemvW4A16Neon, xq_gemv_w4a16_neon.cpp:259). */
XQK_API int xqk_gemv_w4a16(const xqk_matrix* m, const float* x_dev, float* y_dev, void* stream);
/* y = W x on the integer tensor cores (mma.sync m16n8k32, u8 weight codes x s8 digits of x,
 * exact s32 sums, group scale applied once per row and group). No reference counterpart: the
 * same mathematics as xqk_gemv_w4a16 with x held per 64-column group instead of per 32
 * columns, so results agree with it to fp32 rounding, not bit for bit. Served for symmetric
 * version-1 matrices (zero 8) with group 64, fp16-exact scales, cols a multiple of 512 (and
 * of 4096 above 4096), which xqk_matrix_create then also stores in the tensor-core tile
 * layout; other matrices return XQ_ERR_NOT_READY (-2). A non-finite x makes every row NaN, as
 * in fp32. */
XQK_API int xqk_gemv_w4a16_mma(const xqk_matrix* m, const float* x_dev, float* y_dev, void* stream);
/* xqk_gemv_w4a16_mma with fp16 activations: x and y are fp16 device vectors (x 8-byte
 * aligned), the arithmetic is the same exact-integer / fp32 path and y is rounded to fp16 once.
 * The benchmark's single-GEMV configuration (x fp16 [4096], y fp16, fp32 accumulate) in its own
 * format; the reference kernel takes fp32 vectors (gemvW4A16Neon, xq_gemv_w4a16_neon.cpp:259).
 * Both tensor-core GEMVs launch with programmatic dependent launch: the weight stream may start
 * while the previous kernel in the stream finishes, x is read only after it has finished. */
XQK_API int xqk_gemv_w4a16_mma_f16(const xqk_matrix* m, const void* x_dev, void* y_dev, void* stream);
/* Batched W4A16 GEMM for prefill on the 5th-generation tensor cores (tcgen05.mma, fp32
 * accumulators in tensor memory): Y[t][n] = sum_k X[t][k] W[n][k] for t < n_tokens and every
 * row n of m. Replaces the token-serial use of gemvW4A16Neon in CustomModel::prefill
 * (custom_model.cpp:610-640, xq_gemv_w4a16_neon.cpp:259-291) by one GEMM per matrix.
 * x_dev: bf16 [n_tokens][cols] row-major, 16-byte aligned. x_lo_dev: NULL for one bf16 pass
 * (W dequantised to bf16 in shared memory, then X W^T); or the bf16 residual X - X_hi for split
 * mode, where W is also carried as a bf16 pair and three products are accumulated (relative error
 * about 2^-16, near the fp32 path). y_dev: ldy elements per token row (ldy >= rows); out_kind 0 =
 * store fp32, 1 = add into fp32 y, 2 = store bf16. Needs a symmetric matrix (zero 8, fp16-exact
 * scales, group 64, kind 0 of xqk_matrix_info). Asynchronous on `stream`.
 * n_tokens <= 64 (batched decode, short prompt chunks) runs a small-M kernel that multiplies the
 * exact integer codes and applies each group's scale to that group's fp32 partial sum: W is then
 * exact in both modes (one pass: bf16 X times the exact W), and its split-K reduction across a
 * thread-block cluster has a fixed order, so results are bit-reproducible run to run. */
XQK_API int xqk_prefill_gemm_w4a16(const xqk_matrix* m, const void* x_dev, const void* x_lo_dev, int n_tokens,
                                   void* y_dev, int ldy, int out_kind, void* stream);
/* The tensor-core tile layout of a symmetric matrix, written to a host buffer (host only, no
 * GPU): no reference counterpart; for packaging pipelines and tests. packed: rows * cols / 2
 * bytes in the reference's nibble order, scales: rows * cols / 64 fp32 (zero 8 implied, scales
 * stored as fp16). Per 16-row tile and per 128 columns, 1088 bytes: four 32-column slabs of 256
 * bytes (lane L's 8 bytes: byte j of word 0 = code(r, c0 + j) | code(r + 8, c0 + j) << 4, word 1
 * the same for columns c0 + 16 + j, r = 16 * tile + L / 4, c0 = 4 * (L % 4)) then fp16 scales
 * [row r: group 0, group 1 | row r + 8: group 0, group 1] for r = 0..7. Rows past `rows` are
 * code 8, scale 0. *written = the size needed; XQ_ERR_BUFFER_TOO_SMALL (-5) if capacity is
 * short; cols must be a multiple of 128. */
XQK_API int xqk_mma_tiles(const uint8_t* packed, const float* scales, int rows, int cols, uint8_t* out,
                          size_t capacity, size_t* written);
/* Same with host buffers: copies x in, runs, copies y out, synchronises. */
XQK_API int xqk_gemv_w4a16_host(const xqk_matrix* m, const float* x_host, float* y_host);
/* argmax_r (W x)[r], ties to the lowest index (gemvW4A16ArgmaxNeon,
 * xq_gemv_w4a16_neon.cpp:293-348); writes the index and the value to device memory. Uses
 * per-matrix scratch allocated at creation: calls on one matrix must not overlap. */
XQK_API int xqk_gemv_w4a16_argmax(const xqk_matrix* m, const float* x_dev, int32_t* index_dev,
                                  float* value_dev, void* stream);

/* y = x * rsqrt(mean(x^2) + eps) * w (rmsnormReference, ref_rmsnorm.cpp:8-17). */
XQK_API int xqk_rmsnorm(const float* x_dev, const float* w_dev, int n, float eps, float* y_dev, void* stream);

/* One Gated-DeltaNet decode step for all value heads, the fused form the runtime uses:
 * l2-normalise q and k per key head (custom_model.cpp:315-327), beta = sigmoid(b),
 * g = -exp(A_log) * softplus(a + dt_bias) (custom_model.cpp:1075-1082), then the
 * gated delta rule per head (gatedDeltaDecodeReference, ref_delta.cpp:8-41).
 * conv_dev: [2*nk*dk + nv*dv] = q | k | v after conv+SiLU; ab_dev: [a (nv) | b (nv)];
 * state_dev: [nv][dk][dv] fp32, updated in place; out_dev: [nv*dv]. dk = dv = 128. */
XQK_API int xqk_gated_delta_step(const float* conv_dev, const float* ab_dev, const float* a_log_dev,
                                 const float* dt_bias_dev, float* state_dev, float* out_dev, int nk, int nv,
                                 int dk, int dv, void* stream);

/* One full-attention decode step for one layer, the fused form the runtime uses:
 * per-head [query|gate] split of q_proj rows (custom_model.cpp:740-753), head RMSNorm on q
 * and k (applyHeadRms, :301-313), partial NeoX RoPE (applyRopeVector, :351-370), KV append
 * at `position` (appendKv, :673-733, layout [t][kv_head][head_dim]), GQA softmax attention
 * over positions 0..position (:871-928) and the sigmoid output gate (:944-946).
 * qkv_dev: [2*nq*hd | nkv*hd | nkv*hd] raw projections; q_norm/k_norm with +1 applied;
 * k_cache/v_cache: [capacity][nkv][hd], fp32 (kv_fp16 = 0) or fp16 (kv_fp16 = 1).
 * out_dev: [nq*hd]. Uses internal scratch sized for `capacity`; calls must not overlap. */
XQK_API int xqk_attention_step(const float* qkv_dev, const float* q_norm_dev, const float* k_norm_dev,
                               void* k_cache_dev, void* v_cache_dev, int kv_fp16, int capacity, int position,
                               int nq, int nkv, int hd, int rotary_dim, float theta, float eps, float* out_dev,
                               void* stream);

/* xqk_attention_step without any device allocation. No counterpart in the reference (whose
 * CPU kernels need no device memory); it exists for callers that cannot call cudaMalloc
 * while they run: plugin-style hosts that provide every buffer themselves, code under a
 * fixed device-memory budget, or paths where an allocation would synchronise the device.
 * Same arguments, arithmetic and results as xqk_attention_step. Its scratch is a 1 MiB
 * static device array compiled into the library, held by every GPU that loads the library
 * until the process exits; calls needing more (nkv * 32 * (nq / nkv) * (head_dim + 2) + 128
 * floats above 262144, or more than 64 kv heads) are rejected with an error. The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress), so make that first
 * call before any stream capture. All calls share the array: calls that overlap on the GPU
 * (other streams, other host threads) race and must be serialised by the caller. */
XQK_API int xqk_attention_step_noalloc(const float* qkv_dev, const float* q_norm_dev, const float* k_norm_dev,
                                       void* k_cache_dev, void* v_cache_dev, int kv_fp16, int capacity,
                                       int position, int nq, int nkv, int hd, int rotary_dim, float theta, float eps,
                                       float* out_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XQ_KERNELS_H_ */
