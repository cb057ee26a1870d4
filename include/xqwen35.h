/* xqwen35.h: public C ABI of the B200 decode library (libxqwen35.so).
 *
 * Drop-in for the reference header customlib/include/xqwen35.h: every type, enum value and
 * entry point below has the same name, layout and meaning as xqwen35.h:19-77 of the
 * reference, so a host that compiled against that header links against this library
 * unchanged. The work behind it runs on an NVIDIA B200 (sm_100a): weights, KV cache and
 * recurrent state live in HBM and each decode step is one launch of a persistent cooperative
 * kernel (shapes that kernel does not take run the step as a CUDA graph of per-op kernels).
 *
 * Additions (not in the reference): xq_cuda_options + xq_create_cuda, to pick the device
 * and KV-cache precision; everything else is the reference interface.
 */
#ifndef XQWEN35_H_
#define XQWEN35_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XQ_API __attribute__((visibility("default")))

/* Opaque session handle (reference xqwen35.h:19). */
typedef struct xq_session xq_session;

/* Status codes (reference xqwen35.h:21-28). */
typedef enum xq_status {
    XQ_OK = 0,
    XQ_ERR_INVALID_ARGUMENT = -1,
    XQ_ERR_NOT_READY = -2,
    XQ_ERR_MODEL = -3,
    XQ_ERR_RUNTIME = -4,
    XQ_ERR_BUFFER_TOO_SMALL = -5
} xq_status;

/* Creation options (reference xqwen35.h:30-40). backend: any string is accepted and the
 * CUDA path always runs (there is no CPU fallback); threads, quant_bits, group_size,
 * enable_autotune and telemetry_path are accepted and ignored as in the reference's custom
 * path; max_context_tokens sizes the initial KV cache (it grows on demand);
 * use_mnn_fallback is accepted and ignored (the MNN engine is not part of this library). */
typedef struct xq_options {
    size_t struct_size;
    const char* backend;
    int threads;
    int quant_bits;
    int group_size;
    int max_context_tokens;
    int enable_autotune;
    int use_mnn_fallback;
    const char* telemetry_path;
} xq_options;

/* Metrics (reference xqwen35.h:42-58). Copies are bounded by the caller's struct_size. */
typedef struct xq_metrics {
    size_t struct_size;
    uint64_t prompt_tokens;
    uint64_t generated_tokens;
    double load_ms;
    double prefill_ms;
    double first_token_ms;
    double decode_total_ms;
    double total_generate_ms;
    double prefill_tokens_per_second;
    double decode_tokens_per_second;
    uint64_t rss_kb;
    uint64_t pss_kb;
    char backend[64];
    char selected_kernels[512];
    char error[256];
} xq_metrics;

/* Reference xqwen35.h:60 (session.cpp:620-632): load a model directory onto the GPU. */
XQ_API xq_status xq_create(const char* model_dir, const xq_options* options, xq_session** out_session);
/* Reference xqwen35.h:61 (session.cpp:634-636). */
XQ_API void xq_destroy(xq_session* session);
/* Reference xqwen35.h:62 (session.cpp:304-342): token-serial prefill, no logits. */
XQ_API xq_status xq_prefill(xq_session* session, const int32_t* token_ids, size_t n_tokens, xq_metrics* out_metrics);
/* Reference xqwen35.h:63 (session.cpp:344-383): greedy sample, then forward that token. */
XQ_API xq_status xq_decode_one(xq_session* session, int32_t* out_token_id, xq_metrics* out_metrics);
/* Reference xqwen35.h:64-70 (session.cpp:385-421): prefill + max_new_tokens decodes. */
XQ_API xq_status xq_generate(xq_session* session,
                             const int32_t* token_ids,
                             size_t n_tokens,
                             size_t max_new_tokens,
                             int32_t* output_buffer,
                             size_t output_capacity,
                             xq_metrics* out_metrics);
/* Reference xqwen35.h:71 (session.cpp:505-525). */
XQ_API xq_status xq_reset(xq_session* session);
/* Reference xqwen35.h:72. */
XQ_API xq_status xq_get_last_metrics(xq_session* session, xq_metrics* out_metrics);
/* Reference xqwen35.h:73-75: JSON into caller buffers, XQ_ERR_BUFFER_TOO_SMALL if short. */
XQ_API xq_status xq_get_backend_info(xq_session* session, char* json_out, size_t json_capacity);
XQ_API xq_status xq_get_kernel_trace_json(xq_session* session, char* json_out, size_t json_capacity);
XQ_API xq_status xq_get_debug_json(xq_session* session, char* json_out, size_t json_capacity);
/* Reference xqwen35.h:76 (custom_model.cpp:1438-1447): post-final-norm hidden state. */
XQ_API xq_status xq_get_hidden_state(xq_session* session, float* out_values, size_t value_capacity, size_t* out_size);
/* Reference xqwen35.h:77: kept for link compatibility. The Vulkan path is not part of this
 * library; like the reference on a host without Vulkan it writes a JSON saying so and
 * returns XQ_ERR_RUNTIME (vulkan_backend.cpp:1638-1656). */
XQ_API xq_status xq_run_vulkan_w4a16_selftest(char* json_out, size_t json_capacity);

/* ---- CUDA extension (no reference counterpart) ------------------------------------ */
typedef struct xq_cuda_options {
    size_t struct_size;
    int device;        /* CUDA device ordinal; -1 = XQ_CUDA_DEVICE env var or 0 */
    int kv_fp16;       /* 1 = fp16 KV cache, 0 = fp32 KV cache (the reference's precision) */
    int use_graphs;    /* 1 = capture each decode / prefill step as a CUDA graph (default) */
    /* 1 = prefill with every projection of a layer as one tensor-core GEMM over the prompt
     * (tcgen05, split-bf16 operands: agrees with the token-serial prefill to about 1e-5);
     * 0 = the reference's token-serial prefill; -1 = XQ_PREFILL_BATCHED env var or 0. Packages
     * or contexts the batched path does not serve use the token-serial one. (Field added after
     * use_graphs: callers built against the shorter struct get the default.) */
    int prefill_batched;
} xq_cuda_options;

/* xq_create with an explicit device and KV precision; xq_create uses the defaults
 * (device from XQ_CUDA_DEVICE or 0, fp32 KV unless XQ_KV_FP16=1, graphs on). */
XQ_API xq_status xq_create_cuda(const char* model_dir,
                                const xq_options* options,
                                const xq_cuda_options* cuda_options,
                                xq_session** out_session);

/* Run n greedy decode steps back to back on the session's CUDA stream (one graph launch
 * each, no host round trip between steps) and report their device time from CUDA events
 * recorded on that stream. tokens (optional, capacity >= n) receives the sampled ids.
 * Session metrics advance as for n xq_decode_one calls. */
XQ_API xq_status xq_cuda_decode_timed(xq_session* session, size_t n, int32_t* tokens, double* device_ms);

/* ---- Session snapshot / restore (no reference counterpart; the reference only has
 * xq_reset, session.cpp:505-525) ---------------------------------------------------
 * A snapshot holds everything a later decode step reads: the position, the hidden state the
 * next step samples from, every DeltaNet layer's conv and recurrent state and every attention
 * layer's KV cache up to the position, in a self-describing host buffer (header + raw state).
 * Use it to cache a prompt prefix: prefill once, save, then restore it into this or another
 * session of the same model (same shapes and KV precision) and decode from there.
 *   xq_snapshot_size:    bytes a snapshot of the current state needs.
 *   xq_snapshot_save:    write it; XQ_ERR_BUFFER_TOO_SMALL (with *written = bytes needed)
 *                        if capacity is short; XQ_ERR_NOT_READY before a prefill.
 *   xq_snapshot_restore: replace the session's state; XQ_ERR_INVALID_ARGUMENT if the buffer
 *                        is not a snapshot of a model of this shape / KV type. Afterwards the
 *                        session decodes exactly as it would have after the saved state. */
/* ---- Packed B200 weight layout (no reference counterpart; an addition next to the
 * reference's packer, customlib/packer/pack_qwen35_xq4_numpy.py:191-268) ------------------
 * Write every fused weight matrix of the package in model_dir in the kernels' row layout to
 * model_dir/b200/<name>.b200 and model_dir/b200/layout.json. Runs on the host only (no GPU).
 * xq_create then reads those files instead of re-tiling the xq4 files (their shapes are still
 * checked against the manifest); deleting b200/layout.json returns to the xq4 path.
 * XQ_ERR_INVALID_ARGUMENT for a null dir, XQ_ERR_MODEL (message in error_out) for package
 * problems. */
XQ_API xq_status xq_pack_b200_layout(const char* model_dir, char* error_out, size_t error_capacity);

/* ---- Batched decode (no reference counterpart; the reference decodes one sequence per
 * Session, CustomModel::decodeOne, custom_model.cpp:1340-1356) --------------------------
 * `batch` independent sequences of one package on one device, decoded together: each step
 * makes one pass over the weights for all of them (tensor-core GEMMs with the sequences' tokens
 * as the rows, split-bf16 operands), while every sequence keeps its own DeltaNet state, KV cache
 * (max_context positions) and position and follows the reference's order: greedy argmax of
 * lm_head over its final-normed hidden state (ties to the lowest index), then the forward of
 * that token. A sequence's tokens and hidden states equal those of its own xq_session to the
 * GEMMs' rounding (about 1e-5).
 *   xq_batch_create:       load the package (weights shared with its sessions on the device);
 *                          cuda_options may be NULL (device / KV precision as for xq_create).
 *                          XQ_ERR_MODEL for packages the tensor-core GEMMs do not serve.
 *   xq_batch_prefill:      prefill sequence `seq` (0 <= seq < batch) with its prompt; replaces
 *                          that sequence's state. Every sequence must be prefilled before decoding.
 *   xq_batch_decode:       one step for all sequences; tokens[b] receives sequence b's id.
 *                          XQ_ERR_NOT_READY until every sequence is prefilled.
 *   xq_batch_decode_timed: `steps` steps back to back, *device_ms = their CUDA-event time on the
 *                          batch's stream; tokens (optional) receives [steps][batch] ids. If the
 *                          step graph has not been captured yet, one extra step runs first,
 *                          untimed (its tokens are not returned).
 *   xq_batch_hidden_state: post-final-norm hidden state of sequence `seq`. */
typedef struct xq_batch xq_batch;
XQ_API xq_status xq_batch_create(const char* model_dir, const xq_cuda_options* cuda_options, int batch,
                                 int max_context, xq_batch** out_batch);
XQ_API void xq_batch_destroy(xq_batch* batch);
XQ_API xq_status xq_batch_prefill(xq_batch* batch, int seq, const int32_t* token_ids, size_t n_tokens);
XQ_API xq_status xq_batch_decode(xq_batch* batch, int32_t* tokens);
XQ_API xq_status xq_batch_decode_timed(xq_batch* batch, size_t steps, int32_t* tokens, double* device_ms);
XQ_API xq_status xq_batch_hidden_state(xq_batch* batch, int seq, float* out_values, size_t value_capacity,
                                       size_t* out_size);

/* Tensor-parallel decode of ONE sequence over `world` GPUs of a node (extension; the reference
 * decodes on one CPU). One process per GPU, each with its own xq_tp on cuda_options->device;
 * every rank makes the same calls in the same order. Each rank holds a slice of every matrix
 * (column slices of q/k/v, in_proj and gate/up by head and row; K slices of o_proj, out_proj
 * and down, summed by an NCCL all-reduce; a vocabulary slice of lm_head with a cross-rank
 * (max, lowest index) argmax). NCCL (libnccl.so.2) is loaded at run time.
 *   xq_tp_unique_id:       an NCCL unique id (cap >= 128 bytes), made on one rank and passed
 *                          to every rank's xq_tp_create;
 *   xq_tp_create:          load this rank's shard; returns once every rank has joined;
 *   xq_tp_prefill:         token-serial prefill of the prompt (same ids on every rank);
 *   xq_tp_decode:          `steps` greedy steps (sample, then forward); tokens[i] receives the
 *                          i-th sampled id, *device_ms this rank's CUDA-event time of the steps
 *                          (either pointer may be NULL);
 *   xq_tp_hidden_state:    post-final-norm hidden state (replicated on every rank);
 *   xq_tp_plan:            this rank's shard ranges as JSON (half-open [first, last) per
 *                          dimension), from the package manifest alone (no GPU);
 *   xq_tp_argmax_combine:  the cross-rank rule on host arrays: the largest value wins, equal
 *                          values go to the lowest index, NaN never wins. */
typedef struct xq_tp xq_tp;
XQ_API xq_status xq_tp_unique_id(unsigned char* out, size_t capacity);
XQ_API xq_status xq_tp_create(const char* model_dir, const xq_cuda_options* cuda_options, int world, int rank,
                              const unsigned char* unique_id, int max_context, xq_tp** out_tp);
XQ_API void xq_tp_destroy(xq_tp* tp);
XQ_API xq_status xq_tp_prefill(xq_tp* tp, const int32_t* token_ids, size_t n_tokens);
XQ_API xq_status xq_tp_decode(xq_tp* tp, size_t steps, int32_t* tokens, double* device_ms);
XQ_API xq_status xq_tp_hidden_state(xq_tp* tp, float* out_values, size_t value_capacity, size_t* out_size);
XQ_API xq_status xq_tp_plan(const char* model_dir, int world, int rank, char* json, size_t capacity);
XQ_API xq_status xq_tp_argmax_combine(const float* values, const int32_t* indices, int n, int32_t* out_index);

XQ_API xq_status xq_snapshot_size(xq_session* session, size_t* bytes);
XQ_API xq_status xq_snapshot_save(xq_session* session, void* buffer, size_t capacity, size_t* written);
XQ_API xq_status xq_snapshot_restore(xq_session* session, const void* buffer, size_t size);

#ifdef __cplusplus
}
#endif

#endif /* XQWEN35_H_ */
