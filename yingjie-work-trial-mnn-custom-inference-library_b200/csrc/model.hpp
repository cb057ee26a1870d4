// Device-resident model for the decode hot path (replaces the reference's CustomModel,
// customlib/runtime/custom_model.hpp:38-150, for the CUDA path).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <string>
#include <vector>

#include "gemv.hpp"
#include "stepper.cuh"

namespace xqb {

struct ModelDims {
    int hidden = 4096, inter = 12288, vocab = 248320;
    int heads = 16, kv_heads = 4, head_dim = 256, rotary_dim = 64;
    int lk_hd = 128, lv_hd = 128, lk_heads = 16, lv_heads = 32, conv_k = 4;
    int lk_dim = 2048, lv_dim = 4096, conv_dim = 8192;
    float eps = 1.0e-6f, theta = 10000000.0f;
    int layers = 32;
};

// Manifest parsing with the reference's substring rules (custom_model.cpp:38-87, 431-453).
ModelDims parse_manifest(const std::string& json, int* n_layers);

// Package file helpers shared by the loaders.
std::string read_small_file(const std::string& path);
bool file_exists(const std::string& path);
// `expected` floats from a raw little-endian f32 file (false, error set, when missing or short).
bool read_vec(const std::string& path, int expected, std::vector<float>* out, std::string* error);
// The reference's +1 on RMSNorm weights (custom_model.cpp:524).
void add_one(std::vector<float>* v);

struct DevLayer {
    bool full = false;
    DevMatrix in_proj;   // linear: [qkv | z | a | b]; full: [q(+gate) | k | v]
    DevMatrix out_proj;  // linear: out_proj; full: o_proj
    DevMatrix gate_up;   // rows interleaved gate_0, up_0, gate_1, ...
    DevMatrix down;
    float* input_norm = nullptr;  // +1 applied (custom_model.cpp:524)
    float* post_norm = nullptr;
    float* q_norm = nullptr;  // full, +1
    float* k_norm = nullptr;
    float* lin_norm = nullptr;  // linear, no +1 (custom_model.cpp:546)
    float* conv_w = nullptr;
    float* a_log = nullptr;
    float* dt_bias = nullptr;
    float* conv_state = nullptr;  // [conv_dim][conv_k - 1]
    float* rec_state = nullptr;   // [lv_heads][lk_hd][lv_hd]
    void* k_cache = nullptr;      // [capacity][kv_heads][head_dim]
    void* v_cache = nullptr;
};

// Write the fused weight matrices of the package in `dir` in the device row layout to
// dir/b200/*.b200 plus dir/b200/layout.json (host only, no GPU needed); the loader then reads
// them instead of re-tiling the xq4 files.
bool pack_b200_layout(const std::string& dir, std::string* error);

struct SharedWeights;

// Tokens per chunk of the batched prefill (its activation buffers are sized for this).
constexpr int kPrefillChunk = 1024;

struct Options {
    int device = 0;
    bool kv_fp16 = false;
    bool use_graphs = true;
    bool persistent = true;  // one cooperative persistent kernel per step when the model allows it
    bool prefill_batched = false;  // prefill through the tensor-core GEMMs (prefill_batched)
    int initial_capacity = 8192;
};

class DeviceModel {
public:
    DeviceModel() = default;
    ~DeviceModel();
    DeviceModel(const DeviceModel&) = delete;
    DeviceModel& operator=(const DeviceModel&) = delete;

    bool load(const std::string& model_dir, const Options& opts, std::string* error);
    // CustomModel::resetState (custom_model.cpp:555-567) + position 0.
    bool reset(std::string* error);
    // CustomModel::prefill (custom_model.cpp:610-640): reset, then one forward per token.
    bool prefill(const int32_t* ids, size_t n, std::string* error);
    // The same prefill with every projection of a layer as one tensor-core GEMM over the prompt
    // (chunks of up to kPrefillChunk tokens): embeddings, RMSNorm, GEMMs (split-bf16 by default,
    // XQ_PREFILL_PASSES=1 for one bf16 pass), causal conv + the gated delta rule over the sequence,
    // q/k norm + RoPE + KV append, causal attention, SwiGLU, residual adds. Leaves the same state
    // as prefill() (positions, hidden, conv / recurrent states, KV cache) up to rounding.
    // false with *unsupported set when this package's layout or the context needs the
    // token-serial path.
    bool prefill_batched(const int32_t* ids, size_t n, std::string* error, bool* unsupported);
    bool batched_prefill_eligible(size_t n) const;
    // CustomModel::decodeOne (custom_model.cpp:1340-1356): sample, then forward it.
    bool decode_one(int32_t* token, std::string* error);
    // Enqueue `count` decode steps without host synchronisation; tokens land in the ring.
    bool decode_many(size_t count, std::string* error);
    bool read_ring(size_t first, size_t count, int32_t* out, std::string* error);
    // decode_many bracketed by CUDA events on the model stream; returns device milliseconds.
    bool decode_many_timed(size_t count, double* device_ms, std::string* error);
    // Post-final-norm hidden state (what copyHidden returns, custom_model.cpp:1438-1447).
    bool hidden(std::vector<float>* out, std::string* error);
    // Full lm_head logits of the current (normed) hidden state, for debug JSON.
    bool logits(std::vector<float>* out, std::string* error);
    // Decode-state snapshot (no reference counterpart): positions, the hidden state the next
    // step samples from, DeltaNet conv + recurrent states, and the KV cache up to the position,
    // in a self-describing host buffer. Restoring needs a model of the same shape and KV type.
    size_t snapshot_bytes() const;
    bool save_snapshot(void* buf, size_t cap, size_t* written, std::string* error);
    // *invalid is set when the buffer is not a snapshot of a model of this shape / KV type.
    bool restore_snapshot(const void* buf, size_t size, std::string* error, bool* invalid);
    // Device error word set by bounded waits; 0 when clean.
    unsigned device_errors();
    // Zero the error word and the step kernel's barrier and merge counters (session stream).
    void clear_device_errors();
    // false (with a message) when the error word is set after `what`; the word is then cleared
    // so that xq_reset and later steps start clean.
    bool check_device_errors(const char* what, std::string* error);

    const ModelDims& dims() const { return d_; }
    size_t weight_bytes() const { return weight_bytes_; }
    size_t device_bytes() const { return device_bytes_; }
    int position() const { return position_; }
    int capacity() const { return capacity_; }
    bool kv_fp16() const { return opts_.kv_fp16; }
    int kernels_per_decode_step() const;
    int kernels_per_prefill_step() const;
    bool persistent() const { return persistent_; }
    bool tensor_core_step() const { return persistent_ && meta_kind_ == kMetaMma; }
    bool packed_layout() const { return packed_layout_; }
    // Whether this session found its weights already loaded by another live session.
    bool weights_reused() const { return weights_reused_; }
    // Sessions (this one included) currently holding this session's weights.
    long weights_users() const { return weights_.use_count(); }
    cudaStream_t stream() const { return stream_; }
    const std::vector<DevLayer>& layers() const { return layers_; }
    const DevMatrix& lm_head() const { return lm_head_; }
    float* hidden_ptr() const { return d_hidden_; }
    float* final_norm_ptr() const { return d_final_norm_; }
    const uint16_t* embeddings() const { return d_emb_; }
    int num_sms() const { return num_sms_; }

    // Launch sequences (used by graph capture and by the eager path).
    bool enqueue_decode_step(cudaStream_t s);
    bool enqueue_prefill_step(cudaStream_t s);

    // Whether this model runs the generic-shape step (shapes the fused kernels do not take).
    bool generic() const { return generic_; }

private:
    bool enqueue_forward(cudaStream_t s);
    bool enqueue_generic_step(bool decode, cudaStream_t s);
    bool gemv_any(const DevMatrix& m, const float* x, float* y, cudaStream_t s);
    bool ensure_capacity(int needed, std::string* error);
    bool alloc_kv(int capacity, std::string* error);
    bool capture_graphs(std::string* error);
    void destroy_graphs();
    bool run_step(bool decode, std::string* error);
    bool build_phases(std::string* error);
    bool persistent_eligible(int capacity) const;
    template <typename T>
    bool dev_alloc(T** p, size_t count, std::string* error);
    bool upload_vec(float** dst, const std::vector<float>& v, std::string* error);

    ModelDims d_;
    Options opts_;
    std::vector<DevLayer> layers_;
    DevMatrix lm_head_;
    float* d_final_norm_ = nullptr;
    uint16_t* d_emb_ = nullptr;
    // activations
    float *d_hidden_ = nullptr, *d_conv_out_ = nullptr, *d_zab_ = nullptr, *d_attn_raw_ = nullptr;
    float *d_qkv_ = nullptr, *d_attn_out_ = nullptr, *d_ffn_ = nullptr, *d_normed_ = nullptr, *d_logits_ = nullptr;
    // step control
    int *d_pos_ = nullptr, *d_next_pos_ = nullptr, *d_token_ = nullptr, *d_ring_ = nullptr, *d_ring_ctr_ = nullptr;
    int* d_prompt_ = nullptr;
    size_t prompt_cap_ = 0;
    float* d_arg_val_ = nullptr;
    int* d_arg_idx_ = nullptr;
    unsigned* d_arg_counter_ = nullptr;
    float2* d_rope_ = nullptr;  // [capacity][rotary/2] (cos, sin), rebuilt when the KV cache grows
    float* d_attn_part_ = nullptr;
    float* d_head_ss_ = nullptr;  // DeltaNet phase -> out_proj: per-slice sums of squares
    bool generic_ = false;        // generic-shape step (generic.cu)
    float *d_gy_ = nullptr, *d_gqbuf_ = nullptr, *d_gscore_ = nullptr;  // its scratch
    unsigned* d_attn_counters_ = nullptr;
    unsigned* d_err_ = nullptr;
    int32_t* h_token_ = nullptr;  // pinned
    unsigned* h_err_ = nullptr;   // pinned
    // batched prefill buffers (allocated on first use, sized for kPrefillChunk tokens)
    float *pf_H_ = nullptr, *pf_Y_ = nullptr, *pf_conv_ = nullptr, *pf_O_ = nullptr, *pf_Q_ = nullptr;
    void *pf_xhi_ = nullptr, *pf_xlo_ = nullptr;
    int* pf_ids_ = nullptr;
    int pf_ymax_ = 0, pf_kmax_ = 0;
    int ring_cap_ = 1 << 16;

    cudaStream_t stream_ = nullptr;
    cudaGraphExec_t g_decode_ = nullptr, g_prefill_ = nullptr;
    int num_sms_ = 148;
    int capacity_ = 0;
    int position_ = 0;  // host mirror of *d_next_pos_
    size_t ring_count_ = 0;  // host mirror of *d_ring_ctr_
    size_t weight_bytes_ = 0, device_bytes_ = 0;
    std::vector<void*> allocs_;
    bool loaded_ = false;
    // persistent step kernel
    bool persistent_ = false;
    int meta_kind_ = 0;
    int step_slots_ = 0;
    int step_slot_bytes_ = kStepSlotBytes;
    int step_inflight_ = 0;
    int step_l2_prefetch_ = 1;
    int step_l2_ahead_ = 0;  // chunks (XQ_STEP_L2_AHEAD); prefetching into L2 measured slower
    unsigned long long step_wait_ns_ = 0;  // 0: the kernels' default limit (2 s)
    long long stall_launch_ = -1;          // failure-detection test hook (XQ_TEST_STALL_LAUNCH)
    long long step_launches_ = 0;          // step-kernel launches since load
    PhaseDesc* d_phases_decode_ = nullptr;
    void* d_tmaps_ = nullptr;  // CUtensorMap array of the phase lists
    bool packed_layout_ = false;  // weights read from b200/*.b200
    std::shared_ptr<SharedWeights> weights_;  // read-only weights, shared per package and device
    bool weights_reused_ = false;
    unsigned long long* d_block_done_ = nullptr;  // XQ_STEP_TRACE >= 2: per-block phase finish times
    std::vector<double> block_late_ns_;
    std::vector<double> barrier_ns_;
    PhaseDesc* d_phases_prefill_ = nullptr;
    int n_phases_ = 0;
    unsigned* d_grid_bar_ = nullptr;
    unsigned long long* d_step_trace_ = nullptr;  // XQ_STEP_TRACE=1: per-phase timestamps
    std::vector<double> phase_ns_;                // accumulated [phase][3] durations
    std::vector<std::string> phase_names_;
    int traced_steps_ = 0;

public:
    // Per-phase device time summary of the persistent kernel (empty unless tracing).
    std::string phase_trace_summary() const;
    // Per phase name: (phases per step, traced steps, summed device us per step from the phase
    // start to its last block's arrival); empty unless XQ_STEP_TRACE recorded steps.
    struct PhaseTime {
        std::string name;
        int per_step;
        int steps;
        double us_per_step;
    };
    std::vector<PhaseTime> phase_times() const;

private:
};

}  // namespace xqb
