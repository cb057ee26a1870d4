// Batched decode: B independent sequences of one model on one device, decoded together. Every
// step runs ONE pass over the weights for all B tokens (the tcgen05 GEMMs of prefill_gemm.cu with
// M = B, split-bf16 operands) and the per-sequence operations with each sequence's own DeltaNet
// conv / recurrent state, KV cache and position. Each sequence follows the reference's decode
// order (CustomModel::decodeOne, custom_model.cpp:1340-1356: greedy argmax of lm_head over the
// final-normed hidden state, then the forward of that token). No reference counterpart: the
// reference decodes one sequence per Session.
//
// A sequence is prefilled on its own through the single-sequence engine (batched prefill when
// the package allows it, else token-serial), and its state is then copied into the sequence's
// slot. The decode step is captured once as a CUDA graph; positions live on the device.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/xqwen35.h"
#include "model.hpp"
#include "ops.cuh"
#include "prefill_gemm.hpp"
#include "prefill_ops.hpp"

namespace xqb {

namespace {

// pos[b] = next[b]++ (the position the step's forward writes), and the sampled tokens into the
// ring at ring[(*ctr % ring_steps) * B + b].
__global__ void batch_advance_kernel(const int* tokens, int* pos, int* next, int* ring, int* ctr, int ring_steps, int B) {
    pdl_launch_dependents();  // programmatic dependent launch: inputs only after the
    pdl_wait();               // previous kernel has finished
    const int b = threadIdx.x;
    const int k = *ctr;
    __syncthreads();
    if (b < B) {
        pos[b] = next[b];
        next[b] = next[b] + 1;
        ring[static_cast<size_t>(k % ring_steps) * B + b] = tokens[b];
    }
    __syncthreads();
    if (b == 0) *ctr = k + 1;
}

class BatchModel {
public:
    ~BatchModel();
    bool create(const std::string& dir, const Options& opts, int batch, int max_context, std::string* err);
    bool prefill(int seq, const int32_t* ids, size_t n, std::string* err);
    bool decode(int32_t* tokens, std::string* err);
    bool decode_timed(size_t steps, int32_t* tokens, double* device_ms, std::string* err);
    bool hidden(int seq, float* out, size_t cap, size_t* n, std::string* err);
    int batch() const { return B_; }

private:
    bool enqueue_step(cudaStream_t s, std::string* err);
    bool launch_step(std::string* err);
    bool read_ring(size_t first, size_t steps, int32_t* out, std::string* err);
    template <typename T>
    bool alloc(T** p, size_t count, std::string* err) {
        *p = nullptr;
        if (cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(1, count) * sizeof(T)) != cudaSuccess) {
            *err = "batched decode: device allocation failed";
            return false;
        }
        allocs_.push_back(*p);
        return true;
    }

    DeviceModel model_;  // weights (shared per package and device) + the single-sequence prefill
    Options opts_;
    int B_ = 0, cap_ = 0;
    size_t conv_sz_ = 0, rec_sz_ = 0, kv_bstride_ = 0;
    std::vector<float*> conv_state_, rec_state_;  // per layer ([B][...], linear layers)
    std::vector<void*> k_cache_, v_cache_;        // per layer ([B][cap][nkv][hd], full layers)
    float *H_ = nullptr, *Y_ = nullptr, *conv_ = nullptr, *O_ = nullptr, *logits_ = nullptr;
    float* attn_part_ = nullptr;        // [B][nkv][kAttnSplits][group][hd + 2]
    unsigned* attn_counters_ = nullptr;  // [B][nkv], zero between steps
    float* hid_ = nullptr;
    __nv_bfloat16 *xhi_ = nullptr, *xlo_ = nullptr;
    int *tokens_ = nullptr, *pos_ = nullptr, *next_ = nullptr, *ring_ = nullptr, *ring_ctr_ = nullptr;
    unsigned* err_ = nullptr;
    float2* rope_ = nullptr;
    int ring_steps_ = 4096;
    size_t ring_count_ = 0;
    std::vector<int> prefilled_;
    std::vector<void*> allocs_;
    cudaStream_t stream_ = nullptr;
    cudaGraphExec_t graph_ = nullptr;
};

BatchModel::~BatchModel() {
    cudaSetDevice(opts_.device);
    if (stream_) cudaStreamSynchronize(stream_);
    if (graph_) cudaGraphExecDestroy(graph_);
    for (void* p : allocs_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
}

bool BatchModel::create(const std::string& dir, const Options& opts, int batch, int max_context, std::string* err) {
    opts_ = opts;
    opts_.persistent = true;
    if (batch < 1 || batch > 256 || max_context < 2) {
        *err = "batched decode: batch must be 1..256 and max_context >= 2";
        return false;
    }
    Options mo = opts_;
    mo.initial_capacity = std::max(64, max_context);
    if (!model_.load(dir, mo, err)) return false;
    const ModelDims& d = model_.dims();
    if (!model_.batched_prefill_eligible(1) || d.kv_heads <= 0 || d.heads % d.kv_heads != 0 ||
        d.heads / d.kv_heads > kAttnMaxGroup || d.head_dim != kAttnThreads ||
        attention_smem_bytes(d.heads, d.kv_heads, d.head_dim, max_context) > 200 * 1024) {
        *err = "batched decode needs a symmetric W4A16 package the tensor-core GEMMs serve (and a context the "
               "attention kernel holds)";
        return false;
    }
    B_ = batch;
    cap_ = max_context;
    cudaSetDevice(opts_.device);
    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) {
        *err = "batched decode: stream creation failed";
        return false;
    }
    conv_sz_ = static_cast<size_t>(d.conv_dim) * std::max(0, d.conv_k - 1);
    rec_sz_ = static_cast<size_t>(d.lv_heads) * d.lk_hd * d.lv_hd;
    const size_t elem = opts_.kv_fp16 ? 2 : 4;
    kv_bstride_ = static_cast<size_t>(cap_) * d.kv_heads * d.head_dim;  // elements per sequence
    const auto& L = model_.layers();
    conv_state_.assign(L.size(), nullptr);
    rec_state_.assign(L.size(), nullptr);
    k_cache_.assign(L.size(), nullptr);
    v_cache_.assign(L.size(), nullptr);
    for (size_t l = 0; l < L.size(); ++l) {
        if (L[l].full) {
            uint8_t *k = nullptr, *v = nullptr;
            if (!alloc(&k, kv_bstride_ * elem * B_, err) || !alloc(&v, kv_bstride_ * elem * B_, err)) return false;
            k_cache_[l] = k;
            v_cache_[l] = v;
        } else if (!alloc(&conv_state_[l], conv_sz_ * B_, err) || !alloc(&rec_state_[l], rec_sz_ * B_, err)) {
            return false;
        }
    }
    int ymax = 0;
    for (const DevLayer& l : L) ymax = std::max({ymax, l.in_proj.rows, l.gate_up.rows});
    const int kmax = std::max({d.hidden, d.inter, d.lv_dim, d.heads * d.head_dim});
    if (!alloc(&H_, static_cast<size_t>(B_) * d.hidden, err) || !alloc(&Y_, static_cast<size_t>(B_) * ymax, err) ||
        !alloc(&conv_, static_cast<size_t>(B_) * d.conv_dim, err) || !alloc(&O_, static_cast<size_t>(B_) * d.lv_dim, err) ||
        !alloc(&attn_part_, static_cast<size_t>(B_) * d.kv_heads * kAttnSplits * (d.heads / d.kv_heads) * (d.head_dim + 2),
               err) ||
        !alloc(&attn_counters_, static_cast<size_t>(B_) * d.kv_heads, err) ||
        !alloc(&logits_, static_cast<size_t>(B_) * d.vocab, err) || !alloc(&hid_, d.hidden, err) ||
        !alloc(&xhi_, static_cast<size_t>(B_) * kmax, err) || !alloc(&xlo_, static_cast<size_t>(B_) * kmax, err) ||
        !alloc(&tokens_, B_, err) || !alloc(&pos_, B_, err) || !alloc(&next_, B_, err) ||
        !alloc(&ring_, static_cast<size_t>(ring_steps_) * B_, err) || !alloc(&ring_ctr_, 1, err) || !alloc(&err_, 1, err))
        return false;
    std::vector<float2> rope;
    rope_table(0, cap_, d.rotary_dim, d.theta, &rope);
    if (!alloc(&rope_, rope.size(), err) ||
        cudaMemcpy(rope_, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(ring_ctr_, 0, sizeof(int)) != cudaSuccess || cudaMemset(err_, 0, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(attn_counters_, 0, sizeof(unsigned) * B_ * d.kv_heads) != cudaSuccess ||
        cudaMemset(next_, 0, sizeof(int) * B_) != cudaSuccess) {
        *err = "batched decode: set-up copies failed";
        return false;
    }
    prefilled_.assign(B_, 0);
    return true;
}

bool BatchModel::prefill(int seq, const int32_t* ids, size_t n, std::string* err) {
    if (seq < 0 || seq >= B_ || !ids || n == 0) {
        *err = "batched decode: invalid sequence index or empty prompt";
        return false;
    }
    if (n + 1 > static_cast<size_t>(cap_)) {
        *err = "batched decode: prompt longer than the batch's context";
        return false;
    }
    bool unsupported = false;
    if (!model_.prefill_batched(ids, n, err, &unsupported)) {
        if (!unsupported || !model_.prefill(ids, n, err)) return false;
    }
    // the single-sequence state into this sequence's slot
    const ModelDims& d = model_.dims();
    cudaStream_t s = model_.stream();
    const auto& L = model_.layers();
    const size_t elem = opts_.kv_fp16 ? 2 : 4;
    const size_t row = static_cast<size_t>(d.kv_heads) * d.head_dim * elem;
    bool ok = cudaMemcpyAsync(H_ + static_cast<size_t>(seq) * d.hidden, model_.hidden_ptr(), sizeof(float) * d.hidden,
                              cudaMemcpyDeviceToDevice, s) == cudaSuccess;
    for (size_t l = 0; l < L.size() && ok; ++l) {
        if (L[l].full) {
            ok = cudaMemcpyAsync(static_cast<uint8_t*>(k_cache_[l]) + seq * kv_bstride_ * elem, L[l].k_cache, row * n,
                                 cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpyAsync(static_cast<uint8_t*>(v_cache_[l]) + seq * kv_bstride_ * elem, L[l].v_cache, row * n,
                                 cudaMemcpyDeviceToDevice, s) == cudaSuccess;
        } else {
            ok = cudaMemcpyAsync(conv_state_[l] + seq * conv_sz_, L[l].conv_state, sizeof(float) * conv_sz_,
                                 cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpyAsync(rec_state_[l] + seq * rec_sz_, L[l].rec_state, sizeof(float) * rec_sz_,
                                 cudaMemcpyDeviceToDevice, s) == cudaSuccess;
        }
    }
    const int np = static_cast<int>(n);
    ok = ok && cudaMemcpyAsync(next_ + seq, &np, sizeof(int), cudaMemcpyHostToDevice, s) == cudaSuccess &&
         cudaStreamSynchronize(s) == cudaSuccess;
    if (!ok) {
        *err = "batched decode: copying the prefilled state failed";
        return false;
    }
    prefilled_[seq] = 1;
    return true;
}

bool BatchModel::enqueue_step(cudaStream_t s, std::string* err) {
    const ModelDims& d = model_.dims();
    const bool f16 = opts_.kv_fp16;
    auto ok = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        *err = std::string("batched decode: ") + what + ": " + cudaGetErrorString(e);
        return false;
    };
    auto gemm = [&](const DevMatrix& m, float* y, int ldy, int kind) {
        if (launch_prefill_gemm(m, xhi_, xlo_, B_, y, ldy, kind, err_, model_.num_sms(), s)) return true;
        *err = std::string("batched decode: ") + last_error();
        return false;
    };
    // sample (final norm, lm_head, argmax), advance positions, embed the sampled tokens
    if (!ok(prefill_rmsnorm_split(H_, model_.final_norm_ptr(), B_, d.hidden, d.eps, xhi_, xlo_, s), "final norm") ||
        !gemm(model_.lm_head(), logits_, d.vocab, kPgOutF32) ||
        !ok(batch_argmax(logits_, B_, d.vocab, tokens_, s), "argmax"))
        return false;
    launch_ex(batch_advance_kernel, dim3(1), dim3(std::max(32, (B_ + 31) / 32 * 32)), 0, s, pdl_enabled(), tokens_, pos_,
              next_, ring_, ring_ctr_, ring_steps_, B_);
    if (!ok(cudaGetLastError(), "advance") ||
        !ok(prefill_embed(tokens_, model_.embeddings(), H_, B_, d.hidden, d.vocab, s), "embedding"))
        return false;
    const auto& L = model_.layers();
    for (size_t l = 0; l < L.size(); ++l) {
        const DevLayer& ly = L[l];
        if (!ok(prefill_rmsnorm_split(H_, ly.input_norm, B_, d.hidden, d.eps, xhi_, xlo_, s), "input norm")) return false;
        const int ldy = ly.in_proj.rows;
        if (!gemm(ly.in_proj, Y_, ldy, kPgOutF32)) return false;
        if (!ly.full) {
            if (!ok(prefill_conv(Y_, ldy, ly.conv_w, conv_state_[l], conv_, 1, d.conv_dim, s, B_, conv_sz_), "conv") ||
                !ok(prefill_delta(conv_, d.conv_dim, Y_, ldy, d.conv_dim + d.lv_dim, ly.a_log, ly.dt_bias, rec_state_[l],
                                  O_, d.lv_dim, 1, d.lk_heads, d.lv_heads, d.lk_hd, d.lv_hd, s, B_, rec_sz_),
                    "gated delta") ||
                !ok(prefill_gated_norm(O_, d.lv_dim, Y_, ldy, d.conv_dim, ly.lin_norm, d.lv_heads, d.lv_hd, d.eps, B_,
                                       xhi_, xlo_, s),
                    "gated norm"))
                return false;
        } else {
            // split-K decode attention per sequence (q/k norm, RoPE, KV append, 32 splits with
            // the merge by the last split, sigmoid gate), output as the o_proj bf16 pair
            AttnParams ap = {};
            ap.qkv = Y_;
            ap.q_norm = ly.q_norm;
            ap.k_norm = ly.k_norm;
            ap.k_cache = k_cache_[l];
            ap.v_cache = v_cache_[l];
            ap.capacity = cap_;
            ap.pos_ptr = pos_;
            ap.nq = d.heads;
            ap.nkv = d.kv_heads;
            ap.hd = d.head_dim;
            ap.rotary = d.rotary_dim;
            ap.theta = d.theta;
            ap.eps = d.eps;
            ap.rope = rope_;
            ap.rope_stride = d.rotary_dim / 2;
            ap.part = attn_part_;
            ap.counters = attn_counters_;
            ap.err = err_;
            if (!ok(launch_attention_batch(ap, f16, attention_smem_bytes(d.heads, d.kv_heads, d.head_dim, cap_), B_,
                                           ldy, kv_bstride_, xhi_, xlo_, s),
                    "attention"))
                return false;
        }
        if (!gemm(ly.out_proj, H_, d.hidden, kPgOutAddF32) ||
            !ok(prefill_rmsnorm_split(H_, ly.post_norm, B_, d.hidden, d.eps, xhi_, xlo_, s), "post norm") ||
            !gemm(ly.gate_up, Y_, ly.gate_up.rows, kPgOutF32) ||
            !ok(prefill_swiglu(Y_, ly.gate_up.rows, d.inter, B_, xhi_, xlo_, s), "swiglu") ||
            !gemm(ly.down, H_, d.hidden, kPgOutAddF32))
            return false;
    }
    return true;
}

bool BatchModel::launch_step(std::string* err) {
    for (int b = 0; b < B_; ++b)
        if (!prefilled_[b]) {
            *err = "batched decode requires every sequence to be prefilled";
            return false;
        }
    cudaSetDevice(opts_.device);
    if (!graph_) {
        // captured once from the launch sequence of a step (relaxed mode: the launchers set
        // kernel attributes on their first use), then replayed for every step
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed) != cudaSuccess) {
            *err = "batched decode: stream capture failed to start";
            return false;
        }
        const bool ok = enqueue_step(stream_, err);
        const cudaError_t e = cudaStreamEndCapture(stream_, &g);
        if (!ok || e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            if (ok) *err = std::string("batched decode: capture failed: ") + cudaGetErrorString(e);
            return false;
        }
        const cudaError_t ie = cudaGraphInstantiate(&graph_, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
            *err = std::string("batched decode: graph instantiation failed: ") + cudaGetErrorString(ie);
            return false;
        }
    }
    if (cudaGraphLaunch(graph_, stream_) != cudaSuccess) {
        *err = "batched decode: graph launch failed";
        return false;
    }
    ++ring_count_;
    return true;
}

bool BatchModel::read_ring(size_t first, size_t steps, int32_t* out, std::string* err) {
    for (size_t i = 0; i < steps; ++i) {
        const size_t k = (first + i) % static_cast<size_t>(ring_steps_);
        if (cudaMemcpyAsync(out + i * B_, ring_ + k * B_, sizeof(int) * B_, cudaMemcpyDeviceToHost, stream_) !=
            cudaSuccess) {
            *err = "batched decode: token copy failed";
            return false;
        }
    }
    if (cudaStreamSynchronize(stream_) != cudaSuccess) {
        *err = "batched decode: step failed on the device";
        return false;
    }
    unsigned e = 0;
    cudaMemcpy(&e, err_, sizeof e, cudaMemcpyDeviceToHost);
    if (e) {
        cudaMemset(err_, 0, sizeof(unsigned));
        *err = "batched decode: a bounded device wait ran out or a kernel saw an unsupported configuration";
        return false;
    }
    return true;
}

bool BatchModel::decode(int32_t* tokens, std::string* err) {
    const size_t first = ring_count_;
    if (!launch_step(err)) return false;
    std::vector<int32_t> t(B_);
    if (!read_ring(first, 1, t.data(), err)) return false;
    if (tokens) std::memcpy(tokens, t.data(), sizeof(int32_t) * B_);
    return true;
}

bool BatchModel::decode_timed(size_t steps, int32_t* tokens, double* device_ms, std::string* err) {
    if (steps == 0 || steps > static_cast<size_t>(ring_steps_)) {
        *err = "batched decode: 1 .. 4096 steps per timed call";
        return false;
    }
    // every position the steps write must fit the batch's KV cache
    std::vector<int> next(B_);
    cudaMemcpy(next.data(), next_, sizeof(int) * B_, cudaMemcpyDeviceToHost);
    for (int v : next)
        if (v + static_cast<int>(steps) > cap_) {
            *err = "batched decode: the steps would run past the batch's context";
            return false;
        }
    if (!graph_) {  // the step that captures the graph runs untimed, before the timed steps
        const size_t before = ring_count_;
        if (!launch_step(err)) return false;
        std::vector<int32_t> t(B_);
        if (!read_ring(before, 1, t.data(), err)) return false;
        for (int v : next)
            if (v + 1 + static_cast<int>(steps) > cap_) {
                *err = "batched decode: the steps would run past the batch's context";
                return false;
            }
    }
    const size_t first = ring_count_;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, stream_);
    bool ok = true;
    for (size_t i = 0; i < steps && ok; ++i) ok = launch_step(err);
    cudaEventRecord(e1, stream_);
    cudaEventSynchronize(e1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (!ok) return false;
    *device_ms = static_cast<double>(ms);
    std::vector<int32_t> t(steps * B_);
    if (!read_ring(first, steps, t.data(), err)) return false;
    if (tokens) std::memcpy(tokens, t.data(), sizeof(int32_t) * t.size());
    return true;
}

bool BatchModel::hidden(int seq, float* out, size_t cap, size_t* n, std::string* err) {
    const ModelDims& d = model_.dims();
    if (n) *n = static_cast<size_t>(d.hidden);
    if (seq < 0 || seq >= B_) {
        *err = "batched decode: invalid sequence index";
        return false;
    }
    if (!out) return true;
    if (cap < static_cast<size_t>(d.hidden)) {
        *err = "buffer too small";
        return false;
    }
    cudaSetDevice(opts_.device);
    rmsnorm_kernel<<<1, 1024, 0, stream_>>>(H_ + static_cast<size_t>(seq) * d.hidden, model_.final_norm_ptr(), d.hidden,
                                             d.eps, hid_);
    if (cudaMemcpyAsync(out, hid_, sizeof(float) * d.hidden, cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess) {
        *err = "batched decode: hidden state copy failed";
        return false;
    }
    return true;
}

thread_local std::string g_batch_error;

}  // namespace
}  // namespace xqb

struct xq_batch {
    xqb::BatchModel m;
};

extern "C" {

XQ_API xq_status xq_batch_create(const char* model_dir, const xq_cuda_options* cuda_options, int batch,
                                 int max_context, xq_batch** out) {
    if (!model_dir || !out) return XQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    xqb::Options o;
    if (const char* v = std::getenv("XQ_CUDA_DEVICE")) o.device = std::atoi(v);
    if (const char* v = std::getenv("XQ_KV_FP16")) o.kv_fp16 = std::atoi(v) != 0;
    if (cuda_options) {
        const size_t n = cuda_options->struct_size;
        if (n >= offsetof(xq_cuda_options, device) + sizeof(int) && cuda_options->device >= 0)
            o.device = cuda_options->device;
        if (n >= offsetof(xq_cuda_options, kv_fp16) + sizeof(int)) o.kv_fp16 = cuda_options->kv_fp16 != 0;
    }
    auto b = std::make_unique<xq_batch>();
    std::string err;
    if (!b->m.create(model_dir, o, batch, max_context, &err)) {
        xqb::g_batch_error = err;
        xqb::set_last_error("xq_batch_create: " + err);
        return (batch < 1 || max_context < 2) ? XQ_ERR_INVALID_ARGUMENT : XQ_ERR_MODEL;
    }
    *out = b.release();
    return XQ_OK;
}

XQ_API void xq_batch_destroy(xq_batch* b) { delete b; }

XQ_API xq_status xq_batch_prefill(xq_batch* b, int seq, const int32_t* ids, size_t n) {
    if (!b || !ids || n == 0) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!b->m.prefill(seq, ids, n, &err)) {
        xqb::set_last_error("xq_batch_prefill: " + err);
        return (seq < 0 || seq >= b->m.batch()) ? XQ_ERR_INVALID_ARGUMENT : XQ_ERR_RUNTIME;
    }
    return XQ_OK;
}

XQ_API xq_status xq_batch_decode(xq_batch* b, int32_t* tokens) {
    if (!b) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!b->m.decode(tokens, &err)) {
        xqb::set_last_error("xq_batch_decode: " + err);
        return err.find("prefilled") != std::string::npos ? XQ_ERR_NOT_READY : XQ_ERR_RUNTIME;
    }
    return XQ_OK;
}

XQ_API xq_status xq_batch_decode_timed(xq_batch* b, size_t steps, int32_t* tokens, double* device_ms) {
    if (!b || !device_ms) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!b->m.decode_timed(steps, tokens, device_ms, &err)) {
        xqb::set_last_error("xq_batch_decode_timed: " + err);
        return err.find("prefilled") != std::string::npos ? XQ_ERR_NOT_READY : XQ_ERR_RUNTIME;
    }
    return XQ_OK;
}

XQ_API xq_status xq_batch_hidden_state(xq_batch* b, int seq, float* out, size_t cap, size_t* out_size) {
    if (!b) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!b->m.hidden(seq, out, cap, out_size, &err)) {
        xqb::set_last_error("xq_batch_hidden_state: " + err);
        return err == "buffer too small" ? XQ_ERR_BUFFER_TOO_SMALL : XQ_ERR_INVALID_ARGUMENT;
    }
    return XQ_OK;
}

}  // extern "C"
