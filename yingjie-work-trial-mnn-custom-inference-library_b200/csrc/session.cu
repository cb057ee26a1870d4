// Session state machine and the public C ABI (xqwen35.h). Mirrors the reference Session
// (customlib/runtime/session.{hpp,cpp}): same status codes, metric definitions, error
// strings and JSON getter contracts, with the model running on the GPU.
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/xqwen35.h"
#include "model.hpp"

namespace xqb {
namespace {

using Clock = std::chrono::steady_clock;

double elapsed_ms(Clock::time_point a, Clock::time_point b) {
    return std::chrono::duration<double, std::milli>(b - a).count();
}

void copy_string(char* dst, size_t cap, const std::string& src) {
    if (cap == 0) return;
    const size_t n = std::min(cap - 1, src.size());
    std::memcpy(dst, src.data(), n);
    dst[n] = '\0';
}

std::string json_escape(const std::string& v) {
    std::ostringstream o;
    for (char c : v) {
        switch (c) {
            case '\\': o << "\\\\"; break;
            case '"': o << "\\\""; break;
            case '\n': o << "\\n"; break;
            case '\r': o << "\\r"; break;
            case '\t': o << "\\t"; break;
            default: o << c;
        }
    }
    return o.str();
}

// KernelTrace schema of the reference (custom_model.cpp:374-417): rows keyed by name with
// op_family, backend, calls, total/mean/min/max ms. Ops fused inside a CUDA graph are
// counted per execution; their time is carried by the step row of the graph they ran in.
struct TraceStat {
    uint64_t calls = 0;
    double total = 0.0, mn = 0.0, mx = 0.0;
    std::string backend;
};

std::string op_family(const std::string& n) {  // traceOpFamily, custom_model.cpp:116-179
    struct Rule {
        const char* key;
        const char* family;
    };
    static const Rule rules[] = {
        {"linear_q_proj", "q_proj"}, {"linear_k_proj", "k_proj"}, {"linear_v_proj", "v_proj"},
        {"linear_o_proj", "o_proj"}, {"linear_gate_proj", "gate_proj"}, {"linear_up_proj", "up_proj"},
        {"linear_down_proj", "down_proj"}, {"linear_attn", "linear_attention_projection"},
        {"linear_attention_state", "linear_attention_state"}, {"linear_attention_conv", "linear_attention_state"},
        {"linear_attention_qk", "linear_attention_state"}, {"linear_attention_gated", "linear_attention_state"},
        {"rmsnorm", "rmsnorm"}, {"rope", "rope"}, {"attention_score", "attention_score"},
        {"attention_softmax", "attention_softmax"}, {"attention_v_reduce", "attention_v_reduce"},
        {"attention", "attention"}, {"lm_head", "lm_head"}, {"sampling", "sampling"},
        {"prefill_kv_build", "prefill_kv_build"}, {"kv_append", "prefill_kv_build"},
        {"kv_cache", "prefill_kv_build"}, {"embedding_load", "prefill_kv_build"}, {"silu", "activation"}};
    for (const Rule& r : rules)
        if (n.find(r.key) != std::string::npos) return r.family;
    return "other";
}

class Trace {
public:
    void add(const std::string& name, uint64_t calls, double ms, const std::string& backend) {
        TraceStat& s = rows_[name];
        const double per = calls ? ms / static_cast<double>(calls) : 0.0;
        if (s.calls == 0) {
            s.mn = per;
            s.mx = per;
            s.backend = backend;
        } else {
            s.mn = std::min(s.mn, per);
            s.mx = std::max(s.mx, per);
            if (s.backend != backend) s.backend = "mixed";
        }
        s.calls += calls;
        s.total += ms;
    }
    void reset() { rows_.clear(); }
    std::string json() const {
        std::ostringstream o;
        o << "{\"rows\":[";
        bool first = true;
        for (const auto& kv : rows_) {
            if (!first) o << ",";
            first = false;
            const TraceStat& s = kv.second;
            o << "{\"name\":\"" << json_escape(kv.first) << "\",\"op_family\":\"" << op_family(kv.first)
              << "\",\"backend\":\"" << json_escape(s.backend) << "\",\"calls\":" << s.calls
              << ",\"total_ms\":" << s.total << ",\"mean_ms\":" << (s.calls ? s.total / s.calls : 0.0)
              << ",\"min_ms\":" << s.mn << ",\"max_ms\":" << s.mx << "}";
        }
        o << "]}";
        return o.str();
    }

private:
    std::map<std::string, TraceStat> rows_;
};

struct RuntimeOptions {  // normalizeOptions, session.cpp:152-178
    std::string backend = "cpu";
    int threads = 4;
    int quant_bits = 4;
    int group_size = 64;
    int max_context_tokens = 8192;
    bool enable_autotune = true;
    bool use_mnn_fallback = true;
    std::string telemetry_path;
};

RuntimeOptions normalize(const xq_options* o) {
    RuntimeOptions r;
    if (!o) return r;
    if (o->backend && o->backend[0]) r.backend = o->backend;
    if (o->threads > 0) r.threads = o->threads;
    if (o->quant_bits == 2 || o->quant_bits == 3 || o->quant_bits == 4) r.quant_bits = o->quant_bits;
    if (o->group_size > 0) r.group_size = o->group_size;
    if (o->max_context_tokens > 0) r.max_context_tokens = o->max_context_tokens;
    r.enable_autotune = o->enable_autotune != 0;
    r.use_mnn_fallback = o->use_mnn_fallback != 0;
    if (o->telemetry_path) r.telemetry_path = o->telemetry_path;
    return r;
}

void copy_metrics(const xq_metrics& src, xq_metrics* dst) {  // copyMetrics, session.cpp:180-189
    if (!dst) return;
    const size_t want = dst->struct_size ? dst->struct_size : sizeof(xq_metrics);
    const size_t n = std::min(want, sizeof(xq_metrics));
    std::memset(dst, 0, n);
    std::memcpy(dst, &src, n);
    dst->struct_size = sizeof(xq_metrics);
}

class Session {
public:
    Session(std::string dir, RuntimeOptions o, Options cuda) : dir_(std::move(dir)), opts_(std::move(o)), cuda_(cuda) {
        metrics_.struct_size = sizeof(xq_metrics);
        copy_string(metrics_.backend, sizeof metrics_.backend, opts_.backend);
    }

    xq_status load() {
        const auto t0 = Clock::now();
        model_ = std::make_unique<DeviceModel>();
        std::string err;
        cuda_.initial_capacity = std::max(64, opts_.max_context_tokens);
        if (!model_->load(dir_, cuda_, &err)) {
            set_error(err);
            // xq_create returns no metrics: keep the message for xqk_last_error on this thread too.
            set_last_error("xq_create: " + err);
            model_.reset();
            return XQ_ERR_MODEL;
        }
        loaded_ = true;
        metrics_.load_ms = elapsed_ms(t0, Clock::now());
        copy_string(metrics_.backend, sizeof metrics_.backend, "xq_custom_decode_cuda_sm100a");
        copy_string(metrics_.selected_kernels, sizeof metrics_.selected_kernels, coverage());
        copy_string(metrics_.error, sizeof metrics_.error, "");
        return XQ_OK;
    }

    xq_status prefill(const int32_t* ids, size_t n, xq_metrics* out) {  // session.cpp:304-342
        if (!loaded_) {
            set_error("session is not loaded");
            copy_metrics(metrics_, out);
            return XQ_ERR_NOT_READY;
        }
        if (!ids || n == 0) {
            set_error("prefill requires at least one token");
            copy_metrics(metrics_, out);
            return XQ_ERR_INVALID_ARGUMENT;
        }
        const auto t0 = Clock::now();
        position_ = n;
        std::string err;
        bool done = false;
        if (cuda_.prefill_batched && model_->batched_prefill_eligible(n)) {
            bool unsupported = false;
            done = model_->prefill_batched(ids, n, &err, &unsupported);
            if (!done && !unsupported) {
                set_error(err);
                copy_metrics(metrics_, out);
                return XQ_ERR_RUNTIME;
            }
        }
        if (!done && !model_->prefill(ids, n, &err)) {
            set_error(err);
            copy_metrics(metrics_, out);
            return XQ_ERR_MODEL;
        }
        has_prefill_ = true;
        const double ms = elapsed_ms(t0, Clock::now());
        trace_prefill(n, ms);
        metrics_.prompt_tokens = n;
        metrics_.generated_tokens = 0;
        metrics_.prefill_ms = ms;
        metrics_.first_token_ms = 0.0;
        metrics_.decode_total_ms = 0.0;
        metrics_.total_generate_ms = ms;
        update_rates();
        copy_string(metrics_.selected_kernels, sizeof metrics_.selected_kernels, coverage());
        copy_string(metrics_.error, sizeof metrics_.error, "");
        copy_metrics(metrics_, out);
        return XQ_OK;
    }

    xq_status decode_one(int32_t* token, xq_metrics* out) {  // session.cpp:344-383
        if (!loaded_ || !has_prefill_) {
            set_error("decode requires a loaded session and completed prefill");
            copy_metrics(metrics_, out);
            return XQ_ERR_NOT_READY;
        }
        if (!token) {
            set_error("decode output pointer is null");
            copy_metrics(metrics_, out);
            return XQ_ERR_INVALID_ARGUMENT;
        }
        const auto t0 = Clock::now();
        std::string err;
        int32_t t = 0;
        if (!model_->decode_one(&t, &err)) {
            set_error(err);
            copy_metrics(metrics_, out);
            return XQ_ERR_RUNTIME;
        }
        ++position_;
        *token = t;
        const double ms = elapsed_ms(t0, Clock::now());
        trace_decode(1, ms);
        if (metrics_.generated_tokens == 0) metrics_.first_token_ms = ms;
        metrics_.generated_tokens += 1;
        metrics_.decode_total_ms += ms;
        metrics_.total_generate_ms = metrics_.prefill_ms + metrics_.decode_total_ms;
        update_rates();
        copy_string(metrics_.error, sizeof metrics_.error, "");
        copy_metrics(metrics_, out);
        return XQ_OK;
    }

    // session.cpp:385-421. The first token is returned synchronously (first_token_ms); the
    // remaining steps are enqueued back to back and their tokens read once at the end.
    xq_status generate(const int32_t* ids, size_t n, size_t max_new, int32_t* out_buf, size_t cap,
                       xq_metrics* out) {
        if (!out_buf || cap < max_new) {
            set_error("output buffer is too small");
            copy_metrics(metrics_, out);
            return XQ_ERR_BUFFER_TOO_SMALL;
        }
        const auto t0 = Clock::now();
        xq_status st = prefill(ids, n, nullptr);
        if (st != XQ_OK) {
            copy_metrics(metrics_, out);
            return st;
        }
        if (max_new > 0) {
            st = decode_one(&out_buf[0], nullptr);
            if (st != XQ_OK) {
                copy_metrics(metrics_, out);
                return st;
            }
        }
        size_t done = 1;
        while (done < max_new) {
            const size_t batch = std::min<size_t>(max_new - done, 4096);
            const auto t1 = Clock::now();
            std::string err;
            const size_t first = ring_first();
            if (!model_->decode_many(batch, &err) || !model_->read_ring(first, batch, out_buf + done, &err)) {
                set_error(err);
                copy_metrics(metrics_, out);
                return XQ_ERR_RUNTIME;
            }
            const double ms = elapsed_ms(t1, Clock::now());
            trace_decode(batch, ms);
            position_ += batch;
            metrics_.generated_tokens += batch;
            metrics_.decode_total_ms += ms;
            done += batch;
        }
        metrics_.total_generate_ms = elapsed_ms(t0, Clock::now());
        update_rates();
        copy_string(metrics_.selected_kernels, sizeof metrics_.selected_kernels, coverage());
        copy_metrics(metrics_, out);
        return XQ_OK;
    }

    xq_status decode_timed(size_t n, int32_t* tokens, double* device_ms) {
        if (!loaded_ || !has_prefill_) {
            set_error("decode requires a loaded session and completed prefill");
            return XQ_ERR_NOT_READY;
        }
        if (!device_ms) return XQ_ERR_INVALID_ARGUMENT;
        std::string err;
        const size_t first = ring_first();
        const auto t0 = Clock::now();
        if (!model_->decode_many_timed(n, device_ms, &err) ||
            (tokens && n && !model_->read_ring(first, n, tokens, &err))) {
            set_error(err);
            return XQ_ERR_RUNTIME;
        }
        const double ms = elapsed_ms(t0, Clock::now());
        trace_decode(n, ms);
        position_ += n;
        if (metrics_.generated_tokens == 0 && n) metrics_.first_token_ms = ms / static_cast<double>(n);
        metrics_.generated_tokens += n;
        metrics_.decode_total_ms += ms;
        metrics_.total_generate_ms = metrics_.prefill_ms + metrics_.decode_total_ms;
        update_rates();
        return XQ_OK;
    }

    xq_status snapshot_size(size_t* bytes) {
        if (!loaded_ || !has_prefill_) {
            set_error("snapshot requires a loaded session and completed prefill");
            return XQ_ERR_NOT_READY;
        }
        *bytes = model_->snapshot_bytes();
        return XQ_OK;
    }
    xq_status snapshot_save(void* buf, size_t cap, size_t* written) {
        if (!loaded_ || !has_prefill_) {
            set_error("snapshot requires a loaded session and completed prefill");
            return XQ_ERR_NOT_READY;
        }
        const size_t need = model_->snapshot_bytes();
        if (written) *written = need;
        if (!buf || cap < need) {
            set_error("snapshot buffer too small");
            return XQ_ERR_BUFFER_TOO_SMALL;
        }
        std::string err;
        if (!model_->save_snapshot(buf, cap, written, &err)) {
            set_error(err);
            return XQ_ERR_RUNTIME;
        }
        return XQ_OK;
    }
    xq_status snapshot_restore(const void* buf, size_t size) {
        if (!loaded_) {
            set_error("session is not loaded");
            return XQ_ERR_NOT_READY;
        }
        std::string err;
        bool invalid = false;
        if (!model_->restore_snapshot(buf, size, &err, &invalid)) {
            set_error(err);
            return invalid ? XQ_ERR_INVALID_ARGUMENT : XQ_ERR_RUNTIME;
        }
        position_ = static_cast<size_t>(model_->position());
        has_prefill_ = position_ > 0;
        return XQ_OK;
    }

    xq_status reset() {  // session.cpp:505-525
        has_prefill_ = false;
        position_ = 0;
        metrics_ = {};
        metrics_.struct_size = sizeof(xq_metrics);
        trace_.reset();
        if (model_) {
            std::string err;
            if (!model_->reset(&err)) {
                set_error(err);
                return XQ_ERR_RUNTIME;
            }
        }
        copy_string(metrics_.backend, sizeof metrics_.backend, opts_.backend);
        copy_string(metrics_.selected_kernels, sizeof metrics_.selected_kernels, coverage());
        return XQ_OK;
    }

    xq_status last_metrics(xq_metrics* out) const {
        copy_metrics(metrics_, out);
        return XQ_OK;
    }

    xq_status backend_info(char* buf, size_t cap) const {
        if (!buf || cap == 0) return XQ_ERR_INVALID_ARGUMENT;
        cudaDeviceProp prop = {};
        cudaGetDeviceProperties(&prop, cuda_.device);
        std::ostringstream o;
        o << "{\"backend\":\"" << json_escape(opts_.backend) << "\",\"engine\":\"xqwen35_b200\",\"device\":\""
          << json_escape(prop.name) << "\",\"device_ordinal\":" << cuda_.device << ",\"sm\":\"sm_"
          << prop.major << prop.minor << "a\",\"kv_dtype\":\"" << (cuda_.kv_fp16 ? "f16" : "f32")
          << "\",\"cuda_graphs\":" << (cuda_.use_graphs ? "true" : "false")
          << ",\"quant_bits\":" << opts_.quant_bits << ",\"group_size\":" << opts_.group_size
          << ",\"threads\":" << opts_.threads;
        if (model_)
          o << ",\"weight_bytes\":" << model_->weight_bytes() << ",\"device_bytes\":" << model_->device_bytes()
            << ",\"kv_capacity\":" << model_->capacity()
            << ",\"kernels_per_decode_step\":" << model_->kernels_per_decode_step()
            << ",\"persistent_step_kernel\":" << (model_->persistent() ? "true" : "false")
            << ",\"packed_layout\":" << (model_->packed_layout() ? "true" : "false")
            << ",\"tensor_core_gemv\":" << (model_->tensor_core_step() ? "true" : "false")
            << ",\"step_kernel_binary_version\":" << step_kernel_binary_version()
            << ",\"weights_reused\":" << (model_->weights_reused() ? "true" : "false")
            << ",\"weights_users\":" << model_->weights_users();
        if (model_ && !model_->phase_trace_summary().empty())
            o << ",\"step_phase_trace\":" << model_->phase_trace_summary();
        o << ",\"selected_kernels\":\"" << json_escape(coverage()) << "\"}";
        return copy_json(o.str(), buf, cap);
    }

    xq_status trace_json(char* buf, size_t cap) const {
        if (!buf || cap == 0) return XQ_ERR_INVALID_ARGUMENT;
        if (!model_ || !model_->persistent() || model_->phase_times().empty()) return copy_json(trace_.json(), buf, cap);
        // With the step-kernel phase trace on (XQ_STEP_TRACE), add one row per phase kind with
        // its measured device time, named so the reference's op_family rules classify it.
        Trace t = trace_;
        static const std::map<std::string, std::string> rows = {
            {"lm_head_argmax", "lm_head_argmax_step_phase"},
            {"gemv_in_proj_conv", "linear_attn_in_proj_conv_step_phase"},
            {"delta", "linear_attention_state_step_phase"},
            {"gemv_out_proj", "linear_attn_out_proj_gated_rms_step_phase"},
            {"gemv_qkv", "linear_q_proj_k_v_step_phase"},
            {"attention", "attention_decode_step_phase"},
            {"gemv_o_proj", "linear_o_proj_step_phase"},
            {"gemv_gate_up", "linear_gate_proj_up_proj_swiglu_step_phase"},
            {"gemv_down", "linear_down_proj_step_phase"},
            {"embed", "embedding_load_step_phase"}};
        for (const auto& pt : model_->phase_times()) {
            const auto it = rows.find(pt.name);
            const std::string name = it != rows.end() ? it->second : pt.name + "_step_phase";
            t.add(name, static_cast<uint64_t>(pt.per_step) * pt.steps, pt.us_per_step * pt.steps / 1000.0,
                  "cuda_persistent_kernel");
        }
        return copy_json(t.json(), buf, cap);
    }

    // debugJson (custom_model.cpp:1382-1436): hidden statistics + top-10 lm_head logits.
    xq_status debug_json(char* buf, size_t cap) const {
        if (!buf || cap == 0) return XQ_ERR_INVALID_ARGUMENT;
        if (!model_) return copy_json("{\"debug\":\"unavailable\"}", buf, cap);
        std::vector<float> h, logits;
        std::string err;
        if (!model_->hidden(&h, &err) || !model_->logits(&logits, &err)) return XQ_ERR_RUNTIME;
        double sum = 0.0, sq = 0.0;
        float mn = h.empty() ? 0.0f : h[0], mx = mn;
        int nonfinite = 0;
        for (float v : h) {
            if (!std::isfinite(v)) {
                ++nonfinite;
                continue;
            }
            sum += v;
            sq += static_cast<double>(v) * v;
            mn = std::min(mn, v);
            mx = std::max(mx, v);
        }
        const double n = static_cast<double>(h.size());
        const double mean = n > 0 ? sum / n : 0.0;
        const double var = n > 0 ? std::max(0.0, sq / n - mean * mean) : 0.0;
        std::vector<int> best;
        for (int i = 0; i < static_cast<int>(logits.size()); ++i) {
            const float v = logits[static_cast<size_t>(i)];
            size_t pos = 0;
            while (pos < best.size() && logits[static_cast<size_t>(best[pos])] >= v) ++pos;
            if (pos < 10) {
                best.insert(best.begin() + static_cast<std::ptrdiff_t>(pos), i);
                if (best.size() > 10) best.pop_back();
            }
        }
        std::ostringstream o;
        o << "{\"hidden\":{\"size\":" << h.size() << ",\"mean\":" << mean << ",\"std\":" << std::sqrt(var)
          << ",\"min\":" << mn << ",\"max\":" << mx << ",\"l2\":" << std::sqrt(sq) << ",\"nonfinite\":" << nonfinite
          << "},\"lm_head_topk\":[";
        for (size_t i = 0; i < best.size(); ++i) {
            if (i) o << ",";
            o << "{\"token\":" << best[i] << ",\"logit\":" << logits[static_cast<size_t>(best[i])] << "}";
        }
        o << "]}";
        return copy_json(o.str(), buf, cap);
    }

    xq_status hidden_state(float* out, size_t cap, size_t* out_size) const {  // session.cpp:701-706
        if (!model_) return XQ_ERR_NOT_READY;
        std::vector<float> h;
        std::string err;
        if (!model_->hidden(&h, &err)) return XQ_ERR_RUNTIME;
        if (out_size) *out_size = h.size();
        if (!out || cap < h.size()) return XQ_ERR_BUFFER_TOO_SMALL;
        std::memcpy(out, h.data(), h.size() * sizeof(float));
        return XQ_OK;
    }

private:
    static xq_status copy_json(const std::string& s, char* buf, size_t cap) {
        if (s.size() + 1 > cap) return XQ_ERR_BUFFER_TOO_SMALL;
        std::memcpy(buf, s.c_str(), s.size() + 1);
        return XQ_OK;
    }
    void set_error(const std::string& m) { copy_string(metrics_.error, sizeof metrics_.error, m); }
    // The reference declares rss_kb / pss_kb and leaves them 0; here rss_kb is the host
    // process's resident set (VmRSS) and pss_kb the device memory this session holds.
    void update_memory() {
        std::ifstream f("/proc/self/status");
        std::string line;
        while (std::getline(f, line))
            if (line.rfind("VmRSS:", 0) == 0) metrics_.rss_kb = std::strtoull(line.c_str() + 6, nullptr, 10);
        if (model_) metrics_.pss_kb = model_->device_bytes() / 1024;
    }
    void update_rates() {  // session.cpp:595-602
        update_memory();
        metrics_.prefill_tokens_per_second =
            metrics_.prefill_ms > 0.0 ? static_cast<double>(metrics_.prompt_tokens) * 1000.0 / metrics_.prefill_ms : 0.0;
        metrics_.decode_tokens_per_second =
            metrics_.decode_total_ms > 0.0
                ? static_cast<double>(metrics_.generated_tokens) * 1000.0 / metrics_.decode_total_ms
                : 0.0;
    }
    size_t ring_first() const { return static_cast<size_t>(metrics_.generated_tokens); }
    std::string coverage() const {
        std::ostringstream o;
        o << "custom_decode_loop;hotpath_replaced=true;full_custom_decode=true;backend_request=" << opts_.backend
          << ";device=cuda_sm100a;linear=w4a16_g64_gemv_dp4a_bulkcopy_fused;lm_head=gemv_fused_argmax;"
          << "rmsnorm=fused_gemv_prologue;rope=fused_attention;attention=split_k_flash_decode_"
          << (cuda_.kv_fp16 ? "kv_f16" : "kv_f32") << ";linear_attention_state=gated_delta_column_split;"
          << "linear_attention_conv=fused_gemv_epilogue;sampling=device_greedy_argmax;"
          << "prefill_kv_build=token_serial;step=" << (model_ && model_->persistent() ? "persistent_kernel" : "cuda_graph")
          << ";fallback_ops=none";
        return o.str();
    }
    void trace_step_ops(uint64_t steps, bool decode) {
        if (!model_) return;
        const std::string b = step_backend();
        int full = 0, lin = 0;
        for (const DevLayer& L : model_->layers()) (L.full ? full : lin) += 1;
        if (decode) {
            trace_.add("lm_head_custom", steps, 0.0, b);
            trace_.add("sampling_greedy_custom", steps, 0.0, b);
        }
        trace_.add("embedding_bf16_row_read", steps, 0.0, b);
        trace_.add("rmsnorm_input", steps * (full + lin), 0.0, b);
        trace_.add("rmsnorm_post_attention", steps * (full + lin), 0.0, b);
        trace_.add("linear_gate_proj_w4a16", steps * (full + lin), 0.0, b);
        trace_.add("linear_up_proj_w4a16", steps * (full + lin), 0.0, b);
        trace_.add("silu_gate_mul_custom", steps * (full + lin), 0.0, b);
        trace_.add("linear_down_proj_w4a16", steps * (full + lin), 0.0, b);
        if (lin) {
            trace_.add("linear_attn_in_proj_qkv_w4a16", steps * lin, 0.0, b);
            trace_.add("linear_attention_conv1d_custom", steps * lin, 0.0, b);
            trace_.add("linear_attention_qk_l2norm_custom", steps * lin, 0.0, b);
            trace_.add("linear_attention_state_update_custom", steps * lin, 0.0, b);
            trace_.add("linear_attention_gated_rmsnorm_custom", steps * lin, 0.0, b);
            trace_.add("linear_attn_out_proj_w4a16", steps * lin, 0.0, b);
        }
        if (full) {
            trace_.add("linear_q_proj_w4a16", steps * full, 0.0, b);
            trace_.add("linear_k_proj_w4a16", steps * full, 0.0, b);
            trace_.add("linear_v_proj_w4a16", steps * full, 0.0, b);
            trace_.add("rope_qk_custom", steps * full, 0.0, b);
            trace_.add("kv_append_custom", steps * full, 0.0, b);
            trace_.add("prefill_kv_build_custom", steps * full, 0.0, b);
            trace_.add("attention_score_custom", steps * full, 0.0, b);
            trace_.add("attention_softmax_custom", steps * full, 0.0, b);
            trace_.add("attention_v_reduce_custom", steps * full, 0.0, b);
            trace_.add("attention_output_gate_custom", steps * full, 0.0, b);
            trace_.add("linear_o_proj_w4a16", steps * full, 0.0, b);
        }
        trace_.add("rmsnorm_final", steps, 0.0, b);
    }
    std::string step_backend() const {
        if (model_ && model_->persistent()) return "cuda_persistent_kernel";
        return cuda_.use_graphs ? "cuda_graph" : "cuda";
    }
    void trace_prefill(uint64_t n, double ms) {
        trace_.add("prefill_token_custom", n, ms, step_backend());
        trace_step_ops(n, false);
    }
    void trace_decode(uint64_t n, double ms) {
        trace_.add("decode_step_custom", n, ms, step_backend());
        trace_step_ops(n, true);
    }

    std::string dir_;
    RuntimeOptions opts_;
    Options cuda_;
    std::unique_ptr<DeviceModel> model_;
    xq_metrics metrics_{};
    Trace trace_;
    bool loaded_ = false;
    bool has_prefill_ = false;
    size_t position_ = 0;
};

Options default_cuda_options() {
    Options o;
    const char* dev = std::getenv("XQ_CUDA_DEVICE");
    o.device = dev ? std::atoi(dev) : 0;
    const char* kv = std::getenv("XQ_KV_FP16");
    o.kv_fp16 = kv && std::atoi(kv) != 0;
    const char* gr = std::getenv("XQ_CUDA_GRAPHS");
    o.use_graphs = !(gr && std::atoi(gr) == 0);
    const char* pb = std::getenv("XQ_PREFILL_BATCHED");
    o.prefill_batched = pb && std::atoi(pb) != 0;
    return o;
}

}  // namespace
}  // namespace xqb

extern "C" {

xq_status xq_create_cuda(const char* model_dir, const xq_options* options, const xq_cuda_options* cuda_options,
                         xq_session** out_session) {
    if (!model_dir || !out_session) return XQ_ERR_INVALID_ARGUMENT;
    *out_session = nullptr;
    xqb::Options cuda = xqb::default_cuda_options();
    if (cuda_options) {
        const size_t n = cuda_options->struct_size;
        if (n >= offsetof(xq_cuda_options, device) + sizeof(int) && cuda_options->device >= 0)
            cuda.device = cuda_options->device;
        if (n >= offsetof(xq_cuda_options, kv_fp16) + sizeof(int)) cuda.kv_fp16 = cuda_options->kv_fp16 != 0;
        if (n >= offsetof(xq_cuda_options, use_graphs) + sizeof(int)) cuda.use_graphs = cuda_options->use_graphs != 0;
        if (n >= offsetof(xq_cuda_options, prefill_batched) + sizeof(int) && cuda_options->prefill_batched >= 0)
            cuda.prefill_batched = cuda_options->prefill_batched != 0;
    }
    auto s = std::make_unique<xqb::Session>(model_dir, xqb::normalize(options), cuda);
    const xq_status st = s->load();
    if (st != XQ_OK) return st;
    *out_session = reinterpret_cast<xq_session*>(s.release());
    return XQ_OK;
}

xq_status xq_create(const char* model_dir, const xq_options* options, xq_session** out_session) {
    return xq_create_cuda(model_dir, options, nullptr, out_session);
}

void xq_destroy(xq_session* session) { delete reinterpret_cast<xqb::Session*>(session); }

#define XQ_SESSION(s) reinterpret_cast<xqb::Session*>(s)

xq_status xq_prefill(xq_session* s, const int32_t* ids, size_t n, xq_metrics* m) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->prefill(ids, n, m);
}
xq_status xq_decode_one(xq_session* s, int32_t* t, xq_metrics* m) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->decode_one(t, m);
}
xq_status xq_generate(xq_session* s, const int32_t* ids, size_t n, size_t max_new, int32_t* out, size_t cap,
                      xq_metrics* m) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->generate(ids, n, max_new, out, cap, m);
}
xq_status xq_reset(xq_session* s) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->reset();
}
xq_status xq_get_last_metrics(xq_session* s, xq_metrics* m) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->last_metrics(m);
}
xq_status xq_get_backend_info(xq_session* s, char* b, size_t c) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->backend_info(b, c);
}
xq_status xq_get_kernel_trace_json(xq_session* s, char* b, size_t c) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->trace_json(b, c);
}
xq_status xq_get_debug_json(xq_session* s, char* b, size_t c) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->debug_json(b, c);
}
xq_status xq_get_hidden_state(xq_session* s, float* v, size_t cap, size_t* out_size) {
    if (!s || !out_size) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->hidden_state(v, cap, out_size);
}

xq_status xq_cuda_decode_timed(xq_session* s, size_t n, int32_t* tokens, double* device_ms) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->decode_timed(n, tokens, device_ms);
}

xq_status xq_pack_b200_layout(const char* model_dir, char* error_out, size_t error_capacity) {
    if (error_out && error_capacity) error_out[0] = '\0';
    if (!model_dir || !model_dir[0]) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!xqb::pack_b200_layout(model_dir, &err)) {
        if (error_out && error_capacity) xqb::copy_string(error_out, error_capacity, err);
        return XQ_ERR_MODEL;
    }
    return XQ_OK;
}

xq_status xq_snapshot_size(xq_session* s, size_t* bytes) {
    if (!s || !bytes) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->snapshot_size(bytes);
}
xq_status xq_snapshot_save(xq_session* s, void* buffer, size_t capacity, size_t* written) {
    if (!s) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->snapshot_save(buffer, capacity, written);
}
xq_status xq_snapshot_restore(xq_session* s, const void* buffer, size_t size) {
    if (!s || !buffer) return XQ_ERR_INVALID_ARGUMENT;
    return XQ_SESSION(s)->snapshot_restore(buffer, size);
}

// runVulkanW4A16SelfTestJson on a host without Vulkan (vulkan_backend.cpp:1638-1656).
xq_status xq_run_vulkan_w4a16_selftest(char* json_out, size_t json_capacity) {
    const std::string j =
        "{\"engine\":\"customlib\",\"test\":\"vulkan_w4a16_gemv_correctness\",\"custom_backend_requested\":\"vulkan\","
        "\"custom_backend_actual\":\"unavailable\",\"vulkan_runtime_initialized\":false,"
        "\"vulkan_compute_queue_found\":false,\"vulkan_generation_kernels_used\":false,\"vulkan_device_name\":\"\","
        "\"status\":\"error\",\"pass\":false,\"error\":\"Vulkan is not part of the CUDA build\"}";
    if (json_out && json_capacity) xqb::copy_string(json_out, json_capacity, j);
    return XQ_ERR_RUNTIME;
}

}  // extern "C"
