// DeviceModel: loads a reference-format package onto one B200, keeps weights, KV cache and
// recurrent state resident, and runs each token step as one CUDA graph whose kernels are
// chained with programmatic dependent launch.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cerrno>
#include <sys/stat.h>
#include <array>
#include <map>
#include <climits>
#include <memory>
#include <mutex>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

#include "model.hpp"
#include "prefill_gemm.hpp"
#include "prefill_ops.hpp"
#include "generic.hpp"
#include "mma_gemv.hpp"
#include "ops.cuh"

namespace xqb {

std::string read_small_file(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) return {};
    std::ostringstream oss;
    oss << in.rdbuf();
    return oss.str();
}

bool file_exists(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    return in.good();
}

namespace {

// findJsonInt / findJsonFloat (custom_model.cpp:38-87): first occurrence of "key", then the
// first character of "-0123456789" after the next ':'.
size_t json_value_pos(const std::string& json, const std::string& key) {
    const std::string needle = "\"" + key + "\"";
    const size_t pos = json.find(needle);
    if (pos == std::string::npos) return std::string::npos;
    const size_t colon = json.find(':', pos + needle.size());
    if (colon == std::string::npos) return std::string::npos;
    return json.find_first_of("-0123456789", colon + 1);
}

int json_int(const std::string& json, const std::string& key, int fallback) {
    const size_t first = json_value_pos(json, key);
    if (first == std::string::npos) return fallback;
    size_t last = first + 1;
    while (last < json.size() && json[last] >= '0' && json[last] <= '9') ++last;
    try {
        return std::stoi(json.substr(first, last - first));
    } catch (...) {
        return fallback;
    }
}

float json_float(const std::string& json, const std::string& key, float fallback) {
    const size_t first = json_value_pos(json, key);
    if (first == std::string::npos) return fallback;
    size_t last = first + 1;
    while (last < json.size() && (std::isdigit(static_cast<unsigned char>(json[last])) || json[last] == '.' ||
                                  json[last] == 'e' || json[last] == 'E' || json[last] == '-' || json[last] == '+'))
        ++last;
    try {
        return std::stof(json.substr(first, last - first));
    } catch (...) {
        return fallback;
    }
}

}  // namespace

bool read_vec(const std::string& path, int expected, std::vector<float>* out, std::string* error) {
    std::ifstream in(path, std::ios::binary);
    if (!in) {
        *error = "missing vector file: " + path;
        return false;
    }
    out->assign(static_cast<size_t>(expected), 0.0f);
    in.read(reinterpret_cast<char*>(out->data()), static_cast<std::streamsize>(out->size() * 4));
    if (in.gcount() != static_cast<std::streamsize>(out->size() * 4)) {
        *error = "short vector file: " + path;
        return false;
    }
    return true;
}

void add_one(std::vector<float>* v) {
    for (float& x : *v) x += 1.0f;
}

namespace {

std::string shape_str(const HostMatrix& m) { return std::to_string(m.rows) + "x" + std::to_string(m.cols); }

// Whether an XQ4 file's group size (header field 4) is `group` (false when unreadable).
bool package_group_is(const std::string& path, uint32_t group) {
    std::ifstream in(path, std::ios::binary);
    char head[28] = {};
    in.read(head, sizeof head);
    if (!in) return false;
    uint32_t g = 0;
    std::memcpy(&g, head + 20, 4);
    return g == group;
}

bool expect_shape(const HostMatrix& m, int rows, int cols, const std::string& name, std::string* error) {
    if (m.rows != rows || m.cols != cols) {
        *error = "unexpected shape for " + name + ": " + shape_str(m) + ", expected " + std::to_string(rows) + "x" +
                 std::to_string(cols);
        return false;
    }
    return true;
}

}  // namespace

ModelDims parse_manifest(const std::string& js, int* n_layers) {
    ModelDims d;  // defaults: custom_model.hpp:98-114
    d.hidden = json_int(js, "hidden_size", d.hidden);
    d.inter = json_int(js, "intermediate_size", d.inter);
    d.vocab = json_int(js, "vocab_size", d.vocab);
    d.heads = json_int(js, "num_attention_heads", d.heads);
    d.kv_heads = json_int(js, "num_key_value_heads", d.kv_heads);
    d.head_dim = json_int(js, "head_dim", d.head_dim);
    const float partial = json_float(js, "partial_rotary_factor", 0.25f);
    d.rotary_dim = std::max(2, static_cast<int>(std::round(static_cast<float>(d.head_dim) * partial)));
    if (d.rotary_dim & 1) --d.rotary_dim;  // custom_model.cpp:438-442
    d.lk_hd = json_int(js, "linear_key_head_dim", d.lk_hd);
    d.lv_hd = json_int(js, "linear_value_head_dim", d.lv_hd);
    d.lk_heads = json_int(js, "linear_num_key_heads", d.lk_heads);
    d.lv_heads = json_int(js, "linear_num_value_heads", d.lv_heads);
    d.conv_k = json_int(js, "linear_conv_kernel_dim", d.conv_k);
    d.lk_dim = d.lk_hd * d.lk_heads;
    d.lv_dim = d.lv_hd * d.lv_heads;
    d.conv_dim = 2 * d.lk_dim + d.lv_dim;
    d.eps = json_float(js, "rms_norm_eps", d.eps);
    d.theta = json_float(js, "rope_theta", d.theta);
    d.layers = json_int(js, "num_hidden_layers", 32);
    if (n_layers) *n_layers = d.layers;
    return d;
}

DeviceModel::~DeviceModel() {
    if (!stream_ && allocs_.empty()) return;  // (weights_ releases itself)
    cudaSetDevice(opts_.device);
    if (stream_) cudaStreamSynchronize(stream_);
    destroy_graphs();
    for (DevLayer& L : layers_) {  // matrices and weights belong to weights_
        cudaFree(L.k_cache);
        cudaFree(L.v_cache);
    }
    cudaFree(d_rope_);
    cudaFree(d_gscore_);
    cudaFree(d_phases_decode_);
    cudaFree(d_tmaps_);
    cudaFree(d_phases_prefill_);
    for (void* p : allocs_) cudaFree(p);
    if (h_token_) cudaFreeHost(h_token_);
    if (h_err_) cudaFreeHost(h_err_);
    if (stream_) cudaStreamDestroy(stream_);
}

template <typename T>
bool DeviceModel::dev_alloc(T** p, size_t count, std::string* error) {
    *p = nullptr;
    const size_t bytes = std::max<size_t>(1, count) * sizeof(T);
    const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes);
    if (e != cudaSuccess) {
        *error = std::string("device allocation failed: ") + cudaGetErrorString(e);
        return false;
    }
    allocs_.push_back(*p);
    device_bytes_ += bytes;
    if (cudaMemset(*p, 0, bytes) != cudaSuccess) {
        *error = "cudaMemset failed";
        return false;
    }
    return true;
}

bool DeviceModel::upload_vec(float** dst, const std::vector<float>& v, std::string* error) {
    if (!dev_alloc(dst, v.size(), error)) return false;
    if (cudaMemcpy(*dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        *error = "vector upload failed";
        return false;
    }
    return true;
}

namespace {
// One device matrix of the model: the XQ4 files it is fused from (row-wise, or gate/up pairs
// interleaved), their expected shapes, and where it lives. Shared by the loader and the packer
// so both read exactly the same files in the same order.
struct FusedSpec {
    std::string name;  // packed file name (b200/<name>.b200)
    std::vector<std::string> files;
    std::vector<std::pair<int, int>> shapes;  // (rows, cols) per file
    std::vector<std::string> labels;
    bool interleave = false;
    int layer = -1;  // -1: lm_head
    int slot = 0;    // 0 in_proj, 1 out_proj, 2 gate_up, 3 down
};

std::vector<FusedSpec> fused_specs(const std::string& dir, const ModelDims& d, int n_layers,
                                   std::vector<bool>* full) {
    std::vector<FusedSpec> out;
    out.push_back({"lm_head", {dir + "/lm_head_weight.xq4"}, {{d.vocab, d.hidden}}, {"lm_head"}, false, -1, 0});
    full->assign(static_cast<size_t>(n_layers), false);
    const int qd = d.heads * d.head_dim, kvd = d.kv_heads * d.head_dim;
    for (int i = 0; i < n_layers; ++i) {
        const std::string p = dir + "/layers_" + std::to_string(i) + "_";
        const std::string n = "layers_" + std::to_string(i) + "_";
        // custom_model.cpp:526: full attention iff the q_proj file exists.
        const bool f = file_exists(p + "self_attn_q_proj_weight.xq4");
        (*full)[static_cast<size_t>(i)] = f;
        if (f) {
            out.push_back({n + "in_proj",
                           {p + "self_attn_q_proj_weight.xq4", p + "self_attn_k_proj_weight.xq4",
                            p + "self_attn_v_proj_weight.xq4"},
                           {{2 * qd, d.hidden}, {kvd, d.hidden}, {kvd, d.hidden}},
                           {"self_attn_q_proj (gated)", "self_attn_k_proj", "self_attn_v_proj"}, false, i, 0});
            out.push_back({n + "out_proj", {p + "self_attn_o_proj_weight.xq4"}, {{d.hidden, qd}},
                           {"self_attn_o_proj"}, false, i, 1});
        } else {
            out.push_back({n + "in_proj",
                           {p + "linear_attn_in_proj_qkv_weight.xq4", p + "linear_attn_in_proj_z_weight.xq4",
                            p + "linear_attn_in_proj_a_weight.xq4", p + "linear_attn_in_proj_b_weight.xq4"},
                           {{d.conv_dim, d.hidden}, {d.lv_dim, d.hidden}, {d.lv_heads, d.hidden}, {d.lv_heads, d.hidden}},
                           {"linear_attn_in_proj_qkv", "linear_attn_in_proj_z", "linear_attn_in_proj_a",
                            "linear_attn_in_proj_b"},
                           false, i, 0});
            out.push_back({n + "out_proj", {p + "linear_attn_out_proj_weight.xq4"}, {{d.hidden, d.lv_dim}},
                           {"linear_attn_out_proj"}, false, i, 1});
        }
        out.push_back({n + "gate_up", {p + "mlp_gate_proj_weight.xq4", p + "mlp_up_proj_weight.xq4"},
                       {{d.inter, d.hidden}, {d.inter, d.hidden}}, {"mlp_gate_proj", "mlp_up_proj"}, true, i, 2});
        out.push_back({n + "down", {p + "mlp_down_proj_weight.xq4"}, {{d.hidden, d.inter}}, {"mlp_down_proj"}, false,
                       i, 3});
    }
    return out;
}

// Read a spec's XQ4 files, check their shapes and build the fused rows in host memory.
bool build_spec_rows(const FusedSpec& sp, DevMatrix* shape, std::vector<uint8_t>* host, std::string* error) {
    std::vector<HostMatrix> parts(sp.files.size());
    std::vector<const HostMatrix*> ptrs;
    for (size_t k = 0; k < sp.files.size(); ++k) {
        if (!read_xq4_file(sp.files[k], &parts[k], error) ||
            !expect_shape(parts[k], sp.shapes[k].first, sp.shapes[k].second, sp.labels[k], error))
            return false;
        if (parts[k].group != 64) {
            *error = "group size " + std::to_string(parts[k].group) + " not supported by the CUDA path";
            return false;
        }
        ptrs.push_back(&parts[k]);
    }
    return build_matrix_rows(ptrs, sp.interleave, shape, host, error);
}

const char* kB200LayoutFile = "/b200/layout.json";
}  // namespace

bool pack_b200_layout(const std::string& dir, std::string* error) {
    if (!file_exists(dir + "/xqwen35_manifest.json")) {
        *error = "missing xqwen35_manifest.json in " + dir;
        return false;
    }
    int n_layers = 0;
    const ModelDims d = parse_manifest(read_small_file(dir + "/xqwen35_manifest.json"), &n_layers);
    if (n_layers <= 0) {
        *error = "missing or empty xqwen35_manifest.json in " + dir;
        return false;
    }
    std::vector<bool> full;
    const std::vector<FusedSpec> specs = fused_specs(dir, d, n_layers, &full);
    const std::string out_dir = dir + "/b200";
    if (mkdir(out_dir.c_str(), 0755) != 0 && errno != EEXIST) {
        *error = "cannot create " + out_dir;
        return false;
    }
    std::remove((dir + kB200LayoutFile).c_str());  // an interrupted pack leaves no layout behind
    for (const FusedSpec& sp : specs) {
        DevMatrix shape;
        std::vector<uint8_t> host;
        if (!build_spec_rows(sp, &shape, &host, error) ||
            !write_b200_file(out_dir + "/" + sp.name + ".b200", shape, host, error))
            return false;
    }
    std::ofstream f(dir + kB200LayoutFile, std::ios::trunc);
    f << "{\"format\":\"xq_b200_rows\",\"version\":1,\"matrices\":" << specs.size()
      << ",\"source\":\"xq4\",\"note\":\"fused W4A16 rows in the sm_100a kernel layout; the loader uses "
         "them instead of re-tiling the xq4 files\"}\n";
    if (!f) {
        *error = "cannot write " + dir + kB200LayoutFile;
        return false;
    }
    return true;
}

// Read-only device weights of one package on one device, shared by every session that loads
// the same package there (the reference's sessions each hold a CustomModel; on the GPU the
// 4.2 GB of matrices, their tile copy and the 2 GB embedding table are loaded once per
// device): fused matrices (+ tensor-core tiles), norm and conv weights, gates, final norm,
// embeddings. Freed when the last session releases it.
struct SharedWeights {
    int device = 0;
    std::vector<DevLayer> layers;  // weight fields only; states stay null
    DevMatrix lm_head;
    float* final_norm = nullptr;
    uint16_t* emb = nullptr;
    bool packed_layout = false;
    size_t weight_bytes = 0, device_bytes = 0;
    std::vector<void*> allocs;

    bool alloc(void** p, size_t bytes, std::string* error) {
        *p = nullptr;
        if (cudaMalloc(p, std::max<size_t>(1, bytes)) != cudaSuccess) {
            *error = "device allocation failed for the shared weights";
            return false;
        }
        allocs.push_back(*p);
        device_bytes += bytes;
        return true;
    }
    bool upload(float** dst, const std::vector<float>& v, std::string* error) {
        if (!alloc(reinterpret_cast<void**>(dst), v.size() * 4, error)) return false;
        if (cudaMemcpy(*dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            *error = "vector upload failed";
            return false;
        }
        return true;
    }
    ~SharedWeights() {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        for (DevLayer& L : layers) {
            free_matrix(&L.in_proj);
            free_matrix(&L.out_proj);
            free_matrix(&L.gate_up);
            free_matrix(&L.down);
        }
        free_matrix(&lm_head);
        for (void* q : allocs) cudaFree(q);
        cudaSetDevice(prev);
    }
};

namespace {
// Registry of loaded weights, keyed by canonical dir | device | tiles. The global mutex guards
// the map only; each key has its own mutex, held while that package loads, so loading one
// package (seconds at 9B) does not hold up sessions of other packages or devices.
struct WeightsEntry {
    std::mutex mu;
    std::weak_ptr<SharedWeights> w;
};
std::mutex g_weights_mu;
std::map<std::string, std::shared_ptr<WeightsEntry>> g_weights;

std::shared_ptr<WeightsEntry> weights_entry(const std::string& key) {
    std::lock_guard<std::mutex> lock(g_weights_mu);
    for (auto it = g_weights.begin(); it != g_weights.end();) {  // drop released, idle entries
        if (it->first != key && it->second.use_count() == 1 && it->second->w.expired())
            it = g_weights.erase(it);
        else
            ++it;
    }
    std::shared_ptr<WeightsEntry>& e = g_weights[key];
    if (!e) e = std::make_shared<WeightsEntry>();
    return e;
}

bool load_shared_weights(const std::string& dir, const ModelDims& d, int n_layers, bool want_tiles, bool generic,
                         SharedWeights* w, std::string* error) {
    std::vector<float> v;
    if (!read_vec(dir + "/norm_weight.f32", d.hidden, &v, error)) return false;
    add_one(&v);
    if (!w->upload(&w->final_norm, v, error)) return false;
    // Weight matrices: the packed B200 layout (b200/*.b200, written by the packer) when present,
    // else the xq4 files re-tiled here. Either way every matrix is checked against the
    // manifest's shapes.
    w->layers.resize(static_cast<size_t>(n_layers));
    {
        std::vector<bool> full;
        const std::vector<FusedSpec> specs = fused_specs(dir, d, n_layers, &full);
        w->packed_layout = !generic && file_exists(dir + kB200LayoutFile);
        for (const FusedSpec& sp : specs) {
            DevMatrix shape;
            std::vector<uint8_t> host;
            if (generic) {
                // shapes the fused kernels do not take: each fused matrix in the layout its shape
                // allows (the reference's own arrays for the generic GEMV kernel)
                std::vector<HostMatrix> parts(sp.files.size());
                std::vector<const HostMatrix*> ptrs;
                for (size_t k = 0; k < sp.files.size(); ++k) {
                    if (!read_xq4_file(sp.files[k], &parts[k], error) ||
                        !expect_shape(parts[k], sp.shapes[k].first, sp.shapes[k].second, sp.labels[k], error))
                        return false;
                    ptrs.push_back(&parts[k]);
                }
                DevMatrix* dst = &w->lm_head;
                if (sp.layer >= 0) {
                    DevLayer& L = w->layers[static_cast<size_t>(sp.layer)];
                    L.full = full[static_cast<size_t>(sp.layer)];
                    dst = sp.slot == 0 ? &L.in_proj : sp.slot == 1 ? &L.out_proj : sp.slot == 2 ? &L.gate_up : &L.down;
                }
                if (!upload_matrix(ptrs, sp.interleave, dst, error)) return false;
                w->weight_bytes += dst->bytes;
                w->device_bytes += dst->bytes;
                continue;
            }
            if (w->packed_layout) {
                if (!read_b200_file(dir + "/b200/" + sp.name + ".b200", &shape, &host, error)) return false;
                int rows = 0;
                for (const auto& sh : sp.shapes) rows += sh.first;
                if (shape.rows != rows || shape.cols != sp.shapes[0].second || shape.group != 64) {
                    *error = "packed B200 matrix " + sp.name + " does not match the manifest; re-run the packer";
                    return false;
                }
            } else if (!build_spec_rows(sp, &shape, &host, error)) {
                return false;
            }
            DevMatrix* dst = &w->lm_head;
            if (sp.layer >= 0) {
                DevLayer& L = w->layers[static_cast<size_t>(sp.layer)];
                L.full = full[static_cast<size_t>(sp.layer)];
                dst = sp.slot == 0 ? &L.in_proj : sp.slot == 1 ? &L.out_proj : sp.slot == 2 ? &L.gate_up : &L.down;
            }
            *dst = shape;
            if (!upload_matrix_rows(host, dst, error)) return false;
            w->weight_bytes += dst->bytes;
            w->device_bytes += dst->bytes;
            if (want_tiles && dst->kind == 0) {
                if (!attach_mma_tiles(host, dst, error)) return false;
                w->device_bytes += dst->tile_bytes;
            }
        }
    }
    for (int i = 0; i < n_layers; ++i) {
        DevLayer& L = w->layers[static_cast<size_t>(i)];
        const std::string p = dir + "/layers_" + std::to_string(i) + "_";
        if (!read_vec(p + "input_layernorm_weight.f32", d.hidden, &v, error)) return false;
        add_one(&v);
        if (!w->upload(&L.input_norm, v, error)) return false;
        if (!read_vec(p + "post_attention_layernorm_weight.f32", d.hidden, &v, error)) return false;
        add_one(&v);
        if (!w->upload(&L.post_norm, v, error)) return false;
        if (L.full) {  // set with the layer's matrices above
            if (!read_vec(p + "self_attn_q_norm_weight.f32", d.head_dim, &v, error)) return false;
            add_one(&v);
            if (!w->upload(&L.q_norm, v, error)) return false;
            if (!read_vec(p + "self_attn_k_norm_weight.f32", d.head_dim, &v, error)) return false;
            add_one(&v);
            if (!w->upload(&L.k_norm, v, error)) return false;
        } else {
            if (!read_vec(p + "linear_attn_norm_weight.f32", d.lv_hd, &v, error)) return false;
            if (!w->upload(&L.lin_norm, v, error)) return false;
            if (!read_vec(p + "linear_attn_conv1d_weight.f32", d.conv_dim * d.conv_k, &v, error)) return false;
            if (!w->upload(&L.conv_w, v, error)) return false;
            if (!read_vec(p + "linear_attn_A_log.f32", d.lv_heads, &v, error)) return false;
            if (!w->upload(&L.a_log, v, error)) return false;
            if (!read_vec(p + "linear_attn_dt_bias.f32", d.lv_heads, &v, error)) return false;
            if (!w->upload(&L.dt_bias, v, error)) return false;
        }
        for (const DevMatrix* m : {&L.in_proj, &L.out_proj, &L.gate_up, &L.down}) {
            if (!generic && !m->fast()) {
                *error = "layer " + std::to_string(i) + ": matrix shape not supported by the fused kernels";
                return false;
            }
        }
    }
    if (!generic && !w->lm_head.fast()) {
        *error = "lm_head shape not supported by the fused kernels";
        return false;
    }
    // Embedding table, resident in device memory (the reference reads one row from disk
    // per token, custom_model.cpp:569-608).
    {
        const size_t bytes = static_cast<size_t>(d.vocab) * d.hidden * 2;
        std::ifstream in(dir + "/embeddings_bf16.bin", std::ios::binary);
        if (!w->alloc(reinterpret_cast<void**>(&w->emb), bytes, error)) return false;
        const size_t chunk = 64u << 20;
        void* staging = nullptr;
        if (cudaMallocHost(&staging, chunk) != cudaSuccess) {
            *error = "pinned staging allocation failed";
            return false;
        }
        size_t done = 0;
        bool ok = true;
        while (done < bytes && ok) {
            const size_t n = std::min(chunk, bytes - done);
            in.read(static_cast<char*>(staging), static_cast<std::streamsize>(n));
            if (in.gcount() != static_cast<std::streamsize>(n)) {
                ok = false;
                break;
            }
            ok = cudaMemcpy(reinterpret_cast<uint8_t*>(w->emb) + done, staging, n, cudaMemcpyHostToDevice) ==
                 cudaSuccess;
            done += n;
        }
        cudaFreeHost(staging);
        if (!ok) {
            *error = "short embeddings_bf16.bin";
            return false;
        }
    }
    return true;
}
}  // namespace

bool DeviceModel::load(const std::string& dir, const Options& opts, std::string* error) {
    opts_ = opts;
    if (cudaSetDevice(opts.device) != cudaSuccess) {
        *error = "CUDA device " + std::to_string(opts.device) + " unavailable";
        return false;
    }
    cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, opts.device);
    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) {
        *error = "cudaStreamCreate failed";
        return false;
    }
    if (!gemv_init_device()) {
        *error = last_error();
        return false;
    }
    if (attention_init_device(200 * 1024) != cudaSuccess) {
        *error = "attention kernel setup failed";
        return false;
    }

    int n_layers = 0;
    d_ = parse_manifest(read_small_file(dir + "/xqwen35_manifest.json"), &n_layers);
    const ModelDims& d = d_;
    // Shapes the fused kernels are written for (all Qwen3.5-9B shapes satisfy them).
    if (n_layers <= 0 || d.hidden <= 0 || d.inter <= 0 || d.vocab <= 0 || d.heads <= 0 || d.kv_heads <= 0 ||
        d.head_dim <= 0 || d.lk_heads <= 0 || d.lv_heads <= 0 || d.lk_hd <= 0 || d.lv_hd <= 0 || d.conv_k < 1) {
        *error = "invalid model dimensions in the manifest";
        return false;
    }
    // Shapes the fused kernels are written for (all Qwen3.5-9B shapes satisfy them); other
    // shapes run the generic-shape step (generic.cu) on the GPU.
    generic_ = d.head_dim != 256 || d.rotary_dim != 64 || d.lk_hd != 128 || d.lv_hd % 32 != 0 || d.lv_hd > 1024 ||
               (d.lv_hd & (d.lv_hd - 1)) != 0 || d.heads % d.kv_heads != 0 || d.heads / d.kv_heads > kAttnMaxGroup ||
               d.lv_heads % d.lk_heads != 0 || !fast_shape(d.hidden, 64) || !fast_shape(d.inter, 64) ||
               !fast_shape(d.lv_dim, 64) || !fast_shape(d.heads * d.head_dim, 64) ||
               !package_group_is(dir + "/lm_head_weight.xq4", 64);
    if (generic_) opts_.kv_fp16 = false;  // the generic attention keeps an fp32 cache
    if (!file_exists(dir + "/embeddings_bf16.bin")) {
        *error = "missing embeddings_bf16.bin";
        return false;
    }
    // Tensor-core tiles for the step kernel (XQ_STEP_MMA=0 keeps the dp4a row loop): a second
    // copy of every symmetric matrix in 16-row tiles, built from the same host rows.
    const char* em = std::getenv("XQ_STEP_MMA");
    const char* ep = std::getenv("XQ_PERSISTENT");
    const bool want_tiles = !generic_ && opts.persistent && !(ep && std::atoi(ep) == 0) && !(em && std::atoi(em) == 0);
    {
        // Weights: shared with the other live sessions of this package on this device.
        char real[PATH_MAX];
        const std::string canon = realpath(dir.c_str(), real) ? std::string(real) : dir;
        const std::string key = canon + "|" + std::to_string(opts.device) + "|" +
                                (generic_ ? "generic" : want_tiles ? "tiles" : "rows");
        const std::shared_ptr<WeightsEntry> entry = weights_entry(key);
        std::lock_guard<std::mutex> lock(entry->mu);
        weights_ = entry->w.lock();
        weights_reused_ = weights_ != nullptr;
        if (!weights_) {
            auto w = std::make_shared<SharedWeights>();
            w->device = opts.device;
            if (!load_shared_weights(dir, d, n_layers, want_tiles, generic_, w.get(), error)) return false;
            entry->w = w;
            weights_ = w;
        }
    }
    layers_ = weights_->layers;
    lm_head_ = weights_->lm_head;
    d_final_norm_ = weights_->final_norm;
    d_emb_ = weights_->emb;
    packed_layout_ = weights_->packed_layout;
    weight_bytes_ = weights_->weight_bytes;
    device_bytes_ += weights_->device_bytes;
    for (DevLayer& L : layers_) {  // this session's DeltaNet states
        if (L.full) continue;
        if (!dev_alloc(&L.conv_state, static_cast<size_t>(d.conv_dim) * std::max(0, d.conv_k - 1), error) ||
            !dev_alloc(&L.rec_state, static_cast<size_t>(d.lv_heads) * d.lk_hd * d.lv_hd, error))
            return false;
    }
    const int qkv_rows = 2 * d.heads * d.head_dim + 2 * d.kv_heads * d.head_dim;
    const int group = d.heads / d.kv_heads;
    if (!dev_alloc(&d_hidden_, d.hidden, error) || !dev_alloc(&d_conv_out_, d.conv_dim, error) ||
        !dev_alloc(&d_zab_, d.lv_dim + 2 * d.lv_heads, error) || !dev_alloc(&d_attn_raw_, d.lv_dim, error) ||
        !dev_alloc(&d_qkv_, qkv_rows, error) || !dev_alloc(&d_attn_out_, d.heads * d.head_dim, error) ||
        !dev_alloc(&d_ffn_, d.inter, error) || !dev_alloc(&d_normed_, d.hidden, error) ||
        !dev_alloc(&d_logits_, d.vocab, error) || !dev_alloc(&d_pos_, 1, error) || !dev_alloc(&d_next_pos_, 1, error) ||
        !dev_alloc(&d_token_, 1, error) || !dev_alloc(&d_ring_, ring_cap_, error) ||
        !dev_alloc(&d_ring_ctr_, 1, error) || !dev_alloc(&d_arg_val_, num_sms_, error) ||
        !dev_alloc(&d_arg_idx_, num_sms_, error) || !dev_alloc(&d_arg_counter_, 1, error) ||
        !dev_alloc(&d_attn_part_, static_cast<size_t>(d.kv_heads) * kAttnSplits * group * (d.head_dim + 2), error) ||
        !dev_alloc(&d_attn_counters_, d.kv_heads, error) || !dev_alloc(&d_err_, 1, error) ||
        !dev_alloc(&d_head_ss_, static_cast<size_t>(d.lv_heads) * std::max(1, d.lv_hd / kDeltaCols), error))
        return false;
    if (generic_) {
        int ymax = d.hidden;
        for (const DevLayer& L : layers_) ymax = std::max({ymax, L.in_proj.rows, L.gate_up.rows, L.out_proj.rows});
        if (!dev_alloc(&d_gy_, static_cast<size_t>(ymax), error) ||
            !dev_alloc(&d_gqbuf_, static_cast<size_t>(d.heads + d.kv_heads) * d.head_dim, error))
            return false;
    }
    if (cudaMallocHost(&h_err_, sizeof(unsigned)) != cudaSuccess) {
        *error = "pinned allocation failed";
        return false;
    }
    if (cudaMallocHost(&h_token_, sizeof(int32_t)) != cudaSuccess) {
        *error = "pinned allocation failed";
        return false;
    }
    if (!alloc_kv(std::max(64, opts.initial_capacity), error)) return false;
    if (!dev_alloc(&d_grid_bar_, 1, error)) return false;
    {
        const char* e = std::getenv("XQ_PERSISTENT");
        const bool want = opts.persistent && !(e && std::atoi(e) == 0);
        meta_kind_ = lm_head_.kind;
        persistent_ = want && !generic_ && persistent_eligible(capacity_) && step_init_device() == cudaSuccess;
        bool tiles = lm_head_.d_tiles != nullptr;
        for (const DevLayer& L : layers_)
            tiles = tiles && L.in_proj.d_tiles && L.out_proj.d_tiles && L.gate_up.d_tiles && L.down.d_tiles;
        if (persistent_ && tiles) meta_kind_ = kMetaMma;
        if (persistent_) {
            step_slot_bytes_ = kStepSlotBytes;
            if (meta_kind_ == kMetaMma) {
                // pairs of groups per ring slot (XQ_STEP_MMA_PAIRS: 8..32, a multiple of 8)
                int pairs = kMmaStepSlotBytes / kMmaUnitBytes;
                if (const char* v = std::getenv("XQ_STEP_MMA_PAIRS")) pairs = std::max(8, std::min(32, std::atoi(v))) & ~7;
                step_slot_bytes_ = pairs * kMmaUnitBytes;
            }
            step_slots_ = step_max_slots(step_slot_bytes_);
            step_inflight_ = step_slots_;
            if (const char* v = std::getenv("XQ_STEP_INFLIGHT")) step_inflight_ = std::atoi(v);
            step_inflight_ = std::max(1, std::min(step_inflight_, step_slots_));
            if (const char* v = std::getenv("XQ_STEP_L2_PREFETCH")) step_l2_prefetch_ = std::atoi(v) != 0;
            // L2 prefetch of weight chunks ahead of the ring: row-layout path only (on the
            // tensor-core tiles' 35 KB chunks it measured 47 tok/s at 4 chunks ahead)
            if (const char* v = std::getenv("XQ_STEP_L2_AHEAD"))
                step_l2_ahead_ = meta_kind_ == kMetaMma ? 0 : std::max(0, std::min(64, std::atoi(v)));
            // XQ_STEP_WAIT_MS: limit of the step kernel's bounded waits (default 2000 ms).
            // XQ_TEST_STALL_LAUNCH=N (failure-detection tests only): the N-th step-kernel launch
            // of this session, counted from 0 at load, has a grid barrier that can never complete;
            // its wait runs out and the step reports XQ_ERR_RUNTIME.
            if (const char* v = std::getenv("XQ_STEP_WAIT_MS"))
                step_wait_ns_ = static_cast<unsigned long long>(std::max(1, std::min(60000, std::atoi(v)))) * 1000000ull;
            if (const char* v = std::getenv("XQ_TEST_STALL_LAUNCH")) stall_launch_ = std::atoll(v);
            if (!build_phases(error)) return false;
            const char* tr = std::getenv("XQ_STEP_TRACE");
            if (tr && std::atoi(tr) != 0 && !dev_alloc(&d_step_trace_, kStepTraceSlots * static_cast<size_t>(n_phases_), error))
                return false;
            if (tr && std::atoi(tr) >= 2 &&
                !dev_alloc(&d_block_done_, static_cast<size_t>(n_phases_) * num_sms_, error))
                return false;
        }
    }
    if (cudaDeviceSynchronize() != cudaSuccess) {
        *error = "device synchronisation after load failed";
        return false;
    }
    loaded_ = true;
    return true;
}

bool DeviceModel::alloc_kv(int capacity, std::string* error) {
    const size_t elem = opts_.kv_fp16 ? 2 : 4;
    const size_t per_pos = static_cast<size_t>(d_.kv_heads) * d_.head_dim * elem;
    for (DevLayer& L : layers_) {
        if (!L.full) continue;
        void *k = nullptr, *v = nullptr;
        if (cudaMalloc(&k, per_pos * capacity) != cudaSuccess || cudaMalloc(&v, per_pos * capacity) != cudaSuccess) {
            cudaFree(k);
            *error = "KV cache allocation failed for capacity " + std::to_string(capacity);
            return false;
        }
        cudaMemset(k, 0, per_pos * capacity);
        cudaMemset(v, 0, per_pos * capacity);
        if (L.k_cache) {  // keep positions already written
            const size_t keep = per_pos * std::min(capacity_, capacity);
            cudaMemcpyAsync(k, L.k_cache, keep, cudaMemcpyDeviceToDevice, stream_);
            cudaMemcpyAsync(v, L.v_cache, keep, cudaMemcpyDeviceToDevice, stream_);
            cudaStreamSynchronize(stream_);
            cudaFree(L.k_cache);
            cudaFree(L.v_cache);
            device_bytes_ -= 2 * per_pos * capacity_;
        }
        L.k_cache = k;
        L.v_cache = v;
        device_bytes_ += 2 * per_pos * capacity;
    }
    if (generic_) {  // the generic attention's score scratch [heads][capacity]
        float* sc = nullptr;
        if (cudaMalloc(&sc, sizeof(float) * static_cast<size_t>(d_.heads) * capacity) != cudaSuccess) {
            *error = "attention score scratch allocation failed";
            return false;
        }
        cudaFree(d_gscore_);
        d_gscore_ = sc;
    }
    // RoPE table for every position the cache can hold.
    std::vector<float2> rope;
    rope_table(0, capacity, d_.rotary_dim, d_.theta, &rope);
    if (d_rope_) cudaFree(d_rope_);
    d_rope_ = nullptr;
    if (cudaMalloc(&d_rope_, rope.size() * sizeof(float2)) != cudaSuccess ||
        cudaMemcpy(d_rope_, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess) {
        *error = "rope table upload failed";
        return false;
    }
    capacity_ = capacity;
    return true;
}

bool DeviceModel::ensure_capacity(int needed, std::string* error) {
    if (needed <= capacity_) return true;
    int cap = capacity_;
    while (cap < needed) cap *= 2;
    if (!generic_ && attention_smem_bytes(d_.heads, d_.kv_heads, d_.head_dim, cap) > 200 * 1024) {
        *error = "context length " + std::to_string(needed) + " exceeds the attention kernel's limit";
        return false;
    }
    destroy_graphs();  // graphs hold the old cache pointers and the attention smem size
    if (!alloc_kv(cap, error)) return false;
    if (persistent_) {
        if (!persistent_eligible(cap)) {
            persistent_ = false;  // longer contexts than the step kernel's attention scratch
        } else if (!build_phases(error)) {
            return false;
        }
    }
    return true;
}

bool DeviceModel::persistent_eligible(int capacity) const {
    const int group = d_.heads / d_.kv_heads;
    const size_t attn_floats =
        static_cast<size_t>(group) * d_.head_dim + static_cast<size_t>(group) * ((capacity + kAttnSplits - 1) / kAttnSplits);
    if (attn_floats * sizeof(float) > static_cast<size_t>(kStepAttnDynBytes)) return false;
    if (d_.lk_hd != 128 || d_.lv_hd % kDeltaCols != 0) return false;
    if (d_.kv_heads * kAttnSplits > num_sms_) return false;  // one attention item per block
    auto ok = [&](const DevMatrix& m) {
        return m.fast() && m.kind == lm_head_.kind && m.cols / 32 <= kStepConsumers &&
               m.row_stride * 4 <= kStepSlotBytes;
    };
    if (!ok(lm_head_)) return false;
    for (const DevLayer& L : layers_)
        if (!ok(L.in_proj) || !ok(L.out_proj) || !ok(L.gate_up) || !ok(L.down)) return false;
    return true;
}

// The phase list of one step: [head] + 5 phases per layer. head = lm_head argmax + next
// embedding (decode) or the prompt's embedding (prefill).
bool DeviceModel::build_phases(std::string* error) {
    const ModelDims& d = d_;
    bool staged_ok = true;  // every GEMV's inputs fit the step kernel's staging areas, 16-byte aligned
    auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    auto gemv = [&](const DevMatrix& m, int pro, int epi, int unit, GemvParams g) {
        if (step_act_bytes(pro, m.cols, g.head_dim) > static_cast<size_t>(kStepActBytes) || !aligned(g.x) ||
            !aligned(g.norm_w) || !aligned(g.gate_z) || !aligned(g.out) || !aligned(g.conv_w) ||
            !aligned(g.conv_state) || (epi == kEpiConv && g.conv_k != 4) || (epi == kEpiResidual && m.rows % 4 != 0) ||
            (pro == kProGatedRms && (g.head_dim < 32 || m.cols / g.head_dim > 32 || 32 % (g.head_dim / 32) != 0)))
            staged_ok = false;
        PhaseDesc D = {};
        D.kind = kPhaseGemv;
        D.pro = pro;
        D.epi = epi;
        g.w = m.d_rows;
        g.rows = m.rows;
        g.cols = m.cols;
        g.row_stride = m.row_stride;
        g.meta_offset = m.meta_offset;
        g.rows_per_chunk = kStepSlotBytes / m.row_stride >= 8 ? 8 : 4;
        if (meta_kind_ == kMetaMma) {
            // chunks of up to one ring slot of pairs (16 by default), a multiple of 8 (an even
            // number per warp of a team) that divides the tile's pairs
            g.w = m.d_tiles;
            g.mma_pairs = m.cols / 128;
            g.mma_ppc = 0;
            for (int k = 8; k * kMmaUnitBytes <= step_slot_bytes_; k += 8)
                if (g.mma_pairs % k == 0) g.mma_ppc = k;
            if (g.mma_ppc == 0) staged_ok = false;
        }
        g.stages = 0;
        g.unit = unit;
        g.evict_first = gemv_evict_first();
        g.err = d_err_;
        D.g = g;
        return D;
    };
    std::vector<PhaseDesc> forward;
    for (DevLayer& L : layers_) {
        if (!L.full) {
            GemvParams p = {};
            p.x = d_hidden_;
            p.norm_w = L.input_norm;
            p.eps = d.eps;
            p.out = d_conv_out_;
            p.out2 = d_zab_;
            p.conv_w = L.conv_w;
            p.conv_state = L.conv_state;
            p.conv_channels = d.conv_dim;
            p.conv_k = d.conv_k;
            forward.push_back(gemv(L.in_proj, kProRms, kEpiConv, 1, p));
            PhaseDesc D = {};
            D.kind = kPhaseDelta;
            D.d = DeltaParams{d_conv_out_, d_zab_ + d.lv_dim, L.a_log, L.dt_bias, L.rec_state, d_attn_raw_,
                              d.lk_heads, d.lv_heads, d.lk_hd, d.lv_hd};
            // tensor-core path: the gated head norm's elementwise part and per-slice sums of
            // squares in the DeltaNet phase; the out_proj prologue only scales each head
            const bool fuse_norm = meta_kind_ == kMetaMma && d_head_ss_ != nullptr;
            if (fuse_norm) {
                D.d.z = d_zab_;
                D.d.norm_w = L.lin_norm;
                D.d.head_ss = d_head_ss_;
            }
            forward.push_back(D);
            GemvParams q = {};
            q.x = d_attn_raw_;
            q.norm_w = L.lin_norm;
            q.gate_z = d_zab_;
            q.head_dim = d.lv_hd;
            q.eps = d.eps;
            q.out = d_hidden_;
            q.head_ss = d_head_ss_;
            q.head_ss_slices = d.lv_hd / kDeltaCols;
            forward.push_back(gemv(L.out_proj, fuse_norm ? kProHeadScale : kProGatedRms, kEpiResidual, 1, q));
        } else {
            GemvParams p = {};
            p.x = d_hidden_;
            p.norm_w = L.input_norm;
            p.eps = d.eps;
            p.out = d_qkv_;
            forward.push_back(gemv(L.in_proj, kProRms, kEpiStore, 1, p));
            PhaseDesc D = {};
            D.kind = kPhaseAttn;
            AttnParams& ap = D.a;
            ap.qkv = d_qkv_;
            ap.q_norm = L.q_norm;
            ap.k_norm = L.k_norm;
            ap.k_cache = L.k_cache;
            ap.v_cache = L.v_cache;
            ap.capacity = capacity_;
            ap.pos_ptr = d_pos_;
            ap.nq = d.heads;
            ap.nkv = d.kv_heads;
            ap.hd = d.head_dim;
            ap.rotary = d.rotary_dim;
            ap.theta = d.theta;
            ap.eps = d.eps;
            ap.rope = d_rope_;
            ap.rope_stride = d.rotary_dim / 2;
            ap.part = d_attn_part_;
            ap.counters = d_attn_counters_;
            ap.out = d_attn_out_;
            ap.err = d_err_;
            forward.push_back(D);
            GemvParams q = {};
            q.x = d_attn_out_;
            q.out = d_hidden_;
            forward.push_back(gemv(L.out_proj, kProPlain, kEpiResidual, 1, q));
        }
        GemvParams g = {};
        g.x = d_hidden_;
        g.norm_w = L.post_norm;
        g.eps = d.eps;
        g.out = d_ffn_;
        forward.push_back(gemv(L.gate_up, kProRms, kEpiSwiglu, 2, g));
        GemvParams dn = {};
        dn.x = d_ffn_;
        dn.out = d_hidden_;
        forward.push_back(gemv(L.down, kProPlain, kEpiResidual, 1, dn));
    }
    std::vector<PhaseDesc> dec, pre;
    {
        GemvParams p = {};
        p.x = d_hidden_;
        p.norm_w = d_final_norm_;  // runFinalNorm, custom_model.cpp:1258-1279
        p.eps = d.eps;
        p.part_val = d_arg_val_;
        p.part_idx = d_arg_idx_;
        p.counter = d_arg_counter_;
        p.token_out = d_token_;
        p.emb = d_emb_;
        p.hidden_out = d_hidden_;
        p.hidden = d.hidden;
        p.pos = d_pos_;
        p.next_pos = d_next_pos_;
        p.ring = d_ring_;
        p.ring_ctr = d_ring_ctr_;
        p.ring_cap = ring_cap_;
        dec.push_back(gemv(lm_head_, kProRms, kEpiArgmax, 1, p));
        PhaseDesc E = {};
        E.kind = kPhaseEmbed;
        pre.push_back(E);
    }
    dec.insert(dec.end(), forward.begin(), forward.end());
    pre.insert(pre.end(), forward.begin(), forward.end());
    n_phases_ = static_cast<int>(dec.size());
    phase_names_.clear();
    for (const PhaseDesc& D : dec) {
        std::string n;
        if (D.kind == kPhaseDelta) n = "delta";
        else if (D.kind == kPhaseAttn) n = "attention";
        else if (D.kind == kPhaseEmbed) n = "embed";
        else if (D.epi == kEpiArgmax) n = "lm_head_argmax";
        else if (D.epi == kEpiConv) n = "gemv_in_proj_conv";
        else if (D.epi == kEpiSwiglu) n = "gemv_gate_up";
        else if (D.pro == kProGatedRms || D.pro == kProHeadScale) n = "gemv_out_proj";
        else if (D.epi == kEpiStore) n = "gemv_qkv";
        else if (D.g.cols == d.inter) n = "gemv_down";
        else n = "gemv_o_proj";
        phase_names_.push_back(n);
    }
    phase_ns_.assign(kStepTraceSlots * static_cast<size_t>(n_phases_), 0.0);
    if (!staged_ok) {  // this model's shapes run on the per-op graph path instead
        persistent_ = false;
        return true;
    }
    // Tensor maps of every GEMV phase's staged vectors: [list][phase][3] in one device array.
    {
        const size_t per_list = static_cast<size_t>(n_phases_) * 3;
        std::vector<uint8_t> maps(2 * per_list * kStepTmapBytes, 0);
        cudaFree(d_tmaps_);
        d_tmaps_ = nullptr;
        if (cudaMalloc(&d_tmaps_, maps.size()) != cudaSuccess) {
            *error = "tensor map allocation failed";
            return false;
        }
        for (int which = 0; which < 2; ++which) {
            std::vector<PhaseDesc>& list = which == 0 ? dec : pre;
            for (int ph = 0; ph < n_phases_; ++ph) {
                PhaseDesc& D = list[ph];
                if (D.kind == kPhaseDelta && D.d.dk <= 256) {
                    // the phase stages each item's recurrent-state slice with this map
                    const size_t off = ((which * static_cast<size_t>(n_phases_) + ph) * 3) * kStepTmapBytes;
                    if (encode_state_tmap(maps.data() + off, D.d.state, D.d.nv * D.d.dk, D.d.dv, D.d.dk))
                        D.tmap[0] = static_cast<const uint8_t*>(d_tmaps_) + off;
                    continue;
                }
                if (D.kind != kPhaseGemv) continue;
                const GemvParams& g = D.g;
                const float* vec[3] = {g.x, nullptr, nullptr};
                int len[3] = {g.cols, 0, 0};
                if (D.pro == kProRms) vec[1] = g.norm_w, len[1] = g.cols;
                if (D.pro == kProGatedRms) vec[1] = g.gate_z, len[1] = g.cols, vec[2] = g.norm_w, len[2] = g.head_dim;
                for (int k = 0; k < 3; ++k) {
                    if (!vec[k]) continue;
                    const size_t off = ((which * static_cast<size_t>(n_phases_) + ph) * 3 + k) * kStepTmapBytes;
                    if (!encode_vector_tmap(maps.data() + off, vec[k], len[k])) {
                        persistent_ = false;  // no tensor maps: the per-op graph path runs instead
                        return true;
                    }
                    D.tmap[k] = static_cast<const uint8_t*>(d_tmaps_) + off;
                }
            }
        }
        if (cudaMemcpy(d_tmaps_, maps.data(), maps.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
            *error = "tensor map upload failed";
            return false;
        }
    }
    for (int which = 0; which < 2; ++which) {
        PhaseDesc*& dst = which == 0 ? d_phases_decode_ : d_phases_prefill_;
        const std::vector<PhaseDesc>& src = which == 0 ? dec : pre;
        cudaFree(dst);
        dst = nullptr;
        if (cudaMalloc(&dst, src.size() * sizeof(PhaseDesc)) != cudaSuccess ||
            cudaMemcpy(dst, src.data(), src.size() * sizeof(PhaseDesc), cudaMemcpyHostToDevice) != cudaSuccess) {
            *error = "phase list upload failed";
            return false;
        }
    }
    return true;
}

int DeviceModel::kernels_per_decode_step() const {
    if (persistent_) return 1;
    int n = 1;  // lm_head argmax + embedding
    for (const DevLayer& L : layers_) n += L.full ? 5 : 5;
    return n;
}

int DeviceModel::kernels_per_prefill_step() const { return kernels_per_decode_step(); }


bool DeviceModel::enqueue_forward(cudaStream_t s) {
    const ModelDims& d = d_;
    const bool pdl = pdl_enabled();
    LaunchCtx ctx;
    ctx.stream = s;
    ctx.num_sms = num_sms_;
    ctx.pdl = pdl;
    for (DevLayer& L : layers_) {
        if (!L.full) {
            GemvParams p = {};
            p.x = d_hidden_;
            p.norm_w = L.input_norm;
            p.eps = d.eps;
            p.out = d_conv_out_;
            p.out2 = d_zab_;
            p.conv_w = L.conv_w;
            p.conv_state = L.conv_state;
            p.conv_channels = d.conv_dim;
            p.conv_k = d.conv_k;
            p.err = d_err_;
            if (!launch_gemv(L.in_proj, kProRms, kEpiConv, p, 1, ctx)) return false;
            DeltaParams dp{d_conv_out_, d_zab_ + d.lv_dim, L.a_log, L.dt_bias, L.rec_state, d_attn_raw_,
                           d.lk_heads, d.lv_heads, d.lk_hd, d.lv_hd};
            if (launch_ex(gated_delta_kernel, dim3(d.lv_heads, d.lv_hd / kDeltaCols), dim3(d.lk_hd), 0, s, pdl,
                          dp) != cudaSuccess) {
                set_last_error("gated delta launch failed");
                return false;
            }
            GemvParams q = {};
            q.x = d_attn_raw_;
            q.norm_w = L.lin_norm;
            q.gate_z = d_zab_;
            q.head_dim = d.lv_hd;
            q.eps = d.eps;
            q.out = d_hidden_;
            q.err = d_err_;
            if (!launch_gemv(L.out_proj, kProGatedRms, kEpiResidual, q, 1, ctx)) return false;
        } else {
            GemvParams p = {};
            p.x = d_hidden_;
            p.norm_w = L.input_norm;
            p.eps = d.eps;
            p.out = d_qkv_;
            p.err = d_err_;
            if (!launch_gemv(L.in_proj, kProRms, kEpiStore, p, 1, ctx)) return false;
            AttnParams ap = {};
            ap.qkv = d_qkv_;
            ap.q_norm = L.q_norm;
            ap.k_norm = L.k_norm;
            ap.k_cache = L.k_cache;
            ap.v_cache = L.v_cache;
            ap.capacity = capacity_;
            ap.pos_ptr = d_pos_;
            ap.nq = d.heads;
            ap.nkv = d.kv_heads;
            ap.hd = d.head_dim;
            ap.rotary = d.rotary_dim;
            ap.theta = d.theta;
            ap.eps = d.eps;
            ap.rope = d_rope_;
            ap.rope_stride = d.rotary_dim / 2;
            ap.part = d_attn_part_;
            ap.counters = d_attn_counters_;
            ap.out = d_attn_out_;
            ap.err = d_err_;
            const size_t smem = attention_smem_bytes(d.heads, d.kv_heads, d.head_dim, capacity_);
            const cudaError_t e = launch_attention(ap, opts_.kv_fp16, smem, s, pdl);
            if (e != cudaSuccess) {
                set_last_error(std::string("attention launch failed: ") + cudaGetErrorString(e));
                return false;
            }
            GemvParams q = {};
            q.x = d_attn_out_;
            q.out = d_hidden_;
            q.err = d_err_;
            if (!launch_gemv(L.out_proj, kProPlain, kEpiResidual, q, 1, ctx)) return false;
        }
        GemvParams g = {};
        g.x = d_hidden_;
        g.norm_w = L.post_norm;
        g.eps = d.eps;
        g.out = d_ffn_;
        g.err = d_err_;
        if (!launch_gemv(L.gate_up, kProRms, kEpiSwiglu, g, 2, ctx)) return false;
        GemvParams dn = {};
        dn.x = d_ffn_;
        dn.out = d_hidden_;
        dn.err = d_err_;
        if (!launch_gemv(L.down, kProPlain, kEpiResidual, dn, 1, ctx)) return false;
    }
    return true;
}

bool DeviceModel::gemv_any(const DevMatrix& m, const float* x, float* y, cudaStream_t s) {
    if (m.kind == 2) return launch_gemv_generic(m, x, y, s);
    GemvParams p = {};
    p.x = x;
    p.out = y;
    p.err = d_err_;
    LaunchCtx ctx;
    ctx.stream = s;
    ctx.num_sms = num_sms_;
    ctx.pdl = false;
    return launch_gemv(m, kProPlain, kEpiStore, p, 1, ctx);
}

// One step of the generic-shape path: the reference's per-token sequence of operations
// (custom_model.cpp:1138-1279 for a layer, 1340-1356 for decode) with plain GEMVs and the
// generic kernels of generic.cu.
bool DeviceModel::enqueue_generic_step(bool decode, cudaStream_t s) {
    const ModelDims& d = d_;
    auto ok = [](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        set_last_error(std::string("generic step: ") + what + ": " + cudaGetErrorString(e));
        return false;
    };
    if (decode) {
        rmsnorm_kernel<<<1, 1024, 0, s>>>(d_hidden_, d_final_norm_, d.hidden, d.eps, d_normed_);
        if (!gemv_any(lm_head_, d_normed_, d_logits_, s) ||
            !ok(generic_sample(d_logits_, d.vocab, d_emb_, d_hidden_, d.hidden, d_pos_, d_next_pos_, d_token_, d_ring_,
                               d_ring_ctr_, ring_cap_, s),
                "sample"))
            return false;
    } else {
        embed_prefill_kernel<<<1, 512, 0, s>>>(d_prompt_, d_emb_, d_hidden_, d.hidden, d.vocab, d_pos_, d_next_pos_);
        if (!ok(cudaGetLastError(), "embedding")) return false;
    }
    for (DevLayer& L : layers_) {
        rmsnorm_kernel<<<1, 1024, 0, s>>>(d_hidden_, L.input_norm, d.hidden, d.eps, d_normed_);
        if (!gemv_any(L.in_proj, d_normed_, d_gy_, s)) return false;
        if (!L.full) {
            GenericLinearArgs a{d_gy_, L.conv_w, L.conv_state, L.a_log, L.dt_bias, L.rec_state, L.lin_norm, d.eps,
                                d_conv_out_, d_attn_raw_, d.lk_heads, d.lv_heads, d.lk_hd, d.lv_hd, d.conv_k};
            if (!ok(generic_linear_attn(a, s), "linear attention") ||
                !gemv_any(L.out_proj, d_attn_raw_, d_normed_, s))
                return false;
        } else {
            GenericAttnArgs a{d_gy_,     2 * d.heads * d.head_dim, L.q_norm, L.k_norm, d_rope_, d.rotary_dim / 2,
                              static_cast<float*>(L.k_cache), static_cast<float*>(L.v_cache), d_pos_, d_gscore_,
                              d_gqbuf_, d_attn_out_, d.heads, d.kv_heads, d.head_dim, d.rotary_dim, d.eps};
            if (!ok(generic_attention(a, s), "attention") || !gemv_any(L.out_proj, d_attn_out_, d_normed_, s))
                return false;
        }
        if (!ok(generic_add(d_hidden_, d_normed_, d.hidden, s), "residual")) return false;
        rmsnorm_kernel<<<1, 1024, 0, s>>>(d_hidden_, L.post_norm, d.hidden, d.eps, d_normed_);
        if (!gemv_any(L.gate_up, d_normed_, d_gy_, s) || !ok(generic_swiglu(d_gy_, d_ffn_, d.inter, s), "swiglu") ||
            !gemv_any(L.down, d_ffn_, d_normed_, s) || !ok(generic_add(d_hidden_, d_normed_, d.hidden, s), "residual"))
            return false;
    }
    return ok(cudaGetLastError(), "launch");
}

bool DeviceModel::enqueue_decode_step(cudaStream_t s) {
    if (generic_) return enqueue_generic_step(true, s);
    LaunchCtx ctx;
    ctx.stream = s;
    ctx.num_sms = num_sms_;
    ctx.pdl = pdl_enabled();
    GemvParams p = {};
    p.x = d_hidden_;
    p.norm_w = d_final_norm_;  // runFinalNorm, custom_model.cpp:1258-1279
    p.eps = d_.eps;
    p.part_val = d_arg_val_;
    p.part_idx = d_arg_idx_;
    p.counter = d_arg_counter_;
    p.token_out = d_token_;
    p.emb = d_emb_;
    p.hidden_out = d_hidden_;
    p.hidden = d_.hidden;
    p.pos = d_pos_;
    p.next_pos = d_next_pos_;
    p.ring = d_ring_;
    p.ring_ctr = d_ring_ctr_;
    p.ring_cap = ring_cap_;
    p.err = d_err_;
    if (!launch_gemv(lm_head_, kProRms, kEpiArgmax, p, 1, ctx, num_sms_)) return false;
    return enqueue_forward(s);
}

bool DeviceModel::enqueue_prefill_step(cudaStream_t s) {
    if (generic_) return enqueue_generic_step(false, s);
    if (launch_ex(embed_prefill_kernel, dim3(1), dim3(512), 0, s, pdl_enabled(), static_cast<const int*>(d_prompt_),
                  static_cast<const uint16_t*>(d_emb_), d_hidden_, d_.hidden, d_.vocab, d_pos_, d_next_pos_) !=
        cudaSuccess) {
        set_last_error("embedding launch failed");
        return false;
    }
    return enqueue_forward(s);
}

void DeviceModel::destroy_graphs() {
    if (g_decode_) cudaGraphExecDestroy(g_decode_);
    if (g_prefill_) cudaGraphExecDestroy(g_prefill_);
    g_decode_ = g_prefill_ = nullptr;
}

bool DeviceModel::capture_graphs(std::string* error) {
    for (int which = 0; which < 2; ++which) {
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            *error = "cudaStreamBeginCapture failed";
            return false;
        }
        const bool ok = which == 0 ? enqueue_decode_step(stream_) : enqueue_prefill_step(stream_);
        const cudaError_t e = cudaStreamEndCapture(stream_, &graph);
        if (!ok || e != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            *error = std::string("graph capture failed: ") + (ok ? cudaGetErrorString(e) : last_error());
            return false;
        }
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) {
            *error = std::string("graph instantiate failed: ") + cudaGetErrorString(ie);
            return false;
        }
        (which == 0 ? g_decode_ : g_prefill_) = exec;
    }
    return true;
}

bool DeviceModel::run_step(bool decode, std::string* error) {
    if (!ensure_capacity(position_ + 1, error)) return false;
    if (persistent_) {
        StepParams sp = {};
        sp.phases = decode ? d_phases_decode_ : d_phases_prefill_;
        sp.nphases = n_phases_;
        sp.nslots = step_slots_;
        sp.slot_bytes = step_slot_bytes_;
        sp.inflight = step_inflight_;
        sp.l2_prefetch = step_l2_prefetch_;
        sp.l2_ahead = step_l2_ahead_;
        sp.grid_bar = d_grid_bar_;
        sp.err = d_err_;
        sp.wait_ns = step_wait_ns_;
        sp.barrier_extra = (step_launches_ == stall_launch_) ? 1u : 0u;
        sp.prompt = d_prompt_;
        sp.emb = d_emb_;
        sp.hidden = d_hidden_;
        sp.hidden_size = d_.hidden;
        sp.vocab = d_.vocab;
        sp.pos = d_pos_;
        sp.next_pos = d_next_pos_;
        sp.trace = decode ? d_step_trace_ : nullptr;
        sp.block_done = decode ? d_block_done_ : nullptr;
        if (sp.trace) cudaMemsetAsync(d_step_trace_, 0, kStepTraceSlots * static_cast<size_t>(n_phases_) * 8, stream_);
        const cudaError_t e = launch_decode_step(sp, meta_kind_, opts_.kv_fp16, num_sms_, stream_);
        if (e == cudaSuccess && sp.trace) {
            std::vector<unsigned long long> t(kStepTraceSlots * static_cast<size_t>(n_phases_));
            cudaMemcpyAsync(t.data(), d_step_trace_, t.size() * 8, cudaMemcpyDeviceToHost, stream_);
            cudaStreamSynchronize(stream_);
            constexpr int S = kStepTraceSlots;
            for (int ph = 0; ph < n_phases_; ++ph) {
                const double start = static_cast<double>(t[S * ph]);
                const double prev_end = ph ? static_cast<double>(t[S * (ph - 1) + 2]) : start;
                phase_ns_[S * ph] += start - prev_end;  // barrier latency
                for (int k = 1; k < S; ++k) {
                    if (!t[S * ph + k]) continue;
                    if (k == 8 || k == 9)
                        phase_ns_[S * ph + k] += static_cast<double>(t[S * ph + k]);  // durations
                    else
                        phase_ns_[S * ph + k] += static_cast<double>(t[S * ph + k]) - start;
                }
            }
            if (sp.block_done) {
                const size_t G = static_cast<size_t>(num_sms_);
                std::vector<unsigned long long> bd(static_cast<size_t>(n_phases_) * G);
                cudaMemcpy(bd.data(), d_block_done_, bd.size() * 8, cudaMemcpyDeviceToHost);
                block_late_ns_.resize(bd.size(), 0.0);
                barrier_ns_.resize(n_phases_, 0.0);
                for (int ph = 0; ph < n_phases_; ++ph) {
                    unsigned long long lo = ~0ull, hi = 0;
                    for (size_t b = 0; b < G; ++b) {
                        lo = std::min(lo, bd[ph * G + b]);
                        hi = std::max(hi, bd[ph * G + b]);
                    }
                    for (size_t b = 0; b < G; ++b)
                        block_late_ns_[ph * G + b] += static_cast<double>(bd[ph * G + b] - lo);
                    // from the last block's finish to block 0 passing the next phase's barrier
                    if (ph + 1 < n_phases_)
                        barrier_ns_[ph] += static_cast<double>(t[S * (ph + 1)]) - static_cast<double>(hi);
                }
            }
            ++traced_steps_;
        }
        if (e != cudaSuccess) {
            *error = std::string("step kernel launch failed: ") + cudaGetErrorString(e);
            return false;
        }
        ++step_launches_;
        ++position_;
        if (decode) ++ring_count_;
        return true;
    }
    if (opts_.use_graphs) {
        if (!g_decode_ && !capture_graphs(error)) return false;
        const cudaError_t e = cudaGraphLaunch(decode ? g_decode_ : g_prefill_, stream_);
        if (e != cudaSuccess) {
            *error = std::string("graph launch failed: ") + cudaGetErrorString(e);
            return false;
        }
    } else {
        if (!(decode ? enqueue_decode_step(stream_) : enqueue_prefill_step(stream_))) {
            *error = last_error();
            return false;
        }
    }
    ++position_;
    if (decode) ++ring_count_;
    return true;
}

bool DeviceModel::reset(std::string* error) {
    if (!loaded_) {
        *error = "model not loaded";
        return false;
    }
    for (DevLayer& L : layers_) {
        if (L.full) continue;
        cudaMemsetAsync(L.conv_state, 0, sizeof(float) * d_.conv_dim * std::max(0, d_.conv_k - 1), stream_);
        cudaMemsetAsync(L.rec_state, 0, sizeof(float) * d_.lv_heads * d_.lk_hd * d_.lv_hd, stream_);
    }
    cudaMemsetAsync(d_pos_, 0, sizeof(int), stream_);
    cudaMemsetAsync(d_next_pos_, 0, sizeof(int), stream_);
    cudaMemsetAsync(d_ring_ctr_, 0, sizeof(int), stream_);
    clear_device_errors();
    position_ = 0;
    ring_count_ = 0;
    if (cudaStreamSynchronize(stream_) != cudaSuccess) {
        *error = std::string("reset failed: ") + cudaGetErrorString(cudaGetLastError());
        return false;
    }
    return true;
}

bool DeviceModel::prefill(const int32_t* ids, size_t n, std::string* error) {
    if (!ids || n == 0) {
        *error = "custom prefill requires prompt tokens";
        return false;
    }
    cudaSetDevice(opts_.device);
    if (!reset(error)) return false;
    if (n > prompt_cap_) {
        if (d_prompt_) cudaFree(d_prompt_);
        d_prompt_ = nullptr;
        prompt_cap_ = 0;
        if (cudaMalloc(&d_prompt_, n * sizeof(int)) != cudaSuccess) {
            *error = "prompt allocation failed";
            return false;
        }
        prompt_cap_ = n;
        destroy_graphs();  // the prefill graph holds the prompt pointer
    }
    if (cudaMemcpyAsync(d_prompt_, ids, n * sizeof(int), cudaMemcpyHostToDevice, stream_) != cudaSuccess) {
        *error = "prompt upload failed";
        return false;
    }
    for (size_t i = 0; i < n; ++i)
        if (!run_step(false, error)) return false;
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        *error = std::string("prefill failed: ") + cudaGetErrorString(e);
        return false;
    }
    return check_device_errors("prefill", error);
}

bool DeviceModel::batched_prefill_eligible(size_t n) const {
    if (n == 0 || lm_head_.kind != 0) return false;
    for (const DevLayer& L : layers_)
        for (const DevMatrix* m : {&L.in_proj, &L.out_proj, &L.gate_up, &L.down})
            if (m->kind != 0 || !m->d_rows || m->cols % 64 != 0) return false;
    if (d_.head_dim != 256 || d_.lk_hd != 128 || d_.lv_hd % kDeltaCols != 0 || d_.conv_k != 4) return false;
    return prefill_attn_smem(d_.heads, d_.kv_heads, d_.head_dim, static_cast<int>(n)) <= kPrefillAttnMaxSmem;
}

bool DeviceModel::prefill_batched(const int32_t* ids, size_t n, std::string* error, bool* unsupported) {
    *unsupported = false;
    if (!ids || n == 0) {
        *error = "custom prefill requires prompt tokens";
        return false;
    }
    if (!batched_prefill_eligible(n)) {
        *unsupported = true;
        *error = "batched prefill does not serve this package or context";
        return false;
    }
    cudaSetDevice(opts_.device);
    if (!reset(error)) return false;
    if (!ensure_capacity(static_cast<int>(n), error)) return false;
    const ModelDims& d = d_;
    const int C = kPrefillChunk;
    if (!pf_H_) {
        pf_kmax_ = std::max({d.hidden, d.inter, d.lv_dim, d.heads * d.head_dim});
        pf_ymax_ = std::max(lm_head_.cols, 0);
        for (const DevLayer& L : layers_) pf_ymax_ = std::max({pf_ymax_, L.in_proj.rows, L.gate_up.rows});
        if (!dev_alloc(&pf_H_, static_cast<size_t>(C) * d.hidden, error) ||
            !dev_alloc(&pf_Y_, static_cast<size_t>(C) * pf_ymax_, error) ||
            !dev_alloc(&pf_conv_, static_cast<size_t>(C) * d.conv_dim, error) ||
            !dev_alloc(&pf_O_, static_cast<size_t>(C) * d.lv_dim, error) ||
            !dev_alloc(&pf_Q_, static_cast<size_t>(C) * d.heads * d.head_dim, error) ||
            !dev_alloc(reinterpret_cast<uint16_t**>(&pf_xhi_), static_cast<size_t>(C) * pf_kmax_, error) ||
            !dev_alloc(reinterpret_cast<uint16_t**>(&pf_xlo_), static_cast<size_t>(C) * pf_kmax_, error) ||
            !dev_alloc(&pf_ids_, static_cast<size_t>(C), error))
            return false;
    }
    static const int passes = [] {
        const char* v = std::getenv("XQ_PREFILL_PASSES");
        return v && std::atoi(v) == 1 ? 1 : 3;
    }();
    __nv_bfloat16* xhi = static_cast<__nv_bfloat16*>(pf_xhi_);
    __nv_bfloat16* xlo = passes == 1 ? nullptr : static_cast<__nv_bfloat16*>(pf_xlo_);
    cudaStream_t s = stream_;
    const bool f16 = opts_.kv_fp16;
    auto ok = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        *error = std::string("batched prefill: ") + what + ": " + cudaGetErrorString(e);
        return false;
    };
    auto gemm = [&](const DevMatrix& m, int nc, float* y, int ldy, int kind) {
        if (launch_prefill_gemm(m, xhi, xlo, nc, y, ldy, kind, d_err_, num_sms_, s, step_wait_ns_)) return true;
        *error = std::string("batched prefill: ") + last_error();
        return false;
    };
    for (size_t p0 = 0; p0 < n; p0 += C) {
        const int nc = static_cast<int>(std::min<size_t>(C, n - p0));
        if (!ok(cudaMemcpyAsync(pf_ids_, ids + p0, sizeof(int) * nc, cudaMemcpyHostToDevice, s), "prompt upload") ||
            !ok(prefill_embed(pf_ids_, d_emb_, pf_H_, nc, d.hidden, d.vocab, s), "embedding"))
            return false;
        for (DevLayer& L : layers_) {
            if (!ok(prefill_rmsnorm_split(pf_H_, L.input_norm, nc, d.hidden, d.eps, xhi, xlo, s), "input norm"))
                return false;
            const int ldy = L.in_proj.rows;
            if (!gemm(L.in_proj, nc, pf_Y_, ldy, kPgOutF32)) return false;
            if (!L.full) {
                // in_proj rows: [qkv (conv_dim) | z (lv_dim) | a (lv_heads) | b (lv_heads)]
                if (!ok(prefill_conv(pf_Y_, ldy, L.conv_w, L.conv_state, pf_conv_, nc, d.conv_dim, s), "conv") ||
                    !ok(prefill_delta(pf_conv_, d.conv_dim, pf_Y_, ldy, d.conv_dim + d.lv_dim, L.a_log, L.dt_bias,
                                      L.rec_state, pf_O_, d.lv_dim, nc, d.lk_heads, d.lv_heads, d.lk_hd, d.lv_hd, s),
                        "gated delta") ||
                    !ok(prefill_gated_norm(pf_O_, d.lv_dim, pf_Y_, ldy, d.conv_dim, L.lin_norm, d.lv_heads, d.lv_hd,
                                           d.eps, nc, xhi, xlo, s),
                        "gated norm"))
                    return false;
            } else {
                if (!ok(prefill_attn_prep(pf_Y_, ldy, L.q_norm, L.k_norm, d_rope_, d.rotary_dim / 2, pf_Q_, L.k_cache,
                                          L.v_cache, f16, static_cast<int>(p0), nc, d.heads, d.kv_heads, d.head_dim,
                                          d.eps, s),
                        "attention prologue") ||
                    !ok(prefill_attn(pf_Q_, pf_Y_, ldy, L.k_cache, L.v_cache, f16, static_cast<int>(p0), nc, d.heads,
                                     d.kv_heads, d.head_dim, xhi, xlo, s),
                        "attention"))
                    return false;
            }
            if (!gemm(L.out_proj, nc, pf_H_, d.hidden, kPgOutAddF32)) return false;  // residual add
            if (!ok(prefill_rmsnorm_split(pf_H_, L.post_norm, nc, d.hidden, d.eps, xhi, xlo, s), "post norm") ||
                !gemm(L.gate_up, nc, pf_Y_, L.gate_up.rows, kPgOutF32) ||
                !ok(prefill_swiglu(pf_Y_, L.gate_up.rows, d.inter, nc, xhi, xlo, s), "swiglu") ||
                !gemm(L.down, nc, pf_H_, d.hidden, kPgOutAddF32))
                return false;
        }
        if (p0 + nc == n &&
            !ok(cudaMemcpyAsync(d_hidden_, pf_H_ + static_cast<size_t>(nc - 1) * d.hidden, sizeof(float) * d.hidden,
                                cudaMemcpyDeviceToDevice, s),
                "hidden copy"))
            return false;
    }
    // positions as after n token-serial steps: pos = n - 1, next_pos = n
    const int pos[2] = {static_cast<int>(n) - 1, static_cast<int>(n)};
    if (!ok(cudaMemcpyAsync(d_pos_, &pos[0], sizeof(int), cudaMemcpyHostToDevice, s), "positions") ||
        !ok(cudaMemcpyAsync(d_next_pos_, &pos[1], sizeof(int), cudaMemcpyHostToDevice, s), "positions"))
        return false;
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        *error = std::string("batched prefill failed: ") + cudaGetErrorString(e);
        return false;
    }
    position_ = static_cast<int>(n);
    return check_device_errors("batched prefill", error);
}

bool DeviceModel::decode_one(int32_t* token, std::string* error) {
    cudaSetDevice(opts_.device);
    if (!run_step(true, error)) return false;
    if (cudaMemcpyAsync(h_token_, d_token_, sizeof(int32_t), cudaMemcpyDeviceToHost, stream_) != cudaSuccess) {
        *error = "token copy failed";
        return false;
    }
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        *error = std::string("decode failed: ") + cudaGetErrorString(e);
        return false;
    }
    if (!check_device_errors("decode step", error)) return false;
    *token = *h_token_;
    return true;
}

bool DeviceModel::decode_many(size_t count, std::string* error) {
    cudaSetDevice(opts_.device);
    for (size_t i = 0; i < count; ++i)
        if (!run_step(true, error)) return false;
    return true;
}

bool DeviceModel::decode_many_timed(size_t count, double* device_ms, std::string* error) {
    cudaSetDevice(opts_.device);
    // Capture (or re-capture after growth) before the first event so it is not timed.
    if (!ensure_capacity(position_ + static_cast<int>(count), error)) return false;
    if (!persistent_ && opts_.use_graphs && !g_decode_ && !capture_graphs(error)) return false;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, stream_);
    const bool ok = decode_many(count, error);
    cudaEventRecord(e1, stream_);
    const cudaError_t e = cudaEventSynchronize(e1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (!ok) return false;
    if (e != cudaSuccess) {
        *error = std::string("decode failed: ") + cudaGetErrorString(e);
        return false;
    }
    if (!check_device_errors("decode step", error)) return false;
    *device_ms = ms;
    return true;
}

bool DeviceModel::read_ring(size_t first, size_t count, int32_t* out, std::string* error) {
    if (count > static_cast<size_t>(ring_cap_)) {
        *error = "too many tokens requested from the device ring";
        return false;
    }
    for (size_t i = 0; i < count;) {
        const size_t idx = (first + i) % ring_cap_;
        const size_t n = std::min(count - i, ring_cap_ - idx);
        if (cudaMemcpyAsync(out + i, d_ring_ + idx, n * sizeof(int32_t), cudaMemcpyDeviceToHost, stream_) !=
            cudaSuccess) {
            *error = "token ring copy failed";
            return false;
        }
        i += n;
    }
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        *error = std::string("decode failed: ") + cudaGetErrorString(e);
        return false;
    }
    return check_device_errors("decode step", error);
}

bool DeviceModel::hidden(std::vector<float>* out, std::string* error) {
    cudaSetDevice(opts_.device);
    rmsnorm_kernel<<<1, 1024, 0, stream_>>>(d_hidden_, d_final_norm_, d_.hidden, d_.eps, d_normed_);
    out->resize(static_cast<size_t>(d_.hidden));
    cudaMemcpyAsync(out->data(), d_normed_, out->size() * 4, cudaMemcpyDeviceToHost, stream_);
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        *error = std::string("hidden state copy failed: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

bool DeviceModel::logits(std::vector<float>* out, std::string* error) {
    cudaSetDevice(opts_.device);
    rmsnorm_kernel<<<1, 1024, 0, stream_>>>(d_hidden_, d_final_norm_, d_.hidden, d_.eps, d_normed_);
    if (!gemv_any(lm_head_, d_normed_, d_logits_, stream_)) {
        *error = last_error();
        return false;
    }
    out->resize(static_cast<size_t>(d_.vocab));
    cudaMemcpyAsync(out->data(), d_logits_, out->size() * 4, cudaMemcpyDeviceToHost, stream_);
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) {
        *error = std::string("logits failed: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

namespace {
struct SnapshotHeader {
    char magic[8];  // "XQSNAP1\0"
    uint32_t version, kv_elem;
    int32_t position, pos, next_pos, reserved0;
    uint32_t layers, hidden, conv_dim, conv_k, lv_heads, lk_hd, lv_hd, kv_heads, head_dim, full_layers;
    uint64_t bytes;
};
constexpr char kSnapMagic[8] = {'X', 'Q', 'S', 'N', 'A', 'P', '1', '\0'};
}  // namespace

size_t DeviceModel::snapshot_bytes() const {
    const size_t conv = static_cast<size_t>(d_.conv_dim) * std::max(0, d_.conv_k - 1);
    const size_t rec = static_cast<size_t>(d_.lv_heads) * d_.lk_hd * d_.lv_hd;
    const size_t kv = static_cast<size_t>(position_) * d_.kv_heads * d_.head_dim * (opts_.kv_fp16 ? 2 : 4);
    size_t b = sizeof(SnapshotHeader) + sizeof(float) * static_cast<size_t>(d_.hidden);
    for (const DevLayer& L : layers_) b += L.full ? 2 * kv : sizeof(float) * (conv + rec);
    return b;
}

bool DeviceModel::save_snapshot(void* buf, size_t cap, size_t* written, std::string* error) {
    const size_t need = snapshot_bytes();
    if (written) *written = need;
    if (!buf || cap < need) {
        *error = "snapshot buffer too small";
        return false;
    }
    SnapshotHeader h = {};
    std::memcpy(h.magic, kSnapMagic, 8);
    h.version = 1;
    h.kv_elem = opts_.kv_fp16 ? 2 : 4;
    h.position = position_;
    h.layers = static_cast<uint32_t>(layers_.size());
    h.hidden = d_.hidden, h.conv_dim = d_.conv_dim, h.conv_k = d_.conv_k, h.lv_heads = d_.lv_heads;
    h.lk_hd = d_.lk_hd, h.lv_hd = d_.lv_hd, h.kv_heads = d_.kv_heads, h.head_dim = d_.head_dim;
    for (const DevLayer& L : layers_) h.full_layers += L.full ? 1 : 0;
    h.bytes = need;
    uint8_t* p = static_cast<uint8_t*>(buf) + sizeof h;
    auto get = [&](const void* src, size_t bytes) {
        const cudaError_t e = cudaMemcpyAsync(p, src, bytes, cudaMemcpyDeviceToHost, stream_);
        p += bytes;
        return e == cudaSuccess;
    };
    int32_t dev_pos[2] = {0, 0};  // device positions, written to the header once they arrive
    bool ok = cudaMemcpyAsync(dev_pos, d_pos_, 4, cudaMemcpyDeviceToHost, stream_) == cudaSuccess &&
              cudaMemcpyAsync(dev_pos + 1, d_next_pos_, 4, cudaMemcpyDeviceToHost, stream_) == cudaSuccess;
    ok = ok && get(d_hidden_, sizeof(float) * d_.hidden);
    const size_t conv = static_cast<size_t>(d_.conv_dim) * std::max(0, d_.conv_k - 1);
    const size_t rec = static_cast<size_t>(d_.lv_heads) * d_.lk_hd * d_.lv_hd;
    const size_t kv = static_cast<size_t>(position_) * d_.kv_heads * d_.head_dim * h.kv_elem;
    for (const DevLayer& L : layers_) {
        if (L.full)
            ok = ok && get(L.k_cache, kv) && get(L.v_cache, kv);
        else
            ok = ok && get(L.conv_state, sizeof(float) * conv) && get(L.rec_state, sizeof(float) * rec);
    }
    ok = ok && cudaStreamSynchronize(stream_) == cudaSuccess;
    if (!ok) {
        *error = std::string("snapshot copy failed: ") + cudaGetErrorString(cudaGetLastError());
        return false;
    }
    h.pos = dev_pos[0];
    h.next_pos = dev_pos[1];
    std::memcpy(buf, &h, sizeof h);
    return true;
}

bool DeviceModel::restore_snapshot(const void* buf, size_t size, std::string* error, bool* invalid) {
    *invalid = true;
    SnapshotHeader h;
    if (!buf || size < sizeof h) {
        *error = "snapshot too small";
        return false;
    }
    std::memcpy(&h, buf, sizeof h);
    uint32_t full = 0;
    for (const DevLayer& L : layers_) full += L.full ? 1 : 0;
    if (std::memcmp(h.magic, kSnapMagic, 8) != 0 || h.version != 1) {
        *error = "not a snapshot of this library";
        return false;
    }
    if (h.kv_elem != (opts_.kv_fp16 ? 2u : 4u) || h.layers != layers_.size() || h.full_layers != full ||
        h.hidden != static_cast<uint32_t>(d_.hidden) || h.conv_dim != static_cast<uint32_t>(d_.conv_dim) ||
        h.conv_k != static_cast<uint32_t>(d_.conv_k) || h.lv_heads != static_cast<uint32_t>(d_.lv_heads) ||
        h.lk_hd != static_cast<uint32_t>(d_.lk_hd) || h.lv_hd != static_cast<uint32_t>(d_.lv_hd) ||
        h.kv_heads != static_cast<uint32_t>(d_.kv_heads) || h.head_dim != static_cast<uint32_t>(d_.head_dim) ||
        h.position < 0 || h.next_pos != h.position) {
        *error = "snapshot does not match this model (shape, KV type or positions)";
        return false;
    }
    const size_t conv = static_cast<size_t>(d_.conv_dim) * std::max(0, d_.conv_k - 1);
    const size_t rec = static_cast<size_t>(d_.lv_heads) * d_.lk_hd * d_.lv_hd;
    const size_t kv = static_cast<size_t>(h.position) * d_.kv_heads * d_.head_dim * h.kv_elem;
    const size_t need = sizeof h + sizeof(float) * static_cast<size_t>(d_.hidden) +
                        static_cast<size_t>(full) * 2 * kv + (layers_.size() - full) * sizeof(float) * (conv + rec);
    if (size < need || h.bytes != need) {
        *error = "snapshot size does not match its header";
        return false;
    }
    *invalid = false;
    if (!ensure_capacity(std::max(1, h.position), error)) return false;
    const uint8_t* p = static_cast<const uint8_t*>(buf) + sizeof h;
    auto put = [&](void* dst, size_t bytes) {
        const cudaError_t e = cudaMemcpyAsync(dst, p, bytes, cudaMemcpyHostToDevice, stream_);
        p += bytes;
        return e == cudaSuccess;
    };
    bool ok = cudaMemcpyAsync(d_pos_, &h.pos, 4, cudaMemcpyHostToDevice, stream_) == cudaSuccess &&
              cudaMemcpyAsync(d_next_pos_, &h.next_pos, 4, cudaMemcpyHostToDevice, stream_) == cudaSuccess;
    ok = ok && put(d_hidden_, sizeof(float) * d_.hidden);
    for (DevLayer& L : layers_) {
        if (L.full)
            ok = ok && put(L.k_cache, kv) && put(L.v_cache, kv);
        else
            ok = ok && put(L.conv_state, sizeof(float) * conv) && put(L.rec_state, sizeof(float) * rec);
    }
    ok = ok && cudaMemsetAsync(d_ring_ctr_, 0, sizeof(int), stream_) == cudaSuccess;
    ok = ok && cudaStreamSynchronize(stream_) == cudaSuccess;
    if (!ok) {
        *error = std::string("snapshot restore failed: ") + cudaGetErrorString(cudaGetLastError());
        return false;
    }
    position_ = h.position;
    ring_count_ = 0;
    return true;
}

std::vector<DeviceModel::PhaseTime> DeviceModel::phase_times() const {
    std::vector<PhaseTime> out;
    if (!traced_steps_) return out;
    constexpr int S = kStepTraceSlots;
    std::map<std::string, std::pair<int, double>> agg;
    for (int ph = 0; ph < n_phases_; ++ph) {
        auto& a = agg[phase_names_[ph]];
        a.first += 1;
        a.second += (phase_ns_[S * ph] + phase_ns_[S * ph + 2]) / traced_steps_ / 1000.0;  // barrier + phase
    }
    for (const auto& kv : agg) out.push_back({kv.first, kv.second.first, traced_steps_, kv.second.second});
    return out;
}

std::string DeviceModel::phase_trace_summary() const {
    if (!traced_steps_) return "";
    constexpr int S = kStepTraceSlots;
    std::map<std::string, std::array<double, S + 1>> agg;
    for (int ph = 0; ph < n_phases_; ++ph) {
        auto& a = agg[phase_names_[ph]];
        a[0] += 1;
        for (int k = 0; k < S; ++k) a[k + 1] += phase_ns_[S * ph + k] / traced_steps_;
    }
    // Per slot: the summed microseconds of all phases of that name, per step.
    static const char* kSlotNames[S] = {"barrier_us",    "block0_us",     "last_arrival_us", "x_loaded_us",
                                        "limbs_ready_us", "first_chunk_us", "loop_done_us",   "constants_staged_us",
                                        "chunk_wait_us", "producer_slot_wait_us", "x_staged_us",
                                        "barrier_seen_us", "activations_issued_us"};
    std::ostringstream o;
    o << "{\"steps\":" << traced_steps_ << ",\"phases\":[";
    bool first = true;
    for (const auto& kv : agg) {
        if (!first) o << ",";
        first = false;
        o << "{\"name\":\"" << kv.first << "\",\"count\":" << kv.second[0];
        for (int k = 0; k < S; ++k) o << ",\"" << kSlotNames[k] << "\":" << kv.second[k + 1] / 1000.0;
        o << "}";
    }
    o << "]";
    if (!block_late_ns_.empty()) {
        // Per phase name: mean (over phases and steps) of the last block's lateness behind the
        // first, and the blocks that are latest on average.
        const size_t G = static_cast<size_t>(num_sms_);
        std::map<std::string, std::vector<double>> late;
        std::map<std::string, int> cnt;
        for (int ph = 0; ph < n_phases_; ++ph) {
            auto& v = late[phase_names_[ph]];
            v.resize(G, 0.0);
            for (size_t b = 0; b < G; ++b) v[b] += block_late_ns_[ph * G + b] / traced_steps_;
            ++cnt[phase_names_[ph]];
        }
        o << ",\"block_lateness\":[";
        bool f2 = true;
        for (auto& kv : late) {
            std::vector<size_t> idx(G);
            for (size_t b = 0; b < G; ++b) idx[b] = b;
            std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return kv.second[a] > kv.second[b]; });
            double mean = 0.0;
            for (size_t b = 0; b < G; ++b) mean += kv.second[b];
            mean /= static_cast<double>(G) * cnt[kv.first];
            if (!f2) o << ",";
            f2 = false;
            double bar = 0.0;
            for (int ph = 0; ph < n_phases_; ++ph)
                if (phase_names_[ph] == kv.first) bar += barrier_ns_[ph] / traced_steps_;
            o << "{\"name\":\"" << kv.first << "\",\"mean_us\":" << mean / 1000.0
              << ",\"last_done_to_next_start_us\":" << bar / cnt[kv.first] / 1000.0 << ",\"latest\":[";
            for (size_t k = 0; k < 6 && k < G; ++k)
                o << (k ? "," : "") << "[" << idx[k] << "," << kv.second[idx[k]] / cnt[kv.first] / 1000.0 << "]";
            o << "]}";
        }
        o << "]";
    }
    o << "}";
    return o.str();
}

unsigned DeviceModel::device_errors() {
    unsigned v = 0;
    if (cudaMemcpyAsync(h_err_, d_err_, sizeof v, cudaMemcpyDeviceToHost, stream_) == cudaSuccess &&
        cudaStreamSynchronize(stream_) == cudaSuccess)
        v = *h_err_;
    return v;
}

void DeviceModel::clear_device_errors() {
    // The error word, the step kernel's grid-barrier counter and the merge counters of the
    // argmax and attention phases, on the session stream.
    cudaMemsetAsync(d_err_, 0, sizeof(unsigned), stream_);
    cudaMemsetAsync(d_grid_bar_, 0, sizeof(unsigned), stream_);
    cudaMemsetAsync(d_arg_counter_, 0, sizeof(unsigned), stream_);
    cudaMemsetAsync(d_attn_counters_, 0, sizeof(unsigned) * static_cast<size_t>(d_.kv_heads), stream_);
}

bool DeviceModel::check_device_errors(const char* what, std::string* error) {
    const unsigned v = device_errors();
    if (v == 0) return true;
    // Report once, then clear, so that the session can be reset and used again.
    clear_device_errors();
    cudaStreamSynchronize(stream_);
    std::string why;
    if (v & kErrBarrierTimeout) why += "a bounded device wait ran out of time";
    if (v & kErrBadShape) why += std::string(why.empty() ? "" : "; ") + "a kernel saw an unsupported configuration";
    if (v & kErrAttnIndex)
        why += std::string(why.empty() ? "" : "; ") + "an attention bounds check failed (access skipped)";
    *error = std::string(what) + " failed on the device (error word " + std::to_string(v) + "): " + why;
    return false;
}

}  // namespace xqb
