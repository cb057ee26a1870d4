// Tensor-parallel decode of one sequence over W GPUs: one process per GPU, NCCL between them.
// Each rank holds a slice of every matrix:
//   * column (output-row) slices of the projections that feed per-head work: attention q (with
//     its gate rows), k, v by query / kv head; the DeltaNet in_proj by key / value head (its q,
//     k, v conv channels, z, a, b rows); MLP gate and up by intermediate row;
//   * row (K) slices of the matrices that consume them: o_proj, out_proj and down, whose partial
//     outputs are summed across ranks by an NCCL all-reduce before the residual add;
//   * a vocabulary slice of lm_head: each rank's (max, lowest index) over its rows, gathered
//     and reduced with the reference's tie rule (gemvW4A16ArgmaxNeon, xq_gemv_w4a16_neon.cpp:
//     315-318: the first maximum wins).
// The recurrent and convolution states, the KV cache and every per-head operation stay local;
// norms, embeddings and the residual stream are replicated. Two all-reduces of `hidden` floats
// per layer and one 8-byte all-gather per token cross NVLink. The per-op kernels and the
// small-M tensor-core GEMM are those of batched decode; a step (sample, then the forward of the
// sampled token, CustomModel::decodeOne, custom_model.cpp:1340-1356) is one CUDA graph with the
// NCCL calls captured in it. NCCL is resolved at run time (dlopen), so the library loads on
// hosts without it and shares the process's NCCL when one is already loaded.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "../../include/xqwen35.h"
#include "model.hpp"
#include "ops.cuh"
#include "prefill_gemm.hpp"
#include "prefill_ops.hpp"

namespace xqb {

// The cross-rank argmax rule: a larger value wins, equal values go to the lower index, NaN
// never wins (every comparison with it is false).
__host__ __device__ inline bool tp_better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

struct TpPlan {
    int world = 1, rank = 0;
    int q0 = 0, q1 = 0;    // query heads (full attention)
    int kv0 = 0, kv1 = 0;  // kv heads
    int k0 = 0, k1 = 0;    // DeltaNet key heads
    int v0 = 0, v1 = 0;    // DeltaNet value heads
    int i0 = 0, i1 = 0;    // MLP intermediate rows
    int t0 = 0, t1 = 0;    // vocabulary rows of lm_head
};

// The shard of rank `rank` of `world`; false (error set) when the model does not split evenly.
bool tp_plan(const ModelDims& d, int world, int rank, TpPlan* p, std::string* err) {
    if (world < 1 || rank < 0 || rank >= world) {
        *err = "tensor parallel: need 0 <= rank < world";
        return false;
    }
    auto fail = [&](const std::string& m) {
        *err = "tensor parallel over " + std::to_string(world) + " GPUs: " + m;
        return false;
    };
    if (d.heads % world != 0) return fail("query heads do not divide");
    if (d.lk_heads % world != 0 || d.lv_heads % world != 0) return fail("DeltaNet heads do not divide");
    if (d.inter % world != 0 || (d.inter / world) % 512 != 0) return fail("the MLP width does not split into 512-column slices");
    if ((d.heads / world * d.head_dim) % 512 != 0 || (d.lv_heads / world * d.lv_hd) % 512 != 0)
        return fail("the attention output width does not split into 512-column slices");
    p->world = world;
    p->rank = rank;
    const int qn = d.heads / world;
    p->q0 = rank * qn;
    p->q1 = p->q0 + qn;
    if (world <= d.kv_heads) {
        if (d.kv_heads % world != 0) return fail("kv heads do not divide");
        p->kv0 = rank * (d.kv_heads / world);
        p->kv1 = p->kv0 + d.kv_heads / world;
    } else {
        // more ranks than kv heads: each rank's query heads share one kv head, which is
        // replicated on the ranks that use it
        const int group = d.heads / d.kv_heads;
        if (world % d.kv_heads != 0 || group % qn != 0) return fail("kv heads cannot be shared evenly");
        p->kv0 = p->q0 / group;
        p->kv1 = p->kv0 + 1;
    }
    p->k0 = rank * (d.lk_heads / world);
    p->k1 = p->k0 + d.lk_heads / world;
    p->v0 = rank * (d.lv_heads / world);
    p->v1 = p->v0 + d.lv_heads / world;
    p->i0 = rank * (d.inter / world);
    p->i1 = p->i0 + d.inter / world;
    p->t0 = static_cast<int>(static_cast<long long>(rank) * d.vocab / world);
    p->t1 = static_cast<int>(static_cast<long long>(rank + 1) * d.vocab / world);
    return true;
}

namespace {

// NCCL entry points, resolved once.
struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static const NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        a.ok = a.get_unique_id && a.init_rank && a.all_reduce && a.all_gather && a.destroy && a.error_string;
        return a;
    }();
    return api;
}

std::string nccl_error(ncclResult_t r) {
    const NcclApi& n = nccl();
    return n.error_string ? n.error_string(r) : ("NCCL error " + std::to_string(static_cast<int>(r)));
}

// Rows [r0, r1) of a matrix.
HostMatrix slice_rows(const HostMatrix& m, int r0, int r1) {
    HostMatrix o;
    o.rows = r1 - r0;
    o.cols = m.cols;
    o.group = m.group;
    o.version = m.version;
    const size_t rb = static_cast<size_t>(m.cols + 1) / 2, gpr = static_cast<size_t>((m.cols + m.group - 1) / m.group);
    o.packed.assign(m.packed.begin() + r0 * rb, m.packed.begin() + r1 * rb);
    o.scales.assign(m.scales.begin() + r0 * gpr, m.scales.begin() + r1 * gpr);
    o.zeros.assign(m.zeros.begin() + r0 * gpr, m.zeros.begin() + r1 * gpr);
    return o;
}

// Columns [c0, c1) of a matrix (multiples of the group size).
HostMatrix slice_cols(const HostMatrix& m, int c0, int c1) {
    HostMatrix o;
    o.rows = m.rows;
    o.cols = c1 - c0;
    o.group = m.group;
    o.version = m.version;
    const size_t rb = static_cast<size_t>(m.cols) / 2, gpr = static_cast<size_t>(m.cols / m.group);
    const size_t ob = static_cast<size_t>(o.cols) / 2, og = static_cast<size_t>(o.cols / m.group);
    o.packed.resize(static_cast<size_t>(m.rows) * ob);
    o.scales.resize(static_cast<size_t>(m.rows) * og);
    o.zeros.resize(static_cast<size_t>(m.rows) * og);
    for (int r = 0; r < m.rows; ++r) {
        std::memcpy(o.packed.data() + r * ob, m.packed.data() + r * rb + c0 / 2, ob);
        for (size_t g = 0; g < og; ++g) {
            o.scales[r * og + g] = m.scales[r * gpr + c0 / m.group + g];
            o.zeros[r * og + g] = m.zeros[r * gpr + c0 / m.group + g];
        }
    }
    return o;
}

// x = rmsnorm(H (+= P first when P is given)) * w as a bf16 pair; one block of 1024 threads, each
// holding up to two float4s of the row in registers (hidden <= 8192, a multiple of 4), so the
// row is read in one memory round trip.
__global__ void __launch_bounds__(1024) tp_add_norm_split_kernel(float* H, const float* P, const float* w, int n, float eps,
                                                                 __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_launch_dependents();  // programmatic dependent launch: inputs only after the
    pdl_wait();               // previous kernel has finished
    constexpr int kV = 2;
    __shared__ float ws[32];
    const int n4 = n >> 2;
    float4* h4 = reinterpret_cast<float4*>(H);
    const float4* p4 = reinterpret_cast<const float4*>(P);
    float4 v[kV];
#pragma unroll
    for (int i = 0; i < kV; ++i) {
        const int k = threadIdx.x + i * 1024;
        v[i] = k < n4 ? h4[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (P && k < n4) {
            const float4 q = p4[k];
            v[i].x += q.x;
            v[i].y += q.y;
            v[i].z += q.z;
            v[i].w += q.w;
            h4[k] = v[i];
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kV; ++i) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += ws[i];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
    for (int i = 0; i < kV; ++i) {
        const int k = threadIdx.x + i * 1024;
        if (k >= n4) break;
        const float4 g = w4[k];
        const float o[4] = {v[i].x * inv * g.x, v[i].y * inv * g.y, v[i].z * inv * g.z, v[i].w * inv * g.w};
        __nv_bfloat16 hh[4], ll[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            hh[j] = __float2bfloat16_rn(o[j]);
            ll[j] = __float2bfloat16_rn(o[j] - __bfloat162float(hh[j]));
        }
        *reinterpret_cast<uint2*>(hi + 4 * k) = *reinterpret_cast<const uint2*>(hh);
        *reinterpret_cast<uint2*>(lo + 4 * k) = *reinterpret_cast<const uint2*>(ll);
    }
}

__global__ void tp_add_kernel(float* H, const float* P, int n) {
    pdl_launch_dependents();  // programmatic dependent launch: inputs only after the
    pdl_wait();               // previous kernel has finished
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < n) H[k] += P[k];
}

// (max, lowest index) of this rank's logits, the index offset to the global vocabulary; the
// pair is written as two 32-bit words (value bits, index) for the all-gather.
__global__ void __launch_bounds__(1024) tp_local_argmax_kernel(const float* logits, int n, int offset, int* pair) {
    pdl_launch_dependents();  // programmatic dependent launch: inputs only after the
    pdl_wait();               // previous kernel has finished
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        if (tp_better(logits[k], k, bv, bi)) {
            bv = logits[k];
            bi = k;
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (tp_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (tp_better(sv[w], si[w], bv, bi)) {
                bv = sv[w];
                bi = si[w];
            }
        pair[0] = __float_as_int(bv);
        pair[1] = bi == INT_MAX ? INT_MAX : bi + offset;
    }
}

// The global token from the gathered pairs (rank order), then the decode bookkeeping:
// pos = next++, token into the ring.
__global__ void tp_pick_kernel(const int* pairs, int world, int* token, int* pos, int* next, int* ring, int* ctr,
                               int ring_steps) {
    pdl_launch_dependents();  // programmatic dependent launch: inputs only after the
    pdl_wait();               // previous kernel has finished
    if (threadIdx.x != 0) return;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int r = 0; r < world; ++r)
        if (tp_better(__int_as_float(pairs[2 * r]), pairs[2 * r + 1], bv, bi)) {
            bv = __int_as_float(pairs[2 * r]);
            bi = pairs[2 * r + 1];
        }
    const int t = bi == INT_MAX ? 0 : bi;
    *token = t;
    *pos = *next;
    *next = *next + 1;
    ring[*ctr % ring_steps] = t;
    *ctr = *ctr + 1;
}

class TpModel {
public:
    ~TpModel();
    bool create(const std::string& dir, const Options& opts, int world, int rank, const ncclUniqueId& id,
                int max_context, std::string* err);
    bool prefill(const int32_t* ids, size_t n, std::string* err);
    bool decode_steps(size_t steps, int32_t* tokens, double* device_ms, std::string* err);
    bool hidden(float* out, size_t cap, size_t* n, std::string* err);

private:
    struct Layer {
        bool full = false;
        DevMatrix in_proj, out_proj, gate_up, down;
        float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
        float *lin_norm = nullptr, *conv_w = nullptr, *a_log = nullptr, *dt_bias = nullptr;
        float *conv_state = nullptr, *rec_state = nullptr;
        void *kc = nullptr, *vc = nullptr;
    };
    template <typename T>
    bool alloc(T** p, size_t count, std::string* err) {
        *p = nullptr;
        if (cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(1, count) * sizeof(T)) != cudaSuccess) {
            *err = "tensor parallel: device allocation failed";
            return false;
        }
        allocs_.push_back(*p);
        return true;
    }
    bool upload_vec(float** dst, const std::vector<float>& v, std::string* err);
    bool upload_parts(std::vector<HostMatrix>& parts, bool interleave, DevMatrix* out, std::string* err);
    bool load_layer(const std::string& dir, int i, Layer* L, std::string* err);
    bool enqueue_forward(cudaStream_t s, std::string* err);
    bool enqueue_sample(cudaStream_t s, std::string* err);
    bool capture(bool with_sample, cudaGraphExec_t* out, std::string* err);
    bool sync_check(std::string* err);

    ModelDims d_;
    Options opts_;
    TpPlan plan_;
    int n_layers_ = 0, cap_ = 0;
    int nq_ = 0, nkv_ = 0, nk_ = 0, nv_ = 0, conv_dim_ = 0, lv_dim_ = 0, inter_ = 0, vocab_ = 0;
    std::vector<Layer> layers_;
    DevMatrix lm_head_;
    float* final_norm_ = nullptr;
    uint16_t* emb_ = nullptr;
    float *H_ = nullptr, *P_ = nullptr, *Y_ = nullptr, *conv_ = nullptr, *O_ = nullptr, *logits_ = nullptr;
    float *hid_ = nullptr, *attn_part_ = nullptr;
    unsigned* attn_counters_ = nullptr;
    __nv_bfloat16 *xhi_ = nullptr, *xlo_ = nullptr;
    float2* rope_ = nullptr;
    int *tok_ = nullptr, *pos_ = nullptr, *next_ = nullptr, *ring_ = nullptr, *ring_ctr_ = nullptr, *pair_ = nullptr,
        *pairs_ = nullptr;
    unsigned* err_ = nullptr;
    int ring_steps_ = 4096;
    size_t ring_count_ = 0;
    bool prefilled_ = false;
    std::vector<void*> allocs_;
    std::vector<DevMatrix*> mats_;
    cudaStream_t stream_ = nullptr;
    ncclComm_t comm_ = nullptr;
    cudaGraphExec_t g_forward_ = nullptr, g_step_ = nullptr;
};

TpModel::~TpModel() {
    cudaSetDevice(opts_.device);
    if (stream_) cudaStreamSynchronize(stream_);
    // graphs that hold NCCL calls go before the communicator
    if (g_forward_) cudaGraphExecDestroy(g_forward_);
    if (g_step_) cudaGraphExecDestroy(g_step_);
    if (comm_) nccl().destroy(comm_);
    for (DevMatrix* m : mats_) free_matrix(m);
    for (void* p : allocs_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
}

bool TpModel::upload_vec(float** dst, const std::vector<float>& v, std::string* err) {
    if (!alloc(dst, v.size(), err)) return false;
    if (cudaMemcpy(*dst, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        *err = "tensor parallel: upload failed";
        return false;
    }
    return true;
}

bool TpModel::upload_parts(std::vector<HostMatrix>& parts, bool interleave, DevMatrix* out, std::string* err) {
    std::vector<const HostMatrix*> ptrs;
    for (const HostMatrix& m : parts) ptrs.push_back(&m);
    std::vector<uint8_t> host;
    if (!build_matrix_rows(ptrs, interleave, out, &host, err, /*narrow=*/true)) return false;
    if (out->kind != 0) {
        *err = "tensor parallel decode needs symmetric W4 matrices (zero 8, fp16 scales)";
        return false;
    }
    if (!upload_matrix_rows(host, out, err)) return false;
    mats_.push_back(out);
    return true;
}

bool TpModel::load_layer(const std::string& dir, int i, Layer* L, std::string* err) {
    const ModelDims& d = d_;
    const TpPlan& p = plan_;
    const std::string pre = dir + "/layers_" + std::to_string(i) + "_";
    auto read = [&](const std::string& name, int rows, int cols, HostMatrix* m) {
        if (!read_xq4_file(pre + name, m, err)) return false;
        if (m->rows != rows || m->cols != cols || m->group != 64) {
            *err = "tensor parallel: unexpected shape or group for " + name;
            return false;
        }
        return true;
    };
    std::vector<float> v;
    L->full = file_exists(pre + "self_attn_q_proj_weight.xq4");
    if (L->full) {
        const int hd = d.head_dim;
        HostMatrix q, k, vm, o;
        if (!read("self_attn_q_proj_weight.xq4", 2 * d.heads * hd, d.hidden, &q) ||
            !read("self_attn_k_proj_weight.xq4", d.kv_heads * hd, d.hidden, &k) ||
            !read("self_attn_v_proj_weight.xq4", d.kv_heads * hd, d.hidden, &vm) ||
            !read("self_attn_o_proj_weight.xq4", d.hidden, d.heads * hd, &o))
            return false;
        std::vector<HostMatrix> in{slice_rows(q, p.q0 * 2 * hd, p.q1 * 2 * hd), slice_rows(k, p.kv0 * hd, p.kv1 * hd),
                                   slice_rows(vm, p.kv0 * hd, p.kv1 * hd)};
        std::vector<HostMatrix> out{slice_cols(o, p.q0 * hd, p.q1 * hd)};
        if (!upload_parts(in, false, &L->in_proj, err) || !upload_parts(out, false, &L->out_proj, err)) return false;
        if (!read_vec(pre + "self_attn_q_norm_weight.f32", hd, &v, err)) return false;
        add_one(&v);
        if (!upload_vec(&L->q_norm, v, err)) return false;
        if (!read_vec(pre + "self_attn_k_norm_weight.f32", hd, &v, err)) return false;
        add_one(&v);
        if (!upload_vec(&L->k_norm, v, err)) return false;
        const size_t elem = opts_.kv_fp16 ? 2 : 4;
        const size_t kv = static_cast<size_t>(cap_) * nkv_ * hd * elem;
        uint8_t *kc = nullptr, *vc = nullptr;
        if (!alloc(&kc, kv, err) || !alloc(&vc, kv, err)) return false;
        L->kc = kc;
        L->vc = vc;
    } else {
        const int dk = d.lk_hd, dv = d.lv_hd, nk = d.lk_heads;
        HostMatrix qkv, z, a, b, o;
        if (!read("linear_attn_in_proj_qkv_weight.xq4", d.conv_dim, d.hidden, &qkv) ||
            !read("linear_attn_in_proj_z_weight.xq4", d.lv_dim, d.hidden, &z) ||
            !read("linear_attn_in_proj_a_weight.xq4", d.lv_heads, d.hidden, &a) ||
            !read("linear_attn_in_proj_b_weight.xq4", d.lv_heads, d.hidden, &b) ||
            !read("linear_attn_out_proj_weight.xq4", d.hidden, d.lv_dim, &o))
            return false;
        // conv channels [q | k | v] keep their order: this rank's key heads' q, k and its value
        // heads' v, then z, a, b of its value heads
        std::vector<HostMatrix> in{slice_rows(qkv, p.k0 * dk, p.k1 * dk),
                                   slice_rows(qkv, nk * dk + p.k0 * dk, nk * dk + p.k1 * dk),
                                   slice_rows(qkv, 2 * nk * dk + p.v0 * dv, 2 * nk * dk + p.v1 * dv),
                                   slice_rows(z, p.v0 * dv, p.v1 * dv), slice_rows(a, p.v0, p.v1),
                                   slice_rows(b, p.v0, p.v1)};
        std::vector<HostMatrix> out{slice_cols(o, p.v0 * dv, p.v1 * dv)};
        if (!upload_parts(in, false, &L->in_proj, err) || !upload_parts(out, false, &L->out_proj, err)) return false;
        if (!read_vec(pre + "linear_attn_conv1d_weight.f32", d.conv_dim * d.conv_k, &v, err)) return false;
        std::vector<float> cw;
        auto take = [&](int c0, int c1) { cw.insert(cw.end(), v.begin() + c0 * d.conv_k, v.begin() + c1 * d.conv_k); };
        take(p.k0 * dk, p.k1 * dk);
        take(nk * dk + p.k0 * dk, nk * dk + p.k1 * dk);
        take(2 * nk * dk + p.v0 * dv, 2 * nk * dk + p.v1 * dv);
        if (!upload_vec(&L->conv_w, cw, err)) return false;
        if (!read_vec(pre + "linear_attn_A_log.f32", d.lv_heads, &v, err)) return false;
        if (!upload_vec(&L->a_log, std::vector<float>(v.begin() + p.v0, v.begin() + p.v1), err)) return false;
        if (!read_vec(pre + "linear_attn_dt_bias.f32", d.lv_heads, &v, err)) return false;
        if (!upload_vec(&L->dt_bias, std::vector<float>(v.begin() + p.v0, v.begin() + p.v1), err)) return false;
        if (!read_vec(pre + "linear_attn_norm_weight.f32", dv, &v, err)) return false;
        if (!upload_vec(&L->lin_norm, v, err)) return false;
        if (!alloc(&L->conv_state, static_cast<size_t>(conv_dim_) * (d.conv_k - 1), err) ||
            !alloc(&L->rec_state, static_cast<size_t>(nv_) * dk * dv, err))
            return false;
    }
    HostMatrix g, u, dn;
    if (!read("mlp_gate_proj_weight.xq4", d.inter, d.hidden, &g) || !read("mlp_up_proj_weight.xq4", d.inter, d.hidden, &u) ||
        !read("mlp_down_proj_weight.xq4", d.hidden, d.inter, &dn))
        return false;
    std::vector<HostMatrix> gu{slice_rows(g, p.i0, p.i1), slice_rows(u, p.i0, p.i1)};
    std::vector<HostMatrix> down{slice_cols(dn, p.i0, p.i1)};
    if (!upload_parts(gu, true, &L->gate_up, err) || !upload_parts(down, false, &L->down, err)) return false;
    if (!read_vec(pre + "input_layernorm_weight.f32", d.hidden, &v, err)) return false;
    add_one(&v);
    if (!upload_vec(&L->in_norm, v, err)) return false;
    if (!read_vec(pre + "post_attention_layernorm_weight.f32", d.hidden, &v, err)) return false;
    add_one(&v);
    return upload_vec(&L->post_norm, v, err);
}

bool TpModel::create(const std::string& dir, const Options& opts, int world, int rank, const ncclUniqueId& id,
                     int max_context, std::string* err) {
    opts_ = opts;
    cap_ = max_context;
    const std::string manifest = read_small_file(dir + "/xqwen35_manifest.json");
    if (manifest.empty()) {
        *err = "missing xqwen35_manifest.json";
        return false;
    }
    d_ = parse_manifest(manifest, &n_layers_);
    const ModelDims& d = d_;
    if (max_context < 2 || !tp_plan(d, world, rank, &plan_, err)) {
        if (max_context < 2) *err = "tensor parallel: max_context must be >= 2";
        return false;
    }
    if (d.head_dim != kAttnThreads || d.rotary_dim != 64 || d.lk_hd != 128 || d.lv_hd % kDeltaCols != 0 ||
        d.conv_k != 4 || d.hidden % 512 != 0 || d.hidden > 8192) {
        *err = "tensor parallel decode serves the fused shapes only (head_dim 256, rotary 64, DeltaNet key dim 128, "
               "conv kernel 4, hidden a multiple of 512 up to 8192)";
        return false;
    }
    if (!nccl().ok) {
        *err = "tensor parallel: NCCL (libnccl.so.2) could not be loaded";
        return false;
    }
    nq_ = plan_.q1 - plan_.q0;
    nkv_ = plan_.kv1 - plan_.kv0;
    nk_ = plan_.k1 - plan_.k0;
    nv_ = plan_.v1 - plan_.v0;
    conv_dim_ = 2 * nk_ * d.lk_hd + nv_ * d.lv_hd;
    lv_dim_ = nv_ * d.lv_hd;
    inter_ = plan_.i1 - plan_.i0;
    vocab_ = plan_.t1 - plan_.t0;
    if (nq_ / nkv_ > kAttnMaxGroup || attention_smem_bytes(nq_, nkv_, d.head_dim, cap_) > 200 * 1024) {
        *err = "tensor parallel: attention shard or context too large";
        return false;
    }
    if (cudaSetDevice(opts_.device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) {
        *err = "tensor parallel: device or stream set-up failed";
        return false;
    }
    layers_.resize(static_cast<size_t>(n_layers_));
    for (int i = 0; i < n_layers_; ++i)
        if (!load_layer(dir, i, &layers_[static_cast<size_t>(i)], err)) return false;
    {
        HostMatrix lm;
        if (!read_xq4_file(dir + "/lm_head_weight.xq4", &lm, err)) return false;
        if (lm.rows != d.vocab || lm.cols != d.hidden || lm.group != 64) {
            *err = "tensor parallel: unexpected lm_head shape";
            return false;
        }
        std::vector<HostMatrix> parts{slice_rows(lm, plan_.t0, plan_.t1)};
        if (!upload_parts(parts, false, &lm_head_, err)) return false;
    }
    std::vector<float> v;
    if (!read_vec(dir + "/norm_weight.f32", d.hidden, &v, err)) return false;
    add_one(&v);
    if (!upload_vec(&final_norm_, v, err)) return false;
    {
        const size_t count = static_cast<size_t>(d.vocab) * d.hidden;
        std::vector<uint16_t> emb(count);
        std::ifstream in(dir + "/embeddings_bf16.bin", std::ios::binary);
        in.read(reinterpret_cast<char*>(emb.data()), static_cast<std::streamsize>(count * 2));
        if (in.gcount() != static_cast<std::streamsize>(count * 2)) {
            *err = "short embeddings_bf16.bin";
            return false;
        }
        if (!alloc(&emb_, count, err) ||
            cudaMemcpy(emb_, emb.data(), count * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
            *err = "tensor parallel: embedding upload failed";
            return false;
        }
    }
    int ymax = vocab_;
    for (const Layer& L : layers_) ymax = std::max({ymax, L.in_proj.rows, L.gate_up.rows});
    const int kmax = std::max({d.hidden, lv_dim_, nq_ * d.head_dim, inter_});
    if (!alloc(&H_, d.hidden, err) || !alloc(&P_, d.hidden, err) || !alloc(&Y_, ymax, err) ||
        !alloc(&conv_, std::max(1, conv_dim_), err) || !alloc(&O_, std::max(1, lv_dim_), err) ||
        !alloc(&logits_, vocab_, err) || !alloc(&hid_, d.hidden, err) || !alloc(&xhi_, kmax, err) ||
        !alloc(&xlo_, kmax, err) ||
        !alloc(&attn_part_, static_cast<size_t>(nkv_) * kAttnSplits * (nq_ / nkv_) * (d.head_dim + 2), err) ||
        !alloc(&attn_counters_, nkv_, err) || !alloc(&tok_, 1, err) || !alloc(&pos_, 1, err) ||
        !alloc(&next_, 1, err) || !alloc(&ring_, ring_steps_, err) || !alloc(&ring_ctr_, 1, err) ||
        !alloc(&pair_, 2, err) || !alloc(&pairs_, 2 * world, err) || !alloc(&err_, 1, err))
        return false;
    std::vector<float2> rope;
    rope_table(0, cap_, d.rotary_dim, d.theta, &rope);
    if (!alloc(&rope_, rope.size(), err) ||
        cudaMemcpy(rope_, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(attn_counters_, 0, sizeof(unsigned) * nkv_) != cudaSuccess ||
        cudaMemset(ring_ctr_, 0, sizeof(int)) != cudaSuccess || cudaMemset(next_, 0, sizeof(int)) != cudaSuccess ||
        cudaMemset(err_, 0, sizeof(unsigned)) != cudaSuccess) {
        *err = "tensor parallel: set-up copies failed";
        return false;
    }
    const ncclResult_t r = nccl().init_rank(&comm_, world, id, rank);
    if (r != ncclSuccess) {
        comm_ = nullptr;
        *err = "tensor parallel: ncclCommInitRank failed: " + nccl_error(r);
        return false;
    }
    return true;
}

// Forward of the token in tok_ at position pos_: the residual stream ends in H_.
bool TpModel::enqueue_forward(cudaStream_t s, std::string* err) {
    const ModelDims& d = d_;
    auto ok = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        *err = std::string("tensor parallel: ") + what + ": " + cudaGetErrorString(e);
        return false;
    };
    auto gemm = [&](const DevMatrix& m, float* y, int ldy) {
        if (launch_prefill_gemm(m, xhi_, xlo_, 1, y, ldy, kPgOutF32, err_, 148, s)) return true;
        *err = std::string("tensor parallel: ") + last_error();
        return false;
    };
    auto all_reduce = [&](float* buf) {
        const ncclResult_t r = nccl().all_reduce(buf, buf, static_cast<size_t>(d.hidden), ncclFloat, ncclSum, comm_, s);
        if (r == ncclSuccess) return true;
        *err = "tensor parallel: ncclAllReduce failed: " + nccl_error(r);
        return false;
    };
    auto norm = [&](const float* P, const float* w) {
        launch_ex(tp_add_norm_split_kernel, dim3(1), dim3(1024), 0, s, pdl_enabled(), H_, P, w, d.hidden, d.eps, xhi_, xlo_);
        return ok(cudaGetLastError(), "norm");
    };
    if (!ok(prefill_embed(tok_, emb_, H_, 1, d.hidden, d.vocab, s), "embedding")) return false;
    for (size_t l = 0; l < layers_.size(); ++l) {
        const Layer& L = layers_[l];
        if (!norm(l == 0 ? nullptr : P_, L.in_norm)) return false;  // + the previous layer's MLP output
        const int ldy = L.in_proj.rows;
        if (!gemm(L.in_proj, Y_, ldy)) return false;
        if (!L.full) {
            // in_proj shard rows: [q k v (conv_dim_) | z (lv_dim_) | a (nv_) | b (nv_)]
            if (!ok(prefill_conv(Y_, ldy, L.conv_w, L.conv_state, conv_, 1, conv_dim_, s), "conv") ||
                !ok(prefill_delta(conv_, conv_dim_, Y_, ldy, conv_dim_ + lv_dim_, L.a_log, L.dt_bias, L.rec_state, O_,
                                  lv_dim_, 1, nk_, nv_, d.lk_hd, d.lv_hd, s),
                    "gated delta") ||
                !ok(prefill_gated_norm(O_, lv_dim_, Y_, ldy, conv_dim_, L.lin_norm, nv_, d.lv_hd, d.eps, 1, xhi_, xlo_, s),
                    "gated norm"))
                return false;
        } else {
            AttnParams ap = {};
            ap.qkv = Y_;
            ap.q_norm = L.q_norm;
            ap.k_norm = L.k_norm;
            ap.k_cache = L.kc;
            ap.v_cache = L.vc;
            ap.capacity = cap_;
            ap.pos_ptr = pos_;
            ap.nq = nq_;
            ap.nkv = nkv_;
            ap.hd = d.head_dim;
            ap.rotary = d.rotary_dim;
            ap.theta = d.theta;
            ap.eps = d.eps;
            ap.rope = rope_;
            ap.rope_stride = d.rotary_dim / 2;
            ap.part = attn_part_;
            ap.counters = attn_counters_;
            ap.err = err_;
            if (!ok(launch_attention_batch(ap, opts_.kv_fp16, attention_smem_bytes(nq_, nkv_, d.head_dim, cap_), 1, ldy,
                                           0, xhi_, xlo_, s),
                    "attention"))
                return false;
        }
        if (!gemm(L.out_proj, P_, d.hidden) || !all_reduce(P_) || !norm(P_, L.post_norm) ||
            !gemm(L.gate_up, Y_, L.gate_up.rows) ||
            !ok(prefill_swiglu(Y_, L.gate_up.rows, inter_, 1, xhi_, xlo_, s), "swiglu") ||
            !gemm(L.down, P_, d.hidden) || !all_reduce(P_))
            return false;
    }
    launch_ex(tp_add_kernel, dim3((d.hidden + 255) / 256), dim3(256), 0, s, pdl_enabled(), H_, P_, d.hidden);
    return ok(cudaGetLastError(), "residual");
}

// Greedy sample from H_ (final norm, this rank's lm_head rows, argmax across ranks) into tok_,
// then pos_ = next_++.
bool TpModel::enqueue_sample(cudaStream_t s, std::string* err) {
    const ModelDims& d = d_;
    launch_ex(tp_add_norm_split_kernel, dim3(1), dim3(1024), 0, s, pdl_enabled(), H_, nullptr, final_norm_, d.hidden, d.eps, xhi_, xlo_);
    if (!launch_prefill_gemm(lm_head_, xhi_, xlo_, 1, logits_, vocab_, kPgOutF32, err_, 148, s)) {
        *err = std::string("tensor parallel: ") + last_error();
        return false;
    }
    launch_ex(tp_local_argmax_kernel, dim3(1), dim3(1024), 0, s, pdl_enabled(), logits_, vocab_, plan_.t0, pair_);
    const ncclResult_t r = nccl().all_gather(pair_, pairs_, 2, ncclInt32, comm_, s);
    if (r != ncclSuccess) {
        *err = "tensor parallel: ncclAllGather failed: " + nccl_error(r);
        return false;
    }
    launch_ex(tp_pick_kernel, dim3(1), dim3(32), 0, s, pdl_enabled(), pairs_, plan_.world, tok_, pos_, next_, ring_, ring_ctr_, ring_steps_);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("tensor parallel: sample: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

bool TpModel::capture(bool with_sample, cudaGraphExec_t* out, std::string* err) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed) != cudaSuccess) {
        *err = "tensor parallel: stream capture failed to start";
        return false;
    }
    const bool ok = (!with_sample || enqueue_sample(stream_, err)) && enqueue_forward(stream_, err);
    const cudaError_t e = cudaStreamEndCapture(stream_, &g);
    if (!ok || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        if (ok) *err = std::string("tensor parallel: capture failed: ") + cudaGetErrorString(e);
        return false;
    }
    const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
        *out = nullptr;
        *err = std::string("tensor parallel: graph instantiation failed: ") + cudaGetErrorString(ie);
        return false;
    }
    return true;
}

bool TpModel::sync_check(std::string* err) {
    if (cudaStreamSynchronize(stream_) != cudaSuccess) {
        *err = "tensor parallel: step failed on the device";
        return false;
    }
    unsigned e = 0;
    cudaMemcpy(&e, err_, sizeof e, cudaMemcpyDeviceToHost);
    if (e) {
        cudaMemset(err_, 0, sizeof(unsigned));
        *err = "tensor parallel: a bounded device wait ran out or a kernel saw an unsupported configuration";
        return false;
    }
    return true;
}

// Token-serial prefill (the reference's prefill_kv_build order, custom_model.cpp:610-640): the
// forward graph per prompt token with its id and position written before each replay.
bool TpModel::prefill(const int32_t* ids, size_t n, std::string* err) {
    if (!ids || n == 0 || n + 1 > static_cast<size_t>(cap_)) {
        *err = "tensor parallel: empty prompt or prompt longer than the context";
        return false;
    }
    cudaSetDevice(opts_.device);
    if (!g_forward_ && !capture(false, &g_forward_, err)) return false;
    // a new prompt starts from zero recurrent and convolution states (KV rows are overwritten)
    for (const Layer& L : layers_)
        if (!L.full &&
            (cudaMemsetAsync(L.conv_state, 0, sizeof(float) * conv_dim_ * (d_.conv_k - 1), stream_) != cudaSuccess ||
             cudaMemsetAsync(L.rec_state, 0, sizeof(float) * nv_ * d_.lk_hd * d_.lv_hd, stream_) != cudaSuccess)) {
            *err = "tensor parallel: state reset failed";
            return false;
        }
    std::vector<int> host(2 * n);
    for (size_t i = 0; i < n; ++i) {
        host[2 * i] = ids[i];
        host[2 * i + 1] = static_cast<int>(i);
    }
    for (size_t i = 0; i < n; ++i) {
        if (cudaMemcpyAsync(tok_, &host[2 * i], sizeof(int), cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
            cudaMemcpyAsync(pos_, &host[2 * i + 1], sizeof(int), cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
            cudaGraphLaunch(g_forward_, stream_) != cudaSuccess) {
            *err = "tensor parallel: prefill launch failed";
            return false;
        }
    }
    const int np = static_cast<int>(n);
    if (cudaMemcpyAsync(next_, &np, sizeof(int), cudaMemcpyHostToDevice, stream_) != cudaSuccess) {
        *err = "tensor parallel: prefill launch failed";
        return false;
    }
    if (!sync_check(err)) return false;
    prefilled_ = true;
    return true;
}

bool TpModel::decode_steps(size_t steps, int32_t* tokens, double* device_ms, std::string* err) {
    if (!prefilled_) {
        *err = "tensor parallel: prefill first";
        return false;
    }
    if (steps == 0 || steps > static_cast<size_t>(ring_steps_)) {
        *err = "tensor parallel: 1 .. 4096 steps per call";
        return false;
    }
    cudaSetDevice(opts_.device);
    int next = 0;
    cudaMemcpy(&next, next_, sizeof(int), cudaMemcpyDeviceToHost);
    if (next + static_cast<int>(steps) > cap_) {
        *err = "tensor parallel: the steps would run past the context";
        return false;
    }
    if (!g_step_ && !capture(true, &g_step_, err)) return false;
    const size_t first = ring_count_;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, stream_);
    bool ok = true;
    for (size_t i = 0; i < steps && ok; ++i) ok = cudaGraphLaunch(g_step_, stream_) == cudaSuccess;
    cudaEventRecord(e1, stream_);
    const bool synced = sync_check(err);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (!ok) *err = "tensor parallel: graph launch failed";
    if (!ok || !synced) return false;
    ring_count_ += steps;
    if (device_ms) *device_ms = static_cast<double>(ms);
    if (tokens) {
        std::vector<int> ring(static_cast<size_t>(ring_steps_));
        cudaMemcpy(ring.data(), ring_, sizeof(int) * ring.size(), cudaMemcpyDeviceToHost);
        for (size_t i = 0; i < steps; ++i) tokens[i] = ring[(first + i) % static_cast<size_t>(ring_steps_)];
    }
    return true;
}

bool TpModel::hidden(float* out, size_t cap, size_t* n, std::string* err) {
    if (n) *n = static_cast<size_t>(d_.hidden);
    if (!out) return true;
    if (cap < static_cast<size_t>(d_.hidden)) {
        *err = "buffer too small";
        return false;
    }
    cudaSetDevice(opts_.device);
    rmsnorm_kernel<<<1, 1024, 0, stream_>>>(H_, final_norm_, d_.hidden, d_.eps, hid_);
    if (cudaMemcpyAsync(out, hid_, sizeof(float) * d_.hidden, cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess) {
        *err = "tensor parallel: hidden state copy failed";
        return false;
    }
    return true;
}

}  // namespace
}  // namespace xqb

struct xq_tp {
    xqb::TpModel m;
};

namespace {
xqb::Options tp_options(const xq_cuda_options* co) {
    xqb::Options o;
    if (co && co->struct_size >= sizeof(xq_cuda_options)) {
        o.device = co->device;
        o.kv_fp16 = co->kv_fp16 != 0;
    }
    if (const char* v = std::getenv("XQ_CUDA_DEVICE")) o.device = std::atoi(v);
    if (const char* v = std::getenv("XQ_KV_FP16")) o.kv_fp16 = std::atoi(v) != 0;
    return o;
}
}  // namespace

XQ_API xq_status xq_tp_unique_id(unsigned char* out, size_t cap) {
    if (!out || cap < sizeof(ncclUniqueId)) return XQ_ERR_INVALID_ARGUMENT;
    if (!xqb::nccl().ok) {
        xqb::set_last_error("tensor parallel: NCCL (libnccl.so.2) could not be loaded");
        return XQ_ERR_RUNTIME;
    }
    ncclUniqueId id;
    const ncclResult_t r = xqb::nccl().get_unique_id(&id);
    if (r != ncclSuccess) {
        xqb::set_last_error("ncclGetUniqueId failed: " + xqb::nccl_error(r));
        return XQ_ERR_RUNTIME;
    }
    std::memcpy(out, &id, sizeof id);
    return XQ_OK;
}

XQ_API xq_status xq_tp_create(const char* model_dir, const xq_cuda_options* cuda_options, int world, int rank,
                              const unsigned char* unique_id, int max_context, xq_tp** out) {
    if (!model_dir || !unique_id || !out) return XQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof id);
    auto* t = new xq_tp;
    std::string err;
    if (!t->m.create(model_dir, tp_options(cuda_options), world, rank, id, max_context, &err)) {
        xqb::set_last_error(err);
        delete t;
        return (world < 1 || rank < 0 || rank >= world || max_context < 2) ? XQ_ERR_INVALID_ARGUMENT : XQ_ERR_MODEL;
    }
    *out = t;
    return XQ_OK;
}

XQ_API void xq_tp_destroy(xq_tp* t) { delete t; }

XQ_API xq_status xq_tp_prefill(xq_tp* t, const int32_t* ids, size_t n) {
    if (!t || !ids || n == 0) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!t->m.prefill(ids, n, &err)) {
        xqb::set_last_error(err);
        return XQ_ERR_RUNTIME;
    }
    return XQ_OK;
}

XQ_API xq_status xq_tp_decode(xq_tp* t, size_t steps, int32_t* tokens, double* device_ms) {
    if (!t) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!t->m.decode_steps(steps, tokens, device_ms, &err)) {
        xqb::set_last_error(err);
        return err.find("prefill first") != std::string::npos ? XQ_ERR_NOT_READY : XQ_ERR_RUNTIME;
    }
    return XQ_OK;
}

XQ_API xq_status xq_tp_hidden_state(xq_tp* t, float* out, size_t cap, size_t* out_size) {
    if (!t) return XQ_ERR_INVALID_ARGUMENT;
    std::string err;
    if (!t->m.hidden(out, cap, out_size, &err)) {
        xqb::set_last_error(err);
        return err == "buffer too small" ? XQ_ERR_BUFFER_TOO_SMALL : XQ_ERR_RUNTIME;
    }
    return XQ_OK;
}

XQ_API xq_status xq_tp_plan(const char* model_dir, int world, int rank, char* json, size_t cap) {
    if (!model_dir || !json || cap == 0) return XQ_ERR_INVALID_ARGUMENT;
    const std::string manifest = xqb::read_small_file(std::string(model_dir) + "/xqwen35_manifest.json");
    if (manifest.empty()) {
        xqb::set_last_error("missing xqwen35_manifest.json");
        return XQ_ERR_MODEL;
    }
    int n_layers = 0;
    const xqb::ModelDims d = xqb::parse_manifest(manifest, &n_layers);
    xqb::TpPlan p;
    std::string err;
    if (!xqb::tp_plan(d, world, rank, &p, &err)) {
        xqb::set_last_error(err);
        return XQ_ERR_INVALID_ARGUMENT;
    }
    char buf[512];
    const int len = std::snprintf(buf, sizeof buf,
                                  "{\"world\":%d,\"rank\":%d,\"q_heads\":[%d,%d],\"kv_heads\":[%d,%d],\"k_heads\":[%d,%d],"
                                  "\"v_heads\":[%d,%d],\"inter\":[%d,%d],\"vocab\":[%d,%d]}",
                                  p.world, p.rank, p.q0, p.q1, p.kv0, p.kv1, p.k0, p.k1, p.v0, p.v1, p.i0, p.i1, p.t0,
                                  p.t1);
    if (len < 0 || static_cast<size_t>(len) + 1 > cap) return XQ_ERR_BUFFER_TOO_SMALL;
    std::memcpy(json, buf, static_cast<size_t>(len) + 1);
    return XQ_OK;
}

XQ_API xq_status xq_tp_argmax_combine(const float* values, const int32_t* indices, int n, int32_t* out) {
    if (!values || !indices || !out || n < 1) return XQ_ERR_INVALID_ARGUMENT;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int r = 0; r < n; ++r)
        if (xqb::tp_better(values[r], indices[r], bv, bi)) {
            bv = values[r];
            bi = indices[r];
        }
    *out = bi == INT_MAX ? 0 : bi;
    return XQ_OK;
}
