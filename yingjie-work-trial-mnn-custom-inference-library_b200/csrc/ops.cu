// Gated-DeltaNet state update, fused GQA decode attention, embedding and RMSNorm kernels,
// and their kernel-level C ABI entry points (xq_kernels.h).
#include <cuda_fp16.h>

#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/xq_kernels.h"
#include "gemv.hpp"
#include "ops.cuh"

namespace xqb {

// Transpose-reduce 16 per-lane values across a warp: lanes 2m and 2m+1 return the warp
// total of value m.
__device__ __forceinline__ float warp_reduce16(const float (&v)[16], int lane) {
    float a[8], b[4], c[2];
    bool h = lane & 16;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const float keep = h ? v[8 + m] : v[m];
        const float send = h ? v[m] : v[8 + m];
        a[m] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    h = lane & 8;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float keep = h ? a[4 + m] : a[m];
        const float send = h ? a[m] : a[4 + m];
        b[m] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    h = lane & 4;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const float keep = h ? b[2 + m] : b[m];
        const float send = h ? b[m] : b[2 + m];
        c[m] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    h = lane & 2;
    float d = (h ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, h ? c[0] : c[1], 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    return d;
}

// One block = one value head vh and kDeltaCols of its value columns; thread i = key row i.
// Per step (custom_model.cpp:1037-1095, ref_delta.cpp:8-41):
//   q, k <- l2-normalised (eps 1e-6 inside the sqrt); beta = sigmoid(b[vh]);
//   g = -exp(A_log[vh]) * softplus(a[vh] + dt_bias[vh]); S <- exp(g) S;
//   for each column j: delta_j = beta (v_j - sum_i S_ij k_i); S_ij += k_i delta_j;
//   o_j = sum_i S_ij q_i / sqrt(dk).
// Columns are independent, so the [dk x dv] state splits over blocks by column slices.
__global__ void __launch_bounds__(128) gated_delta_kernel(const DeltaParams p) {
    __shared__ float red[4][kDeltaCols];
    __shared__ float bc[kDeltaCols];
    __shared__ float nrm[2][4];
    const int vh = blockIdx.x;
    const int j0 = blockIdx.y * kDeltaCols;
    const int i = threadIdx.x;
    const int lane = i & 31, warp = i >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const int factor = max(1, p.nv / max(1, p.nk));
    const int kh = min(p.nk - 1, vh / factor);
    float q = p.conv[kh * p.dk + i];
    float k = p.conv[p.nk * p.dk + kh * p.dk + i];
    float sq = warp_sum(q * q), sk = warp_sum(k * k);
    if (lane == 0) {
        nrm[0][warp] = sq;
        nrm[1][warp] = sk;
    }
    __syncthreads();
    sq = (nrm[0][0] + nrm[0][1]) + (nrm[0][2] + nrm[0][3]);
    sk = (nrm[1][0] + nrm[1][1]) + (nrm[1][2] + nrm[1][3]);
    q *= 1.0f / sqrtf(sq + 1.0e-6f);
    k *= 1.0f / sqrtf(sk + 1.0e-6f);
    const float beta = dsigmoid(p.ab[p.nv + vh]);
    const float gate = -expf(p.a_log[vh]) * dsoftplus(p.ab[vh] + p.dt_bias[vh]);
    const float decay = expf(gate);

    float4* sp = reinterpret_cast<float4*>(p.state + (static_cast<size_t>(vh) * p.dk + i) * p.dv + j0);
    float s[kDeltaCols], t[kDeltaCols];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float4 v = sp[m];
        s[4 * m] = v.x;
        s[4 * m + 1] = v.y;
        s[4 * m + 2] = v.z;
        s[4 * m + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < kDeltaCols; ++j) {
        s[j] *= decay;
        t[j] = s[j] * k;
    }
    float r = warp_reduce16(t, lane);
    if ((lane & 1) == 0) red[warp][lane >> 1] = r;
    __syncthreads();
    if (i < kDeltaCols) bc[i] = (red[0][i] + red[1][i]) + (red[2][i] + red[3][i]);
    __syncthreads();
    const float* vv = p.conv + 2 * p.nk * p.dk + vh * p.dv + j0;
    const float scale = 1.0f / sqrtf(static_cast<float>(p.dk));
#pragma unroll
    for (int j = 0; j < kDeltaCols; ++j) {
        const float delta = beta * (vv[j] - bc[j]);
        s[j] += k * delta;
        t[j] = s[j] * q * scale;
    }
    r = warp_reduce16(t, lane);
    if ((lane & 1) == 0) red[warp][lane >> 1] = r;
#pragma unroll
    for (int m = 0; m < 4; ++m) sp[m] = make_float4(s[4 * m], s[4 * m + 1], s[4 * m + 2], s[4 * m + 3]);
    __syncthreads();
    if (i < kDeltaCols) p.out[vh * p.dv + j0 + i] = (red[0][i] + red[1][i]) + (red[2][i] + red[3][i]);
}

template <typename KV>
__device__ __forceinline__ float kv_ld(const KV* p);
template <>
__device__ __forceinline__ float kv_ld<float>(const float* p) {
    return __ldcg(p);
}
template <>
__device__ __forceinline__ float kv_ld<__half>(const __half* p) {
    return __half2float(__ldcg(p));
}
__device__ __forceinline__ void kv_st(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_st(__half* p, float v) { *p = __float2half_rn(v); }

// Head RMSNorm (applyHeadRms, custom_model.cpp:301-313: x *= inv * w) and partial NeoX
// RoPE (applyRopeVector, :351-370) on one head held as v[m] = x[lane + 32 m]. The rotated
// pairs (i, 32 + i), i < 32, are v[0], v[1] of lane i (rotary_dim = 64).
__device__ __forceinline__ void norm_rope_head(float (&v)[8], const float* w, int hd, float eps, int lane,
                                               const float2* rope_row) {
    float ss = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; ++m) ss += v[m] * v[m];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(hd) + eps);
#pragma unroll
    for (int m = 0; m < 8; ++m) v[m] *= inv * w[lane + 32 * m];
    const float2 cs = rope_row[lane];
    const float c = cs.x, s = cs.y;
    const float x0 = v[0], x1 = v[1];
    v[0] = x0 * c - x1 * s;
    v[1] = x1 * c + x0 * s;
}

// grid (nkv, kAttnSplits), block 256 (hd = 256, rotary_dim = 64, group <= 8).
// Split-K flash decode: each block scores positions [t0, t1) of one kv head for all its
// query heads, keeps (max, sum, unnormalised output) per head; the last block of a kv head
// merges the splits and applies the sigmoid output gate.
template <typename KV>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
    extern __shared__ float sm[];
    __shared__ float s_m[kAttnMaxGroup], s_l[kAttnMaxGroup];
    __shared__ int s_last;
    const int kh = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd;
    const int group = p.nq / p.nkv;
    const int cmax = (p.capacity + kAttnSplits - 1) / kAttnSplits;
    float* qs = sm;                  // [group][hd]
    float* sc = sm + group * hd;     // [group][cmax]
    KV* kc = static_cast<KV*>(p.k_cache);
    KV* vc = static_cast<KV*>(p.v_cache);

    pdl_launch_dependents();
    pdl_wait();
    const int pos = p.pos_ptr ? *p.pos_ptr : p.pos_const;
    const int L = pos + 1;
    const int chunk = (L + kAttnSplits - 1) / kAttnSplits;
    const int t0 = min(L, split * chunk);
    const int t1 = min(L, t0 + chunk);
    const int n = t1 - t0;
    const float2* rope_row = p.rope + static_cast<size_t>(p.rope_stride) * pos;

    if (warp < group) {  // query head kh*group + warp: [query | gate] split (custom_model.cpp:740-753)
        const float* src = p.qkv + static_cast<size_t>(kh * group + warp) * 2 * hd;
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = src[lane + 32 * m];
        norm_rope_head(v, p.q_norm, hd, p.eps, lane, rope_row);
#pragma unroll
        for (int m = 0; m < 8; ++m) qs[warp * hd + lane + 32 * m] = v[m];
    }
    if (pos >= t0 && pos < t1 && warp == kAttnThreads / 32 - 1) {
        // appendKv (custom_model.cpp:673-733): normed + rotated k and raw v at `pos`.
        const float* ks = p.qkv + static_cast<size_t>(p.nq) * 2 * hd + kh * hd;
        const float* vs = ks + static_cast<size_t>(p.nkv) * hd;
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = ks[lane + 32 * m];
        norm_rope_head(v, p.k_norm, hd, p.eps, lane, rope_row);
        KV* kd = kc + (static_cast<size_t>(pos) * p.nkv + kh) * hd;
        KV* vd = vc + (static_cast<size_t>(pos) * p.nkv + kh) * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            kv_st(kd + lane + 32 * m, v[m]);
            kv_st(vd + lane + 32 * m, vs[lane + 32 * m]);
        }
        __threadfence_block();
    }
    __syncthreads();

    // scores s = q . k / sqrt(hd) (custom_model.cpp:871-885)
    const float rs = sqrtf(static_cast<float>(hd));
    for (int t = t0 + warp; t < t1; t += kAttnThreads / 32) {
        const KV* kr = kc + (static_cast<size_t>(t) * p.nkv + kh) * hd;
        float kv[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) kv[m] = kv_ld(kr + lane + 32 * m);
        for (int g = 0; g < group; ++g) {
            float d = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; ++m) d += qs[g * hd + lane + 32 * m] * kv[m];
            d = warp_sum(d);
            if (lane == 0) sc[g * cmax + (t - t0)] = d / rs;
        }
    }
    __syncthreads();
    if (warp < group) {  // local max-subtracted exponentials (custom_model.cpp:890-905)
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[warp * cmax + j]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int j = lane; j < n; j += 32) {
            const float e = expf(sc[warp * cmax + j] - mx);
            sc[warp * cmax + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            s_m[warp] = mx;
            s_l[warp] = l;
        }
    }
    __syncthreads();
    float o[kAttnMaxGroup];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) o[g] = 0.0f;
    for (int j = 0; j < n; ++j) {  // V reduction (custom_model.cpp:910-928), thread = dim
        const float v = kv_ld(vc + (static_cast<size_t>(t0 + j) * p.nkv + kh) * hd + tid);
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g)
            if (g < group) o[g] += sc[g * cmax + j] * v;
    }
    float* pp = p.part + static_cast<size_t>(kh * kAttnSplits + split) * group * (hd + 2);
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g)
        if (g < group) pp[g * (hd + 2) + tid] = o[g];
    if (tid < group) {
        pp[tid * (hd + 2) + hd] = s_m[tid];
        pp[tid * (hd + 2) + hd + 1] = s_l[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&p.counters[kh], 1u) == kAttnSplits - 1) ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Merge the splits in parallel: (max, sum) of every (split, head) pair to shared memory,
    // one rescale weight per pair, then thread d sums its dimension over the splits.
    __shared__ float s_pm[kAttnSplits * kAttnMaxGroup], s_pl[kAttnSplits * kAttnMaxGroup];
    __shared__ float s_M[kAttnMaxGroup], s_invL[kAttnMaxGroup];
    const float* base = p.part + static_cast<size_t>(kh * kAttnSplits) * group * (hd + 2);
    if (tid < kAttnSplits * group) {
        const float* ps = base + tid * (hd + 2);  // tid = split * group + g
        s_pm[tid] = __ldcg(ps + hd);
        s_pl[tid] = __ldcg(ps + hd + 1);
    }
    __syncthreads();
    if (tid < group) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < kAttnSplits; ++s2) M = fmaxf(M, s_pm[s2 * group + tid]);
        float Ls = 0.0f;
        for (int s2 = 0; s2 < kAttnSplits; ++s2) Ls += s_pl[s2 * group + tid] * expf(s_pm[s2 * group + tid] - M);
        s_M[tid] = M;
        s_invL[tid] = Ls > 0.0f ? 1.0f / Ls : 0.0f;
    }
    __syncthreads();
    if (tid < kAttnSplits * group) s_pm[tid] = expf(s_pm[tid] - s_M[tid % group]);
    __syncthreads();
    for (int g = 0; g < group; ++g) {
        float O = 0.0f;
#pragma unroll 8
        for (int s2 = 0; s2 < kAttnSplits; ++s2) O += __ldcg(base + (s2 * group + g) * (hd + 2) + tid) * s_pm[s2 * group + g];
        const int qh = kh * group + g;
        const float gate = p.qkv[static_cast<size_t>(qh) * 2 * hd + hd + tid];
        p.out[qh * hd + tid] = (O * s_invL[g]) * dsigmoid(gate);  // output gate, custom_model.cpp:944-946
    }
    if (tid == 0) p.counters[kh] = 0u;
}

cudaError_t launch_attention(const AttnParams& p, bool kv_fp16, size_t smem, cudaStream_t s, bool pdl) {
    const dim3 grid(p.nkv, kAttnSplits), block(kAttnThreads);
    return kv_fp16 ? launch_ex(attention_kernel<__half>, grid, block, smem, s, pdl, p)
                   : launch_ex(attention_kernel<float>, grid, block, smem, s, pdl, p);
}

cudaError_t attention_init_device(int max_smem_bytes) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         max_smem_bytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attention_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_bytes);
}

void rope_table(int first, int count, int rotary, float theta, std::vector<float2>* out) {
    const int half = rotary / 2;
    out->resize(static_cast<size_t>(count) * half);
    for (int i = 0; i < half; ++i) {
        const float inv_freq = std::pow(theta, -static_cast<float>(2 * i) / static_cast<float>(rotary));
        for (int p = 0; p < count; ++p) {
            const float angle = static_cast<float>(first + p) * inv_freq;
            (*out)[static_cast<size_t>(p) * half + i] = make_float2(std::cos(angle), std::sin(angle));
        }
    }
}

size_t attention_smem_bytes(int nq, int nkv, int hd, int capacity) {
    const int group = nq / nkv;
    return static_cast<size_t>(group) * (hd + (capacity + kAttnSplits - 1) / kAttnSplits) * sizeof(float);
}

__global__ void embed_prefill_kernel(const int* prompt, const uint16_t* emb, float* hidden, int H, int vocab,
                                     int* pos, int* next_pos) {
    __shared__ int s_tok;
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) {
        long long tok = prompt[*next_pos];
        if (tok < 0 || tok >= vocab) tok = (tok < 0 ? -tok : tok) % (vocab > 1 ? vocab : 1);  // :573-575
        s_tok = static_cast<int>(tok);
    }
    __syncthreads();
    const uint16_t* e = emb + static_cast<size_t>(s_tok) * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x) hidden[k] = bf16_to_f32(e[k]);
    if (threadIdx.x == 0) {
        const int np = *next_pos;
        *pos = np;
        *next_pos = np + 1;
    }
}

__global__ void rmsnorm_kernel(const float* x, const float* w, int n, float eps, float* y) {
    __shared__ float ws[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += ws[i];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * inv * w[i];
}

}  // namespace xqb

// ------------------------------------------------------------------------------------
// Allocation-free attention step: scratch lives in this file-scope device array, which every
// GPU that loads the library holds until the process exits. 1 MiB per device.
// ------------------------------------------------------------------------------------
namespace xqb {
constexpr size_t kNoAllocScratchFloats = 256 * 1024;
}  // namespace xqb
static __device__ __align__(256) float g_attention_noalloc_scratch[xqb::kNoAllocScratchFloats];

// ------------------------------------------------------------------------------------
// Kernel-level C ABI
// ------------------------------------------------------------------------------------
namespace {
struct AttnScratch {
    float* part = nullptr;
    unsigned* counters = nullptr;
    float2* rope = nullptr;
    size_t part_floats = 0;
    int nkv = 0;
};
std::mutex g_attn_mu;
AttnScratch g_attn[64];
}  // namespace

extern "C" {

int xqk_rmsnorm(const float* x_dev, const float* w_dev, int n, float eps, float* y_dev, void* stream) {
    if (!x_dev || !w_dev || !y_dev || n <= 0) return -1;
    xqb::rmsnorm_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x_dev, w_dev, n, eps, y_dev);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int xqk_gated_delta_step(const float* conv_dev, const float* ab_dev, const float* a_log_dev,
                         const float* dt_bias_dev, float* state_dev, float* out_dev, int nk, int nv, int dk, int dv,
                         void* stream) {
    if (!conv_dev || !ab_dev || !a_log_dev || !dt_bias_dev || !state_dev || !out_dev || nk <= 0 || nv <= 0) return -1;
    if (dk != 128 || dv % xqb::kDeltaCols != 0) {
        xqb::set_last_error("xqk_gated_delta_step: needs key head dim 128 and value head dim % 16 == 0");
        return -1;
    }
    xqb::DeltaParams p{conv_dev, ab_dev, a_log_dev, dt_bias_dev, state_dev, out_dev, nk, nv, dk, dv};
    xqb::gated_delta_kernel<<<dim3(nv, dv / xqb::kDeltaCols), 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int xqk_attention_step(const float* qkv_dev, const float* q_norm_dev, const float* k_norm_dev, void* k_cache_dev,
                       void* v_cache_dev, int kv_fp16, int capacity, int position, int nq, int nkv, int hd,
                       int rotary_dim, float theta, float eps, float* out_dev, void* stream) {
    if (!qkv_dev || !q_norm_dev || !k_norm_dev || !k_cache_dev || !v_cache_dev || !out_dev || nq <= 0 || nkv <= 0 ||
        position < 0 || position >= capacity)
        return -1;
    if (hd != xqb::kAttnThreads || rotary_dim != 64 || nq % nkv != 0 || nq / nkv > xqb::kAttnMaxGroup) {
        xqb::set_last_error("xqk_attention_step: needs head_dim 256, rotary_dim 64, q/kv group <= 8");
        return -1;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    const int group = nq / nkv;
    const size_t need = static_cast<size_t>(nkv) * xqb::kAttnSplits * group * (hd + 2);
    std::lock_guard<std::mutex> lock(g_attn_mu);
    AttnScratch& s = g_attn[dev & 63];
    if (s.part_floats < need || s.nkv < nkv) {
        cudaFree(s.part);
        cudaFree(s.counters);
        if (cudaMalloc(&s.part, need * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&s.counters, nkv * sizeof(unsigned)) != cudaSuccess ||
            (!s.rope && cudaMalloc(&s.rope, 512 * sizeof(float2)) != cudaSuccess) ||
            cudaMemset(s.counters, 0, nkv * sizeof(unsigned)) != cudaSuccess) {
            s = AttnScratch();
            xqb::set_last_error("xqk_attention_step: scratch allocation failed");
            return -4;
        }
        s.part_floats = need;
        s.nkv = nkv;
    }
    xqb::AttnParams p = {};
    p.qkv = qkv_dev;
    p.q_norm = q_norm_dev;
    p.k_norm = k_norm_dev;
    p.k_cache = k_cache_dev;
    p.v_cache = v_cache_dev;
    p.capacity = capacity;
    p.pos_ptr = nullptr;
    p.pos_const = position;
    p.nq = nq;
    p.nkv = nkv;
    p.hd = hd;
    p.rotary = rotary_dim;
    p.theta = theta;
    p.eps = eps;
    p.part = s.part;
    p.counters = s.counters;
    p.out = out_dev;
    std::vector<float2> rope;
    xqb::rope_table(position, 1, rotary_dim, theta, &rope);
    if (cudaMemcpyAsync(s.rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess) {
        xqb::set_last_error("xqk_attention_step: rope upload failed");
        return -4;
    }
    p.rope = s.rope;
    p.rope_stride = 0;
    const size_t smem = xqb::attention_smem_bytes(nq, nkv, hd, capacity);
    if (smem > 200 * 1024) {
        xqb::set_last_error("xqk_attention_step: capacity too large for one call");
        return -1;
    }
    cudaError_t e = xqb::attention_init_device(200 * 1024);
    if (e == cudaSuccess) e = xqb::launch_attention(p, kv_fp16 != 0, smem, static_cast<cudaStream_t>(stream), false);
    if (e != cudaSuccess) {
        xqb::set_last_error(std::string("attention launch failed: ") + cudaGetErrorString(e));
        return -4;
    }
    return 0;
}

// Same contract and arithmetic as xqk_attention_step, for callers that must not allocate
// device memory while they run (plugin hosts that hand out all buffers themselves, code
// running under a fixed device-memory budget, or paths where an allocation would
// synchronise the device). Layout of the static scratch: 32 (cos, sin) RoPE pairs, then one
// completion counter per kv head, then the per-split partial results.
int xqk_attention_step_noalloc(const float* qkv_dev, const float* q_norm_dev, const float* k_norm_dev,
                               void* k_cache_dev, void* v_cache_dev, int kv_fp16, int capacity, int position,
                               int nq, int nkv, int hd, int rotary_dim, float theta, float eps, float* out_dev,
                               void* stream) {
    if (!qkv_dev || !q_norm_dev || !k_norm_dev || !k_cache_dev || !v_cache_dev || !out_dev || nq <= 0 || nkv <= 0 ||
        position < 0 || position >= capacity)
        return -1;
    if (hd != xqb::kAttnThreads || rotary_dim != 64 || nq % nkv != 0 || nq / nkv > xqb::kAttnMaxGroup) {
        xqb::set_last_error("xqk_attention_step_noalloc: needs head_dim 256, rotary_dim 64, q/kv group <= 8");
        return -1;
    }
    constexpr size_t kRopeFloats = 64, kCounterFloats = 64;
    const size_t part_floats = static_cast<size_t>(nkv) * xqb::kAttnSplits * (nq / nkv) * (hd + 2);
    if (nkv > static_cast<int>(kCounterFloats) || kRopeFloats + kCounterFloats + part_floats > xqb::kNoAllocScratchFloats) {
        xqb::set_last_error("xqk_attention_step_noalloc: needs " +
                            std::to_string(kRopeFloats + kCounterFloats + part_floats) +
                            " floats of scratch but the static scratch holds " +
                            std::to_string(xqb::kNoAllocScratchFloats) + " (at most 64 kv heads and nkv * 32 * "
                            "group * (head_dim + 2) + 128 floats)");
        return -1;
    }
    const size_t smem = xqb::attention_smem_bytes(nq, nkv, hd, capacity);
    if (smem > 200 * 1024) {
        xqb::set_last_error("xqk_attention_step_noalloc: capacity too large for one call");
        return -1;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        xqb::set_last_error("xqk_attention_step_noalloc: no usable current device");
        return -4;
    }
    // Once per device, with that device current: the device address of the static array
    // (its name in host code is only a host-side stand-in).
    static std::mutex mu;
    static float* base[64] = {};
    float* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!base[dev]) {
            void* ptr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&ptr, g_attention_noalloc_scratch);
            if (e != cudaSuccess) {
                xqb::set_last_error(std::string("xqk_attention_step_noalloc: cudaGetSymbolAddress failed: ") +
                                    cudaGetErrorString(e));
                return -4;
            }
            base[dev] = static_cast<float*>(ptr);
        }
        scratch = base[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float2* rope_dev = reinterpret_cast<float2*>(scratch);
    unsigned* counters = reinterpret_cast<unsigned*>(scratch + kRopeFloats);
    float* part = scratch + kRopeFloats + kCounterFloats;
    std::vector<float2> rope;
    xqb::rope_table(position, 1, rotary_dim, theta, &rope);
    // The counters must start at zero; the array keeps whatever the last call left in it.
    if (cudaMemcpyAsync(rope_dev, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaMemsetAsync(counters, 0, static_cast<size_t>(nkv) * sizeof(unsigned), st) != cudaSuccess) {
        xqb::set_last_error("xqk_attention_step_noalloc: scratch set-up copy failed");
        return -4;
    }
    xqb::AttnParams p = {};
    p.qkv = qkv_dev;
    p.q_norm = q_norm_dev;
    p.k_norm = k_norm_dev;
    p.k_cache = k_cache_dev;
    p.v_cache = v_cache_dev;
    p.capacity = capacity;
    p.pos_ptr = nullptr;
    p.pos_const = position;
    p.nq = nq;
    p.nkv = nkv;
    p.hd = hd;
    p.rotary = rotary_dim;
    p.theta = theta;
    p.eps = eps;
    p.rope = rope_dev;
    p.rope_stride = 0;
    p.part = part;
    p.counters = counters;
    p.out = out_dev;
    cudaError_t e = xqb::attention_init_device(200 * 1024);
    if (e == cudaSuccess) e = xqb::launch_attention(p, kv_fp16 != 0, smem, st, false);
    if (e != cudaSuccess) {
        xqb::set_last_error(std::string("attention launch failed: ") + cudaGetErrorString(e));
        return -4;
    }
    return 0;
}

}  // extern "C"
