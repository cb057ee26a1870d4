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
#include "ops_device.cuh"

namespace xqb {

// One block = one value head vh and kDeltaCols of its value columns; thread i = key row i.
// Per step (custom_model.cpp:1037-1095, ref_delta.cpp:8-41):
//   q, k <- l2-normalised (eps 1e-6 inside the sqrt); beta = sigmoid(b[vh]);
//   g = -exp(A_log[vh]) * softplus(a[vh] + dt_bias[vh]); S <- exp(g) S;
//   for each column j: delta_j = beta (v_j - sum_i S_ij k_i); S_ij += k_i delta_j;
//   o_j = sum_i S_ij q_i / sqrt(dk).
// Columns are independent, so the [dk x dv] state splits over blocks by column slices.
__global__ void __launch_bounds__(128) gated_delta_kernel(const DeltaParams p) {
    __shared__ DeltaScratch sh;
    pdl_launch_dependents();
    pdl_wait();
    delta_item(p, blockIdx.x, blockIdx.y, threadIdx.x, 1, &sh);
}

// grid (nkv, kAttnSplits), block 256 (hd = 256, rotary_dim = 64, group <= 8).
template <typename KV>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
    extern __shared__ float sm[];
    __shared__ AttnScratch sh;
    pdl_launch_dependents();
    pdl_wait();
    attention_item<KV>(p, blockIdx.x, blockIdx.y, threadIdx.x, 1, sm, &sh);
}


cudaError_t launch_attention(const AttnParams& p, bool kv_fp16, size_t smem, cudaStream_t s, bool pdl) {
    const dim3 grid(p.nkv, kAttnSplits), block(kAttnThreads);
    return kv_fp16 ? launch_ex(attention_kernel<__half>, grid, block, smem, s, pdl, p)
                   : launch_ex(attention_kernel<float>, grid, block, smem, s, pdl, p);
}

template <typename KV, int SPLITS>
__global__ void __launch_bounds__(kAttnThreads) attention_batch_kernel(const AttnParams p, int qkv_stride,
                                                                      size_t kv_bstride, __nv_bfloat16* out_hi,
                                                                      __nv_bfloat16* out_lo) {
    extern __shared__ float sm[];
    __shared__ AttnScratch sh;
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.z;
    const size_t ob = static_cast<size_t>(b) * p.nq * p.hd;
    AttnParams q = p;
    q.qkv = p.qkv + static_cast<size_t>(b) * qkv_stride;
    q.k_cache = static_cast<KV*>(p.k_cache) + b * kv_bstride;
    q.v_cache = static_cast<KV*>(p.v_cache) + b * kv_bstride;
    q.pos_ptr = p.pos_ptr + b;
    q.part = p.part + static_cast<size_t>(b) * p.nkv * kAttnSplits * (p.nq / p.nkv) * (p.hd + 2);
    q.counters = p.counters + b * p.nkv;
    q.out = p.out ? p.out + ob : nullptr;
    attention_item<KV, SPLITS>(q, blockIdx.x, blockIdx.y, threadIdx.x, 1, sm, &sh, out_hi ? out_hi + ob : nullptr,
                               out_lo ? out_lo + ob : nullptr);
}

cudaError_t launch_attention_batch(const AttnParams& p, bool kv_fp16, size_t smem, int batch, int qkv_stride,
                                   size_t kv_bstride, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo, cudaStream_t s) {
    if (!p.pos_ptr || batch < 1 || !out_hi != !out_lo || (!out_hi && !p.out)) return cudaErrorInvalidValue;
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    cudaGetDevice(&dev);
    dev &= 63;
    std::call_once(once[dev], [&] {
        const void* ks[] = {reinterpret_cast<const void*>(attention_batch_kernel<float, kAttnSplits>),
                            reinterpret_cast<const void*>(attention_batch_kernel<__half, kAttnSplits>),
                            reinterpret_cast<const void*>(attention_batch_kernel<float, kAttnBatchSplits>),
                            reinterpret_cast<const void*>(attention_batch_kernel<__half, kAttnBatchSplits>)};
        attr_err[dev] = cudaSuccess;
        for (const void* k : ks)
            if (attr_err[dev] == cudaSuccess)
                attr_err[dev] = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    if (attr_err[dev] != cudaSuccess) return attr_err[dev];
    // With enough (sequence, kv head) pairs to fill the GPU, fewer position splits per pair: each
    // block scores more positions and the last one merges fewer partial results.
    const bool few = batch * p.nkv >= kAttnSplits;
    const int splits = few ? kAttnBatchSplits : kAttnSplits;
    const int group = p.nq / p.nkv;
    const size_t need = sizeof(float) * static_cast<size_t>(group) * (p.hd + (p.capacity + splits - 1) / splits);
    if (few) smem = need;
    if (smem < need || smem > 200 * 1024) return cudaErrorInvalidValue;
    const dim3 grid(p.nkv, splits, batch), block(kAttnThreads);
    if (few)
        return kv_fp16 ? launch_ex(attention_batch_kernel<__half, kAttnBatchSplits>, grid, block, smem, s, pdl_enabled(), p,
                                   qkv_stride, kv_bstride, out_hi, out_lo)
                       : launch_ex(attention_batch_kernel<float, kAttnBatchSplits>, grid, block, smem, s, pdl_enabled(), p,
                                   qkv_stride, kv_bstride, out_hi, out_lo);
    return kv_fp16 ? launch_ex(attention_batch_kernel<__half, kAttnSplits>, grid, block, smem, s, pdl_enabled(), p,
                               qkv_stride, kv_bstride, out_hi, out_lo)
                   : launch_ex(attention_batch_kernel<float, kAttnSplits>, grid, block, smem, s, pdl_enabled(), p,
                               qkv_stride, kv_bstride, out_hi, out_lo);
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
struct AbiAttnScratch {
    float* part = nullptr;
    unsigned* counters = nullptr;
    float2* rope = nullptr;
    size_t part_floats = 0;
    int nkv = 0;
};
std::mutex g_attn_mu;
AbiAttnScratch g_attn[64];
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
    AbiAttnScratch& s = g_attn[dev & 63];
    if (s.part_floats < need || s.nkv < nkv) {
        cudaFree(s.part);
        cudaFree(s.counters);
        s.part = nullptr;
        s.counters = nullptr;
        if (cudaMalloc(&s.part, need * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&s.counters, nkv * sizeof(unsigned)) != cudaSuccess ||
            (!s.rope && cudaMalloc(&s.rope, 512 * sizeof(float2)) != cudaSuccess) ||
            cudaMemset(s.counters, 0, nkv * sizeof(unsigned)) != cudaSuccess) {
            // free whatever this attempt (or the first call) did allocate before forgetting it
            cudaFree(s.part);
            cudaFree(s.counters);
            cudaFree(s.rope);
            s = AbiAttnScratch();
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
