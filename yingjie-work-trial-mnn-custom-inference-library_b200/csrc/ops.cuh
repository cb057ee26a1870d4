// Decode-step kernels other than the GEMV: Gated-DeltaNet state update, fused GQA decode
// attention, embedding row load, RMSNorm.
#pragma once

#include <vector>

#include <cuda_bf16.h>

#include "common.cuh"

namespace xqb {

// ---- Gated DeltaNet ----------------------------------------------------------------
constexpr int kDeltaCols = 16;  // value columns of one head per block

struct DeltaParams {
    const float* conv;     // [2*nk*dk + nv*dv]: q | k | v after conv + SiLU
    const float* ab;       // [a (nv) | b (nv)] raw projections
    const float* a_log;    // [nv]
    const float* dt_bias;  // [nv]
    float* state;          // [nv][dk][dv]
    float* out;            // [nv*dv]
    int nk, nv, dk, dv;
    // Optional fused part of the gated head RMSNorm (applyGatedHeadRms, custom_model.cpp:329-349)
    // when z is set: out = o * w * silu(z) and head_ss[vh * (dv / kDeltaCols) + slice] = the sum
    // of o^2 over the item's columns; the consumer multiplies by 1 / sqrt(mean(o^2) + eps) per head.
    const float* z;        // [nv*dv]
    const float* norm_w;   // [dv], no +1
    float* head_ss;        // [nv][dv / kDeltaCols]
};

// grid (nv, dv / kDeltaCols), block dk (= 128)
__global__ void gated_delta_kernel(const DeltaParams p);

// Shared scratch of one DeltaNet work item (one value head, kDeltaCols columns).
struct DeltaScratch {
    float red[4][kDeltaCols];
    float bc[kDeltaCols];
    float nrm[2][4];
};
// One DeltaNet work item run by 128 threads (i = key row) that synchronise with
// bar.sync(bar_id, 128).
// (defined in ops_device.cuh)

// ---- Full attention ------------------------------------------------------------------
constexpr int kAttnSplits = 32;   // blocks per kv head (split over positions)
constexpr int kAttnBatchSplits = 8;  // batched decode with >= 32 (sequence, kv head) pairs
constexpr int kAttnThreads = 256;  // = head_dim
constexpr int kAttnMaxGroup = 8;   // query heads per kv head

struct AttnParams {
    const float* qkv;     // [2*nq*hd | nkv*hd | nkv*hd]
    const float* q_norm;  // [hd], +1 applied
    const float* k_norm;  // [hd], +1 applied
    void* k_cache;        // [capacity][nkv][hd]
    void* v_cache;
    int capacity;
    const int* pos_ptr;   // position of this token (device); pos_const when null
    int pos_const;
    int nq, nkv, hd, rotary;
    float theta, eps;
    const float2* rope;   // (cos, sin) of position * inv_freq[i], i < rotary/2, per position
    int rope_stride;      // floats2 per position row; 0: a single row for this call's position
    float* part;          // [nkv][kAttnSplits][group][hd + 2]
    unsigned* counters;   // [nkv]
    float* out;           // [nq*hd]
    unsigned* err;
};

// Shared scratch of one attention work item besides the dynamic [group][hd] q and
// [group][cmax] score arrays.
struct AttnScratch {
    float m[kAttnMaxGroup], l[kAttnMaxGroup];
    float pm[kAttnSplits * kAttnMaxGroup], pl[kAttnSplits * kAttnMaxGroup];
    float M[kAttnMaxGroup], invL[kAttnMaxGroup];
    int last;
};
// One attention work item (kv head kh, split) run by kAttnThreads threads synchronising with
// bar.sync(bar_id, kAttnThreads); dyn = group*hd + group*cmax floats of shared memory.
// (defined in ops_device.cuh)

// Launch the attention kernel (fp16 or fp32 KV cache); grid (nkv, kAttnSplits).
cudaError_t launch_attention(const AttnParams& p, bool kv_fp16, size_t smem, cudaStream_t s, bool pdl);
// Batched decode: grid (nkv, kAttnSplits, batch). Sequence b reads its projections at
// p.qkv + b * qkv_stride and its position at p.pos_ptr[b], appends to and attends over its own
// KV cache (p.k_cache / p.v_cache + b * kv_bstride elements), and uses its own scratch
// (p.part + b * nkv * kAttnSplits * group * (hd + 2), p.counters + b * nkv) and output rows
// (b * nq * hd into out, or into out_hi / out_lo as a bf16 pair when those are set).
cudaError_t launch_attention_batch(const AttnParams& p, bool kv_fp16, size_t smem, int batch, int qkv_stride,
                                   size_t kv_bstride, __nv_bfloat16* out_hi, __nv_bfloat16* out_lo, cudaStream_t s);
cudaError_t attention_init_device(int max_smem_bytes);
size_t attention_smem_bytes(int nq, int nkv, int hd, int capacity);
// Host-side RoPE table with the reference's arithmetic (applyRopeVector,
// custom_model.cpp:351-370): inv_freq = pow(theta, -2i/rotary), angle = pos * inv_freq,
// (cos, sin) in fp32 through the same libm calls, for positions [first, first + count).
void rope_table(int first, int count, int rotary, float theta, std::vector<float2>* out);

// ---- Small ops ------------------------------------------------------------------------
// hidden = embedding row of prompt[*next_pos]; *pos = *next_pos; ++*next_pos (prefill step).
__global__ void embed_prefill_kernel(const int* prompt, const uint16_t* emb, float* hidden, int H, int vocab,
                                     int* pos, int* next_pos);
// y = rmsnorm(x, w), single block.
__global__ void rmsnorm_kernel(const float* x, const float* w, int n, float eps, float* y);

}  // namespace xqb
