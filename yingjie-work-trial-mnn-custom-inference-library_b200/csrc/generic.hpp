// Generic-shape decode-step kernels (generic.cu): host launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xqb {

struct GenericLinearArgs {
    const float* proj;  // in_proj output [qkv (conv_dim) | z | a | b]
    const float* conv_w;
    float* conv_state;
    const float *a_log, *dt_bias;
    float* rec_state;
    const float* norm_w;  // linear-attention norm weights (no +1)
    float eps;
    float* conv;  // scratch, conv_dim floats
    float* out;   // nv * dv
    int nk, nv, dk, dv, kconv;
};

struct GenericAttnArgs {
    const float* proj;  // q_proj output (q_rows) | k | v
    int q_rows;
    const float *q_norm, *k_norm;  // +1 applied
    const float2* rope;            // [capacity][rope_stride] (cos, sin)
    int rope_stride;
    float *k_cache, *v_cache;  // [capacity][nkv][hd] fp32
    const int* pos;            // device position of this token
    float* scores;             // scratch [nq][capacity]
    float* qbuf;               // scratch (nq + nkv) * hd
    float* out;                // nq * hd
    int nq, nkv, hd, rotary;
    float eps;
};

cudaError_t generic_linear_attn(const GenericLinearArgs& a, cudaStream_t s);
cudaError_t generic_attention(const GenericAttnArgs& a, cudaStream_t s);
cudaError_t generic_swiglu(const float* gu, float* h, int inter, cudaStream_t s);
cudaError_t generic_add(float* hidden, const float* y, int n, cudaStream_t s);
// Greedy sample of the logits, then the token's embedding row into hidden and the positions
// advanced (decode head of a generic-shape step).
cudaError_t generic_sample(const float* logits, int vocab, const uint16_t* emb, float* hidden, int H, int* pos,
                           int* next_pos, int* token_out, int* ring, int* ring_ctr, int ring_cap, cudaStream_t s);

}  // namespace xqb
