// Batched-prefill element kernels (prefill_ops.cu): host launchers. Activations are
// [tokens][width] row-major; GEMM inputs are written as bf16 pairs (hi, lo = bf16(v - hi); lo
// may be null for one bf16 pass).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xqb {

constexpr size_t kPrefillAttnMaxSmem = 200 * 1024;

cudaError_t prefill_embed(const int* ids, const uint16_t* emb, float* H, int n, int hidden, int vocab, cudaStream_t s);
cudaError_t prefill_rmsnorm_split(const float* H, const float* w, int n, int width, float eps, __nv_bfloat16* hi,
                                  __nv_bfloat16* lo, cudaStream_t s);
// nseq > 1 (batched decode): nseq sequences of n rows each, sequence z's state at
// state + z * state_bstride.
cudaError_t prefill_conv(const float* Y, int ldy, const float* w, float* state, float* out, int n, int channels,
                         cudaStream_t s, int nseq = 1, size_t state_bstride = 0);
cudaError_t prefill_delta(const float* conv, int conv_ld, const float* Y, int ldy, int ab_off, const float* a_log,
                          const float* dt_bias, float* state, float* out, int out_ld, int n, int nk, int nv, int dk,
                          int dv, cudaStream_t s, int nseq = 1, size_t state_bstride = 0);
cudaError_t prefill_gated_norm(const float* O, int o_ld, const float* Y, int ldy, int z_off, const float* w, int heads,
                               int hd, float eps, int n, __nv_bfloat16* hi, __nv_bfloat16* lo, cudaStream_t s);
cudaError_t prefill_attn_prep(const float* Y, int ldy, const float* q_norm, const float* k_norm, const float2* rope,
                              int rope_stride, float* Q, void* kc, void* vc, bool kv_fp16, int p0, int n, int nq,
                              int nkv, int hd, float eps, cudaStream_t s, const int* pos_arr = nullptr,
                              size_t kv_bstride = 0);
// Dynamic shared memory of the causal attention kernel for contexts up to max_len positions.
size_t prefill_attn_smem(int nq, int nkv, int hd, int max_len);
// pos_arr (batched decode): row t is sequence t at position pos_arr[t] (< max_len), its KV cache
// at kc / vc + t * kv_bstride elements.
cudaError_t prefill_attn(const float* Q, const float* Y, int ldy, const void* kc, const void* vc, bool kv_fp16, int p0,
                         int n, int nq, int nkv, int hd, __nv_bfloat16* hi, __nv_bfloat16* lo, cudaStream_t s,
                         const int* pos_arr = nullptr, size_t kv_bstride = 0, int max_len = 0);
// Row-wise argmax of logits [rows][n] (ties to the lowest index, gemvW4A16ArgmaxNeon's rule,
// xq_gemv_w4a16_neon.cpp:315-318) into idx[rows].
cudaError_t batch_argmax(const float* logits, int rows, int n, int* idx, cudaStream_t s);
cudaError_t prefill_swiglu(const float* Y, int ldy, int inter, int n, __nv_bfloat16* hi, __nv_bfloat16* lo,
                           cudaStream_t s);

}  // namespace xqb
