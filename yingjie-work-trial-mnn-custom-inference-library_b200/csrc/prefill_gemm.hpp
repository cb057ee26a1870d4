// Batched-prefill W4A16 GEMM on tcgen05 / TMEM (see prefill_gemm.cu): host interface.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.hpp"

namespace xqb {

enum PgOutKind : int {
    kPgOutF32 = 0,     // y = X W^T (fp32)
    kPgOutAddF32 = 1,  // y += X W^T (fp32; the residual add of o_proj / out_proj / down)
    kPgOutBF16 = 2,    // y = X W^T rounded to bf16
};

struct PgParams {
    CUtensorMap map_x;       // X (or X_hi) bf16 [M][K], box 64 x NT, 128-byte swizzle
    CUtensorMap map_x_lo;    // split mode: X_lo = bf16(X - X_hi)
    CUtensorMap map_codes;   // W row layout as bytes [rows][row_stride], box 32 x 128
    CUtensorMap map_scales;  // the same bytes, box 16 x 128 (fp16 scales of 8 groups)
    int M, N, K, meta_offset, ldy, out_kind;
    float* y_f32;
    __nv_bfloat16* y_bf16;
    unsigned* err;
    uint64_t wait_ns;
    const uint8_t* w_rows;  // the row layout itself (small-M kernel: scales read per row)
    int row_stride;
    int split;              // X_lo present
};

// Y[t][n] (ldy elements per token row) = sum_k X[t][k] W[n][k] for t < M, n < rows, on the
// tensor cores. x_lo == nullptr: one bf16 pass over X as given; otherwise split mode (X as a
// bf16 pair). M > 64: W dequantised to bf16 in shared memory (split mode: also its bf16
// residual, three MMA chains, error ~2^-16). M <= 64: the small-M kernel multiplies the exact
// integer codes (code - 8) and applies each group's scale to that group's fp32 partial sum, so
// W is exact in both modes; its K range is split over a thread-block cluster when the row tiles
// alone would leave SMs idle. Needs a symmetric row-layout matrix (kind 0, group 64) and 16-byte
// aligned activations.
bool launch_prefill_gemm(const DevMatrix& w, const __nv_bfloat16* x, const __nv_bfloat16* x_lo, int M, void* y,
                         int ldy, int out_kind, unsigned* err, int num_sms, cudaStream_t s, uint64_t wait_ns = 0);

}  // namespace xqb
