// Test infrastructure only (the parity checker, never the product path).
//
// C-linkage shim compiled TOGETHER WITH the reference library's own sources
// (see oracle/Makefile, target _ref/libxqwen35_ref.so). The reference exposes
// its kernels as C++ functions taking xq::kernels::QuantizedMatrix
// (customlib/kernels/kernels.hpp:11-53); ctypes cannot call those, so each
// wrapper below builds the struct from plain pointers and forwards the call
// unchanged. No arithmetic happens here.
#include "kernels.hpp"

#include <cstdint>
#include <cstring>
#include <vector>

namespace {

xq::kernels::QuantizedMatrix makeMatrix(int rows, int cols, int group_size, int version,
                                        const uint8_t* packed, const float* scales,
                                        const float* zeros) {
    xq::kernels::QuantizedMatrix m;
    m.rows = rows;
    m.cols = cols;
    m.bits = 4;
    m.group_size = group_size;
    m.affine_asymmetric = (version == 2);
    const int gpr = (cols + group_size - 1) / group_size;
    const size_t packed_bytes = static_cast<size_t>(rows) * ((static_cast<size_t>(cols) + 1) / 2);
    const size_t meta = static_cast<size_t>(rows) * gpr;
    m.packed.assign(packed, packed + packed_bytes);
    m.scales.assign(scales, scales + meta);
    m.zeros.assign(zeros, zeros + meta);
    m.bias.assign(static_cast<size_t>(rows), 0.0f);
    return m;
}

}  // namespace

extern "C" {

// customlib/kernels/generated/arm64_neon/xq_gemv_w4a16_neon.cpp:259 (gemvW4A16Neon)
void ref_gemv_w4a16(int rows, int cols, int group_size, int version, const uint8_t* packed,
                    const float* scales, const float* zeros, const float* x, float* y) {
    const auto m = makeMatrix(rows, cols, group_size, version, packed, scales, zeros);
    xq::kernels::gemvW4A16Neon(m, x, y);
}

// customlib/kernels/generated/arm64_neon/xq_gemv_w4a16_neon.cpp:293 (gemvW4A16ArgmaxNeon)
int ref_gemv_w4a16_argmax(int rows, int cols, int group_size, int version, const uint8_t* packed,
                          const float* scales, const float* zeros, const float* x, float* out_value) {
    const auto m = makeMatrix(rows, cols, group_size, version, packed, scales, zeros);
    return xq::kernels::gemvW4A16ArgmaxNeon(m, x, out_value);
}

// customlib/kernels/reference/ref_gemv.cpp:100 (gemvLowBitReference: dense dequant dot)
void ref_gemv_lowbit_reference(int rows, int cols, int group_size, int version, const uint8_t* packed,
                               const float* scales, const float* zeros, const float* x, float* y) {
    const auto m = makeMatrix(rows, cols, group_size, version, packed, scales, zeros);
    xq::kernels::gemvLowBitReference(m, x, y);
}

// customlib/kernels/reference/ref_gemv.cpp:38 (quantizeLowBit, 4-bit only here).
// Output buffers: packed rows*ceil(cols/2) bytes, scales/zeros rows*ceil(cols/group) floats.
void ref_quantize_w4(const float* weights, int rows, int cols, int group_size, uint8_t* packed,
                     float* scales, float* zeros) {
    const auto q = xq::kernels::quantizeLowBit(weights, rows, cols, 4, group_size);
    std::memcpy(packed, q.packed.data(), q.packed.size());
    std::memcpy(scales, q.scales.data(), q.scales.size() * sizeof(float));
    std::memcpy(zeros, q.zeros.data(), q.zeros.size() * sizeof(float));
}

// customlib/kernels/reference/ref_rmsnorm.cpp:8
void ref_rmsnorm(const float* x, const float* weight, int n, float eps, float* y) {
    xq::kernels::rmsnormReference(x, weight, n, eps, y);
}

// customlib/kernels/reference/ref_attention.cpp:10
void ref_attention_decode(const float* q, const float* k_cache, const float* v_cache, int context,
                          int kv_heads, int q_heads, int head_dim, float* out) {
    xq::kernels::attentionDecodeReference(q, k_cache, v_cache, context, kv_heads, q_heads, head_dim, out);
}

// customlib/kernels/reference/ref_delta.cpp:8
void ref_gated_delta_decode(const float* q, const float* k, const float* v, float beta, float gate,
                            int key_dim, int value_dim, float* state, float* out) {
    xq::kernels::gatedDeltaDecodeReference(q, k, v, beta, gate, key_dim, value_dim, state, out);
}

}  // extern "C"
