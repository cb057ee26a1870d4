// Host-side interface of the W4A16 GEMV: device matrix layouts and launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "gemv.cuh"

namespace xqb {

// One matrix in the reference's XQ4 fields (kernels.hpp:11-21, custom_model.cpp:218-262).
struct HostMatrix {
    int rows = 0, cols = 0, group = 0, version = 1;
    std::vector<uint8_t> packed;  // rows * ceil(cols/2)
    std::vector<float> scales;    // rows * ceil(cols/group)
    std::vector<float> zeros;
};

bool read_xq4_file(const std::string& path, HostMatrix* m, std::string* error);

// A device matrix in the fused-kernel row layout (kind 0 / 1) or, for shapes that layout
// does not serve, the reference layout for the generic kernel (kind 2).
struct DevMatrix {
    int rows = 0, cols = 0, group = 0, version = 1;
    int kind = 2;  // 0: fp16 scale, zero 8; 1: float2 {scale, offset}; 2: generic
    int row_stride = 0, meta_offset = 0;
    uint8_t* d_rows = nullptr;  // kinds 0/1
    uint8_t* d_packed = nullptr;  // kind 2
    float* d_scales = nullptr;
    float* d_zeros = nullptr;
    size_t bytes = 0;
    uint8_t* d_tiles = nullptr;  // optional 16-row tensor-core tile copy (symmetric layout)
    size_t tile_bytes = 0;
    bool fast() const { return kind != 2; }
};

// True when the fused kernel serves matrices of this shape.
bool fast_shape(int cols, int group);

// The fused-kernel row layout of the row-wise concatenation of `parts` (as upload_matrix
// builds it) in host memory; false (error set) when the shape has no fused layout. narrow:
// also widths that are a multiple of 512 only (K slices of tensor-parallel shards; served by
// the tensor-core GEMM alone, not by the GEMV kernels).
bool build_matrix_rows(const std::vector<const HostMatrix*>& parts, bool interleave_pairs, DevMatrix* shape,
                       std::vector<uint8_t>* host, std::string* error, bool narrow = false);
// Device copy of rows built by build_matrix_rows (fills d_rows and bytes).
bool upload_matrix_rows(const std::vector<uint8_t>& host, DevMatrix* m, std::string* error);
// The packed B200 layout on disk: a 64-byte header (magic "XQB200\0\0", version, kind, rows,
// cols, group, xq4 version, row_stride, meta_offset, byte count) followed by the rows.
bool write_b200_file(const std::string& path, const DevMatrix& shape, const std::vector<uint8_t>& host,
                     std::string* error);
bool read_b200_file(const std::string& path, DevMatrix* shape, std::vector<uint8_t>* host, std::string* error);

// Build one device matrix from the row-wise concatenation of `parts` (all with the same
// cols and group). interleave_pairs: parts must be two equal-height matrices, emitted as
// rows a0, b0, a1, b1, ... (gate/up pairing for the fused SwiGLU epilogue).
bool upload_matrix(const std::vector<const HostMatrix*>& parts, bool interleave_pairs, DevMatrix* out,
                   std::string* error);
void free_matrix(DevMatrix* m);

struct LaunchCtx {
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    bool pdl = true;
};

// Fill the shape fields of p from m and launch the fused kernel. unit: 2 for gate/up pairs.
// Whether weight rows are streamed with the L2 evict-first policy (XQ_L2_EVICT_FIRST, default 1).
int gemv_evict_first();
bool launch_gemv(const DevMatrix& m, int pro, int epi, GemvParams p, int unit, const LaunchCtx& ctx,
                 int max_blocks = 0);
// Number of blocks launch_gemv uses (argmax partial buffers are sized with this).
int gemv_grid(const DevMatrix& m, int unit, int num_sms, int max_blocks = 0);
// Generic-layout y = W x.
bool launch_gemv_generic(const DevMatrix& m, const float* x, float* y, cudaStream_t stream);
// Register the dynamic shared memory limits of every fused instantiation (once per device).
bool gemv_init_device();

// Programmatic dependent launch between kernels (XQ_PDL=0 turns it off, for A/B measurements).
bool pdl_enabled();

// Launch helper with the programmatic-dependent-launch attribute.
template <typename Kernel, typename... Args>
cudaError_t launch_ex(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace xqb
