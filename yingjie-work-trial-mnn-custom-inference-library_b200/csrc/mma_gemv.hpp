// Tensor-core W4A16 GEMV (mma.sync m16n8k32, u8 codes x s8 activation digits): host side.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "gemv.hpp"

namespace xqb {

// A matrix in the "mma16" tile layout: 16-row tiles, per tile and pair of 64-column groups
// 1088 bytes (four 32-column slabs of fragment-ordered nibbles, then fp16 scales).
constexpr int kMmaUnitBytes = 1088;  // one 16-row tile x one pair of groups (128 columns)

struct MmaMatrix {
    int rows = 0, cols = 0, ntiles = 0, pairs = 0;
    size_t bytes = 0;
    uint8_t* d_tiles = nullptr;
};

// The layout serves symmetric xq4 v1 matrices (zero 8) with group 64, scales exact in fp16,
// cols a multiple of 512 (and of 4096 above 4096).
bool mma_eligible(const HostMatrix& h);
bool build_mma_matrix(const HostMatrix& h, MmaMatrix* out, std::string* error);
void free_mma_matrix(MmaMatrix* m);
// Build the tile copy of a symmetric row-layout matrix from its host rows (as
// build_matrix_rows / read_b200_file give them) into m->d_tiles.
bool attach_mma_tiles(const std::vector<uint8_t>& rows_host, DevMatrix* m, std::string* error);
// The tiles of a symmetric matrix (reference nibble order, fp32 scales rounded to fp16) in host
// memory; cols a multiple of 128. No device work.
bool host_mma_tiles(const uint8_t* packed, const float* scales, int rows, int cols, std::vector<uint8_t>* out);
bool mma_init_device();
// y = W x (fp32 in/out, device pointers); one block per SM, at most num_sms blocks. With `pdl`
// the launch may overlap the previous kernel in the stream (programmatic dependent launch): the
// weights stream at once, x is read after that kernel has finished.
bool launch_mma_gemv(const MmaMatrix& m, const float* x, float* y, unsigned* err, int num_sms, cudaStream_t s,
                     bool pdl = false);
// The same with fp16 x and y (fp32 arithmetic; y rounded to fp16 once).
bool launch_mma_gemv_f16(const MmaMatrix& m, const __half* x, __half* y, unsigned* err, int num_sms, cudaStream_t s,
                         bool pdl = false);

}  // namespace xqb
