// W4A16 GEMV on the integer tensor cores (prototype, standalone): mma.sync m16n8k32 with
// unsigned 8-bit weight codes and signed 8-bit activation digits, exact s32 accumulation.
//
// Same mathematics as gemv_w4a16_kernel (gemvW4A16Neon, neon.cpp:259-291, symmetric layout:
// y[r] = sum_g s[r][g] * sum_{c in g} (code[r][c] - 8) * x[c]): x is held as three signed
// 8-bit digits of a 22-bit fixed-point mantissa per 64-column group (x ~ m * 2^-S_g), so every
// code * x product is an exact integer; the group scale is applied once per (row, group).
//
// Weight layout ("mma16"): rows in tiles of 16; per tile, per pair of groups (128 columns),
// four 32-column slabs of 256 bytes then 64 bytes of fp16 scales (1088 bytes). In a slab, lane
// L's 8 bytes hold its A fragment: byte j of the first word = code(r, c0 + j) in the low nibble
// and code(r + 8, c0 + j) in the high nibble, the second word the same for columns c0 + 16 + j
// (r = L / 4, c0 = (L % 4) * 4), so a0 / a1 / a2 / a3 are the masked low / shifted high nibbles.
// The N dimension carries the digits: columns 0-2 the three digits of the pair's first group,
// 3-5 those of the second, 6-7 zero; one accumulator serves both groups, and the symmetric zero
// (-8 * sum of digits) is its start value.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"
#include "gemv.cuh"
#include "mma_gemv.hpp"

namespace xqb {

namespace {

constexpr int kMmaTeams = 2, kMmaWarpsPerTeam = 4;
constexpr int kMmaConsumerWarps = kMmaTeams * kMmaWarpsPerTeam;
constexpr int kMmaThreads = 32 * (kMmaConsumerWarps + 1);
constexpr int kMmaMaxSlots = 8;

template <typename XT, typename YT>
struct MmaParams {
    const uint8_t* tiles;
    const XT* x;
    YT* y;
    int rows, cols, ntiles, pairs;
    int ppc;  // group pairs per ring chunk
    int cpt;  // chunks per tile
    int nslots;
    unsigned* err;
};

// Shared memory: [0,64) full, [64,128) empty, [128,1152) row sums [2 teams][4 warps][16] (512 B)
// + group exponents etc.; then B fragments [cols/32 slabs][32 lanes][8 B], start values
// [pairs][8] s32, column weights [pairs][8] f32, then the ring.
constexpr int kOffFull = 0, kOffEmpty = 64, kOffRed = 128, kOffFixed = 1152;

__host__ __device__ inline size_t table_bytes(int cols) {
    const size_t pairs = static_cast<size_t>(cols) / 128;
    return static_cast<size_t>(cols) * 8 + pairs * 32 + pairs * 32 + static_cast<size_t>(cols / 64) * 4;
}

// Digit d (0..2) of round_to_nearest_even(x * 2^S), as a signed byte (see gemv_make_limbs).
__device__ __forceinline__ uint32_t digit_byte(float x, float up, int d) {
    const uint32_t u = static_cast<uint32_t>(__float_as_int(fmaf(x, up, 12582912.0f))) + (0x808080u - 0x4B400000u);
    return ((u >> (8 * d)) & 0xffu) ^ 0x80u;
}

// Four consecutive x values as fp32 (x is fp32 or fp16; 16- or 8-byte aligned by construction).
__device__ __forceinline__ float4 load_x4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 load_x4(const __half* p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void store_y(float* y, float v) { *y = v; }
__device__ __forceinline__ void store_y(__half* y, float v) { *y = __float2half_rn(v); }

// The weight stream does not depend on any earlier kernel: with programmatic dependent launch
// the producer starts streaming while the previous kernel in the stream finishes, and the
// consumers wait for it (griddepcontrol.wait) before reading x. Without the launch attribute
// the wait returns at once.
template <typename XT, typename YT>
__global__ void __launch_bounds__(kMmaThreads, 1) gemv_mma_kernel(const MmaParams<XT, YT> p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffFull);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
    float* red = reinterpret_cast<float*>(smem + kOffRed);
    uint2* btab = reinterpret_cast<uint2*>(smem + kOffFixed);
    int* cinit = reinterpret_cast<int*>(smem + kOffFixed + static_cast<size_t>(p.cols) * 8);
    float* wtab = reinterpret_cast<float*>(cinit + p.pairs * 8);
    int* sexp = reinterpret_cast<int*>(wtab + p.pairs * 8);
    uint8_t* ring = smem + kOffFixed + ((table_bytes(p.cols) + 127) & ~static_cast<size_t>(127));
    const int slot_bytes = p.ppc * kMmaUnitBytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x;
    const int t_begin = static_cast<int>(static_cast<long long>(p.ntiles) * blockIdx.x / G);
    const int t_end = static_cast<int>(static_cast<long long>(p.ntiles) * (blockIdx.x + 1) / G);
    const int nchunks = (t_end - t_begin) * p.cpt;
    if (tid == 0) {
        for (int s = 0; s < p.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMmaWarpsPerTeam);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kMmaConsumerWarps) {  // producer: this block's tiles, chunk by chunk
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int issued = 0;
            for (int g = 0; g < nchunks; ++g) {
                const int s = g % p.nslots;
                if (g >= p.nslots &&
                    !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((g / p.nslots) - 1) & 1), p.err))
                    break;
                const int tile = t_begin + g / p.cpt, c = g % p.cpt;
                mbar_expect_tx(&full[s], static_cast<uint32_t>(slot_bytes));
                bulk_g2s_hint(ring + static_cast<size_t>(s) * slot_bytes,
                              p.tiles + (static_cast<size_t>(tile) * p.pairs + static_cast<size_t>(c) * p.ppc) * kMmaUnitBytes,
                              static_cast<uint32_t>(slot_bytes), &full[s], pol);
                ++issued;
            }
            for (int k = max(0, issued - p.nslots); k < issued; ++k)
                mbar_wait_drain(&full[k % p.nslots], static_cast<uint32_t>((k / p.nslots) & 1));
        }
        return;
    }

    // ---- prologue: group exponents, zero-point start values, column weights, B fragments ----
    pdl_wait();  // x may be the previous kernel's output
    constexpr int nthr = kMmaConsumerWarps * 32;
    for (int g = tid; g < p.cols / 64; g += nthr) {
        float amax = 0.0f;
        bool finite = true;  // fmaxf drops NaN operands: test every value
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            v[i] = load_x4(p.x + 64 * g + 4 * i);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            finite = finite && isfinite(v[i].x) && isfinite(v[i].y) && isfinite(v[i].z) && isfinite(v[i].w);
        }
        const int ex = ((__float_as_int(amax) >> 23) & 0xff) - 126;
        const int S = max(-100, min(100, 22 - ex));
        const float up = __int_as_float((S + 127) << 23);
        int zs[3] = {0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int d = 0; d < 3; ++d) zs[d] += static_cast<int>(static_cast<int8_t>(digit_byte(e[j], up, d)));
        }
        sexp[g] = S;
        const int pp = g >> 1, n0 = (g & 1) * 3;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            cinit[pp * 8 + n0 + d] = -8 * zs[d];
            // 256^d * 2^-S; NaN for a group holding a non-finite x (every row's result is then NaN,
            // as in fp32)
            wtab[pp * 8 + n0 + d] = finite ? __int_as_float((127 - S + 8 * d) << 23) : __int_as_float(0x7fc00000);
        }
        if (g & 1) {
            cinit[pp * 8 + 6] = cinit[pp * 8 + 7] = 0;
            wtab[pp * 8 + 6] = wtab[pp * 8 + 7] = 0.0f;
        }
    }
    named_bar(1, nthr);
    for (int e = tid; e < (p.cols / 32) * 32; e += nthr) {
        const int slab = e >> 5, L = e & 31;
        const int s = slab & 3, n = L >> 2;
        const bool valid = (s < 2 && n < 3) || (s >= 2 && n >= 3 && n < 6);
        uint2 b = make_uint2(0u, 0u);
        if (valid) {
            const int d = n % 3, g = 2 * (slab >> 2) + (s >= 2 ? 1 : 0);
            const float up = __int_as_float((sexp[g] + 127) << 23);
            const int k0 = 32 * slab + (L & 3) * 4;
            const float4 lo = load_x4(p.x + k0);
            const float4 hi = load_x4(p.x + k0 + 16);
            b.x = digit_byte(lo.x, up, d) | (digit_byte(lo.y, up, d) << 8) | (digit_byte(lo.z, up, d) << 16) |
                  (digit_byte(lo.w, up, d) << 24);
            b.y = digit_byte(hi.x, up, d) | (digit_byte(hi.y, up, d) << 8) | (digit_byte(hi.z, up, d) << 16) |
                  (digit_byte(hi.w, up, d) << 24);
        }
        btab[e] = b;
    }
    named_bar(1, nthr);

    // ---- main loop: team tau takes tiles tau, tau + 2, ...; warp wt covers 1/4 of each chunk ----
    const int tau = warp / kMmaWarpsPerTeam, wt = warp % kMmaWarpsPerTeam;
    const int q = lane & 3, r = lane >> 2;
    const int pw = p.ppc / kMmaWarpsPerTeam;  // pairs per warp per chunk
    for (int tile = t_begin + tau; tile < t_end; tile += kMmaTeams) {
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int c = 0; c < p.cpt; ++c) {
            const int g = (tile - t_begin) * p.cpt + c;
            const int s = g % p.nslots;
            mbar_wait_bounded(&full[s], static_cast<uint32_t>((g / p.nslots) & 1), p.err);
            const uint8_t* base = ring + static_cast<size_t>(s) * slot_bytes;
            for (int k = 0; k < pw; ++k) {
                const int pl = wt * pw + k, pg = c * p.ppc + pl;
                const uint8_t* pb = base + pl * kMmaUnitBytes;
                const int2 ci = *reinterpret_cast<const int2*>(cinit + pg * 8 + 2 * q);
                int d[4] = {ci.x, ci.y, ci.x, ci.y};
#pragma unroll
                for (int sl = 0; sl < 4; ++sl) {
                    const uint2 a = *reinterpret_cast<const uint2*>(pb + sl * 256 + 8 * lane);
                    const uint2 b = btab[(pg * 4 + sl) * 32 + lane];
                    mma_u8s8(d, a.x & 0x0F0F0F0Fu, (a.x >> 4) & 0x0F0F0F0Fu, a.y & 0x0F0F0F0Fu, (a.y >> 4) & 0x0F0F0F0Fu,
                           b.x, b.y);
                }
                const uint2 sh = *reinterpret_cast<const uint2*>(pb + 1024 + 8 * r);
                const float2 s_r = __half22float2(*reinterpret_cast<const __half2*>(&sh.x));  // (g0, g1) of row r
                const float2 s_r8 = __half22float2(*reinterpret_cast<const __half2*>(&sh.y));  // of row r + 8
                const float2 w = *reinterpret_cast<const float2*>(wtab + pg * 8 + 2 * q);
                const float sa0 = q >= 2 ? s_r.y : s_r.x, sb0 = q >= 1 ? s_r.y : s_r.x;
                const float sa1 = q >= 2 ? s_r8.y : s_r8.x, sb1 = q >= 1 ? s_r8.y : s_r8.x;
                acc0 += static_cast<float>(d[0]) * (w.x * sa0) + static_cast<float>(d[1]) * (w.y * sb0);
                acc1 += static_cast<float>(d[2]) * (w.x * sa1) + static_cast<float>(d[3]) * (w.y * sb1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        float* rb = red + (tau * kMmaWarpsPerTeam + wt) * 16;
        if (q == 0) {
            rb[r] = acc0;
            rb[r + 8] = acc1;
        }
        named_bar(2 + tau, 32 * kMmaWarpsPerTeam);
        if (wt == 0 && lane < 16) {
            const float* t0 = red + tau * kMmaWarpsPerTeam * 16;
            const float yv = (t0[lane] + t0[16 + lane]) + (t0[32 + lane] + t0[48 + lane]);
            const int row = tile * 16 + lane;
            if (row < p.rows) store_y(p.y + row, yv);
        }
        named_bar(2 + tau, 32 * kMmaWarpsPerTeam);
    }
}

}  // namespace

bool mma_eligible(const HostMatrix& h) {
    if (h.version != 1 || h.group != 64 || h.cols % 512 != 0 || (h.cols > 4096 && h.cols % 4096 != 0)) return false;
    for (size_t i = 0; i < h.scales.size(); ++i) {
        if (h.zeros[i] != 8.0f) return false;
        const float s = h.scales[i];
        if (__half2float(__float2half_rn(s)) != s) return false;
    }
    return true;
}

namespace {

// The mma16 tiles of a rows x K matrix given code(row, col) and scale(row, group); rows past
// `rows` are padding (code 8, scale 0: they contribute exact zeros).
// One 16-row tile: per pair of groups, four slabs of fragment-ordered nibbles, then the scales.
template <class Cd, class Sc>
void fill_one_tile(int tile, int pairs, std::vector<uint8_t>* out, const Cd& cd, const Sc& sc) {
    for (int pp = 0; pp < pairs; ++pp) {
        uint8_t* blk = out->data() + (static_cast<size_t>(tile) * pairs + pp) * kMmaUnitBytes;
        for (int sl = 0; sl < 4; ++sl) {
            const int col = 128 * pp + 32 * sl;
            for (int L = 0; L < 32; ++L) {
                const int r = 16 * tile + (L >> 2), c0 = col + (L & 3) * 4;
                for (int j = 0; j < 4; ++j) {
                    blk[sl * 256 + 8 * L + j] = static_cast<uint8_t>(cd(r, c0 + j) | (cd(r + 8, c0 + j) << 4));
                    blk[sl * 256 + 8 * L + 4 + j] =
                        static_cast<uint8_t>(cd(r, c0 + 16 + j) | (cd(r + 8, c0 + 16 + j) << 4));
                }
            }
        }
        __half* s = reinterpret_cast<__half*>(blk + 1024);
        for (int rr = 0; rr < 8; ++rr) {
            const int r = 16 * tile + rr;
            s[4 * rr] = sc(r, 2 * pp);
            s[4 * rr + 1] = sc(r, 2 * pp + 1);
            s[4 * rr + 2] = sc(r + 8, 2 * pp);
            s[4 * rr + 3] = sc(r + 8, 2 * pp + 1);
        }
    }
}

// Tiles are independent: host threads take contiguous ranges of them (a 9B package is ~8e9
// codes, tens of seconds on one core).
template <class Code, class Scale>
void fill_tiles(int rows, int K, Code code, Scale scale, std::vector<uint8_t>* out) {
    const int pairs = K / 128, ntiles = (rows + 15) / 16;
    out->assign(static_cast<size_t>(ntiles) * pairs * kMmaUnitBytes, 0);
    auto cd = [&](int r, int c) -> uint32_t { return r < rows ? code(r, c) : 8u; };
    auto sc = [&](int r, int g) -> __half { return r < rows ? scale(r, g) : __float2half_rn(0.0f); };
    auto fill_range = [&](int t0, int t1) {
        for (int tile = t0; tile < t1; ++tile) fill_one_tile(tile, pairs, out, cd, sc);
    };
    const int hw = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
    const int nthreads = std::max(1, std::min({hw, 64, ntiles / 256}));
    if (nthreads == 1) {
        fill_range(0, ntiles);
        return;
    }
    std::vector<std::thread> pool;
    for (int k = 0; k < nthreads; ++k)
        pool.emplace_back(fill_range, static_cast<int>(static_cast<long long>(ntiles) * k / nthreads),
                          static_cast<int>(static_cast<long long>(ntiles) * (k + 1) / nthreads));
    for (std::thread& t : pool) t.join();
}


bool upload_tiles(const std::vector<uint8_t>& t, uint8_t** dst, std::string* error) {
    if (cudaMalloc(dst, t.size()) != cudaSuccess ||
        cudaMemcpy(*dst, t.data(), t.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(*dst);
        *dst = nullptr;
        *error = "tensor-core tile upload failed";
        return false;
    }
    return true;
}

}  // namespace

bool build_mma_matrix(const HostMatrix& h, MmaMatrix* out, std::string* error) {
    *out = MmaMatrix();
    if (!mma_eligible(h)) {
        *error = "matrix not served by the tensor-core GEMV (symmetric fp16-scale xq4 v1, group 64, "
                 "cols a multiple of 512, and of 4096 above 4096)";
        return false;
    }
    const int K = h.cols, gpr = K / 64;
    std::vector<uint8_t> t;
    fill_tiles(
        h.rows, K,
        [&](int r, int c) -> uint32_t {
            const uint8_t b = h.packed[static_cast<size_t>(r) * (K / 2) + c / 2];
            return (c & 1) ? (b >> 4) : (b & 15u);
        },
        [&](int r, int g) { return __float2half_rn(h.scales[static_cast<size_t>(r) * gpr + g]); }, &t);
    out->rows = h.rows;
    out->cols = K;
    out->ntiles = (h.rows + 15) / 16;
    out->pairs = K / 128;
    out->bytes = t.size();
    return upload_tiles(t, &out->d_tiles, error);
}

bool attach_mma_tiles(const std::vector<uint8_t>& rows_host, DevMatrix* m, std::string* error) {
    if (m->kind != 0 || m->group != 64 || m->cols % 1024 != 0 ||
        rows_host.size() != static_cast<size_t>(m->rows) * m->row_stride) {
        *error = "tensor-core tiles need a symmetric (fp16 scale) row-layout matrix with cols a multiple of 1024";
        return false;
    }
    const int K = m->cols, stride = m->row_stride, meta = m->meta_offset;
    const uint8_t* base = rows_host.data();
    std::vector<uint8_t> t;
    fill_tiles(
        m->rows, K,
        [&](int r, int c) -> uint32_t {
            const uint8_t b = base[static_cast<size_t>(r) * stride + c / 2];
            return (c & 1) ? (b >> 4) : (b & 15u);
        },
        [&](int r, int g) {
            __half h;
            std::memcpy(&h, base + static_cast<size_t>(r) * stride + meta + 2 * g, 2);
            return h;
        },
        &t);
    cudaFree(m->d_tiles);
    m->d_tiles = nullptr;
    if (!upload_tiles(t, &m->d_tiles, error)) return false;
    m->tile_bytes = t.size();
    return true;
}

bool host_mma_tiles(const uint8_t* packed, const float* scales, int rows, int cols, std::vector<uint8_t>* out) {
    if (!packed || !scales || rows <= 0 || cols <= 0 || cols % 128 != 0) return false;
    const int K = cols, gpr = K / 64;
    fill_tiles(
        rows, K,
        [&](int r, int c) -> uint32_t {
            const uint8_t b = packed[static_cast<size_t>(r) * (K / 2) + c / 2];
            return (c & 1) ? (b >> 4) : (b & 15u);
        },
        [&](int r, int g) { return __float2half_rn(scales[static_cast<size_t>(r) * gpr + g]); }, out);
    return true;
}

void free_mma_matrix(MmaMatrix* m) {
    cudaFree(m->d_tiles);
    *m = MmaMatrix();
}

bool mma_init_device() {
    XQB_CUDA_OK(cudaFuncSetAttribute(gemv_mma_kernel<float, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     227 * 1024));
    XQB_CUDA_OK(cudaFuncSetAttribute(gemv_mma_kernel<__half, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     227 * 1024));
    return true;
}

namespace {
template <typename XT, typename YT>
bool launch_mma_gemv_t(const MmaMatrix& m, const XT* x, YT* y, unsigned* err, int num_sms, cudaStream_t s, bool pdl) {
    MmaParams<XT, YT> p = {};
    p.tiles = m.d_tiles;
    p.x = x;
    p.y = y;
    p.rows = m.rows;
    p.cols = m.cols;
    p.ntiles = m.ntiles;
    p.pairs = m.pairs;
    p.ppc = std::min(32, m.pairs);
    p.cpt = m.pairs / p.ppc;
    p.err = err;
    const size_t fixed = kOffFixed + ((table_bytes(m.cols) + 127) & ~static_cast<size_t>(127));
    const size_t slot = static_cast<size_t>(p.ppc) * kMmaUnitBytes;
    const size_t budget = 227 * 1024 - 1024;
    p.nslots = static_cast<int>(std::min<size_t>(kMmaMaxSlots, (budget - fixed) / slot));
    if (p.nslots < 2) {
        set_last_error("tensor-core GEMV: shared memory too small for this width");
        return false;
    }
    const size_t smem = fixed + slot * p.nslots;
    const int grid = std::max(1, std::min(num_sms, m.ntiles));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_mma_kernel<XT, YT>, p);
    if (e != cudaSuccess) {
        set_last_error(std::string("tensor-core GEMV launch failed: ") + cudaGetErrorString(e));
        return false;
    }
    return true;
}
}  // namespace

bool launch_mma_gemv(const MmaMatrix& m, const float* x, float* y, unsigned* err, int num_sms, cudaStream_t s,
                     bool pdl) {
    return launch_mma_gemv_t(m, x, y, err, num_sms, s, pdl);
}

bool launch_mma_gemv_f16(const MmaMatrix& m, const __half* x, __half* y, unsigned* err, int num_sms, cudaStream_t s,
                         bool pdl) {
    return launch_mma_gemv_t(m, x, y, err, num_sms, s, pdl);
}

}  // namespace xqb
