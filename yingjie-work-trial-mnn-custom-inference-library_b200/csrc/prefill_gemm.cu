// W4A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for batched prefill:
// Y[t][n] = sum_k X[t][k] * W[n][k], W int4 group-64 symmetric (fp16 scale, zero 8) in the
// device row layout, X bf16 [M][K] row-major, fp32 accumulation in tensor memory.
//
// The reference builds the KV cache token by token (CustomModel::prefill, custom_model.cpp:
// 610-640, one gemvW4A16Neon per matrix per token, xq_gemv_w4a16_neon.cpp:259-291). Here every
// projection of a layer runs once over all prompt tokens as one GEMM.
//
// One CTA per SM, persistent over output tiles of 128 weight rows x NT tokens, warp-specialised:
//   warp 0      TMA producer: per 64-column K block, the X tile (128-byte swizzle, the UMMA
//               canonical K-major layout) and the raw int4 codes + fp16 scales of 128 rows
//               (plain 2-D tensor copies of the row layout);
//   warp 1      allocates tensor memory; lane 0 issues tcgen05.mma (M = 128, N = NT, K = 16,
//               four per K block) and tcgen05.commit to the mbarriers;
//   warps 2-5   dequantise: thread r turns row r's 64 codes into (code - 8) * scale, rounded to
//               bf16 (split mode: also the bf16 residual), written into the A tile in the same
//               swizzled K-major layout, then a generic -> async proxy fence;
//   warps 6-9   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32 (w % 4) ..),
//               stores (or adds into) Y, token-major, coalesced along the weight rows.
// Two accumulators (2 x NT TMEM columns) let the epilogue of one tile overlap the next tile's
// MMAs. Split mode (exact to ~2^-16): W = W_hi + W_lo exactly (a 4-bit code times an fp16 scale
// has at most 15 significant bits), X = X_hi + X_lo, and the products W_hi X_hi + W_lo X_hi +
// W_hi X_lo are accumulated by three MMA chains into the same accumulator.
//
// Every wait is bounded (error word + time limit); after a timeout the roles fall through their
// loops, the MMA warp drains its last commit (bounded) and tensor memory is released.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "prefill_gemm.hpp"

namespace xqb {

namespace {

constexpr int kPgThreads = 320;  // 10 warps
constexpr int kPgRows = 128;     // weight rows per tile (UMMA M)
constexpr int kPgKb = 64;        // K per block (one group, one 128-byte swizzle row of bf16)
constexpr int kPgLoadStages = 4;
constexpr int kPgCodeBytes = kPgRows * 32;   // 64 codes per row
constexpr int kPgScaleBytes = kPgRows * 16;  // 8 groups' fp16 scales per row (one 16-byte box)

template <bool SPLIT, int NT>
struct PgCfg {
    static constexpr int kXBytes = NT * 128;                        // one bf16 X tile
    static constexpr int kXStage = kXBytes * (SPLIT ? 2 : 1);
    static constexpr int kABytes = kPgRows * 128;                   // one bf16 A tile (16 KB)
    static constexpr int kAStage = kABytes * (SPLIT ? 2 : 1);
    static constexpr int kAStages = SPLIT ? 2 : 3;
    static constexpr int kOffX = 0;
    static constexpr int kOffA = kOffX + kPgLoadStages * kXStage;
    static constexpr int kOffW = kOffA + kAStages * kAStage;
    static constexpr int kWStage = kPgCodeBytes + kPgScaleBytes;
    static constexpr int kOffBar = kOffW + kPgLoadStages * kWStage;
    static constexpr int kSmem = kOffBar + 256 + 1024;  // barriers + alignment slack
    static constexpr uint32_t kTmemCols = 2 * NT;       // two accumulators
    static_assert(kSmem <= 227 * 1024, "prefill GEMM shared memory");
    static_assert(kOffA % 1024 == 0 && kABytes % 1024 == 0 && kXBytes % 1024 == 0, "swizzle atoms");
    static_assert(NT == 128 || NT == 256, "token tile");
};

// ---- tcgen05 / TMA wrappers ---------------------------------------------------------------
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulator).
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte swizzle layout:
// rows of 128 bytes, 8-row atoms 1024 bytes apart (stride byte offset), version 1 (sm_100),
// layout type 2 (SWIZZLE_128B). The K step inside the atom advances the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;             // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;     // stride byte offset: 8-row atoms
    d |= static_cast<uint64_t>(1u) << 46;             // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
    return d;
}
// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

template <bool SPLIT, int NT>
__global__ void __launch_bounds__(kPgThreads, 1) prefill_gemm_kernel(const __grid_constant__ PgParams p) {
    using C = PgCfg<SPLIT, NT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* load_full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint64_t* load_empty = load_full + kPgLoadStages;
    uint64_t* a_full = load_empty + kPgLoadStages;
    uint64_t* a_empty = a_full + 4;
    uint64_t* acc_full = a_empty + 4;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t wait_ns = p.wait_ns ? p.wait_ns : kWaitLimitNs;
    const int mtiles = (p.M + NT - 1) / NT;
    const int ntiles = (p.N + kPgRows - 1) / kPgRows;
    const int tiles = mtiles * ntiles;
    const int kblocks = p.K / kPgKb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPgLoadStages; ++s) {
            mbar_init(&load_full[s], 1);
            mbar_init(&load_empty[s], 4 + 1);  // four dequant warps + the MMA commit
        }
        for (int s = 0; s < C::kAStages; ++s) {
            mbar_init(&a_full[s], 4);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        fence_mbar_init();
    }
    if (warp == 1) {  // the whole warp allocates (and later frees) the accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t g = 0;
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                const int n0 = (tile / mtiles) * kPgRows, m0 = (tile % mtiles) * NT;
                for (int kb = 0; kb < kblocks; ++kb, ++g) {
                    const int s = g % kPgLoadStages;
                    if (g >= kPgLoadStages &&
                        !mbar_wait_bounded(&load_empty[s], ((g / kPgLoadStages) - 1) & 1, p.err, wait_ns))
                        goto producer_done;
                    uint8_t* xs = smem + C::kOffX + s * C::kXStage;
                    uint8_t* ws = smem + C::kOffW + s * C::kWStage;
                    mbar_expect_tx(&load_full[s], C::kXStage + C::kWStage);
                    tma_2d(xs, &p.map_x, kb * kPgKb, m0, &load_full[s]);
                    if constexpr (SPLIT) tma_2d(xs + C::kXBytes, &p.map_x_lo, kb * kPgKb, m0, &load_full[s]);
                    tma_2d(ws, &p.map_codes, kb * 32, n0, &load_full[s]);
                    tma_2d(ws + kPgCodeBytes, &p.map_scales, p.meta_offset + 16 * (kb >> 3), n0, &load_full[s]);
                }
            }
        producer_done:
            // every issued copy lands before the CTA can exit (bounded, independent of errors)
            for (uint32_t k = g > kPgLoadStages ? g - kPgLoadStages : 0; k < g; ++k)
                mbar_wait_drain(&load_full[k % kPgLoadStages], (k / kPgLoadStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc(kPgRows, NT);
            uint32_t g = 0, ga = 0, it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
                const uint32_t b = it & 1;
                if (it >= 2) ok = mbar_wait_bounded(&acc_empty[b], ((it >> 1) - 1) & 1, p.err, wait_ns);
                tc_fence_after();
                const uint32_t d = tmem + b * NT;
                for (int kb = 0; kb < kblocks && ok; ++kb, ++g, ++ga) {
                    const int s = g % kPgLoadStages, as = ga % C::kAStages;
                    ok = mbar_wait_bounded(&load_full[s], (g / kPgLoadStages) & 1, p.err, wait_ns) &&
                         mbar_wait_bounded(&a_full[as], (ga / C::kAStages) & 1, p.err, wait_ns);
                    tc_fence_after();
                    const uint32_t xa = smem_u32(smem + C::kOffX + s * C::kXStage);
                    const uint32_t aa = smem_u32(smem + C::kOffA + as * C::kAStage);
#pragma unroll
                    for (int k = 0; k < kPgKb / 16; ++k) {  // 32 bytes of K per MMA
                        tc_mma(d, sw128_desc(aa + 32 * k), sw128_desc(xa + 32 * k), idesc, (kb | k) != 0);
                        if constexpr (SPLIT) {
                            tc_mma(d, sw128_desc(aa + C::kABytes + 32 * k), sw128_desc(xa + 32 * k), idesc, 1u);
                            tc_mma(d, sw128_desc(aa + 32 * k), sw128_desc(xa + C::kXBytes + 32 * k), idesc, 1u);
                        }
                    }
                    tc_commit(&load_empty[s]);
                    tc_commit(&a_empty[as]);
                }
                tc_commit(&acc_full[b]);
            }
            // the last commit tracks every MMA this thread issued: wait for it before the
            // accumulators are freed
            if (it > 0) mbar_wait_drain(&acc_full[(it - 1) & 1], ((it - 1) >> 1) & 1);
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- dequantise ----------------
        const int row = threadIdx.x - 64;  // 0..127
        const uint32_t row_off = static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128);
        uint32_t g = 0, ga = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            for (int kb = 0; kb < kblocks && ok; ++kb, ++g, ++ga) {
                const int s = g % kPgLoadStages, as = ga % C::kAStages;
                ok = mbar_wait_bounded(&load_full[s], (g / kPgLoadStages) & 1, p.err, wait_ns);
                if (ok && ga >= C::kAStages)
                    ok = mbar_wait_bounded(&a_empty[as], ((ga / C::kAStages) - 1) & 1, p.err, wait_ns);
                const uint8_t* ws = smem + C::kOffW + s * C::kWStage;
                const uint4 c0 = *reinterpret_cast<const uint4*>(ws + row * 32);
                const uint4 c1 = *reinterpret_cast<const uint4*>(ws + row * 32 + 16);
                const __half sh = *reinterpret_cast<const __half*>(ws + kPgCodeBytes + row * 16 + 2 * (kb & 7));
                const float sc = __half2float(sh);
                uint8_t* at = smem + C::kOffA + as * C::kAStage + row_off;
                const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int w = 0; w < 8; ++w) {  // word w: columns 8w .. 8w + 7 (one 16-byte chunk)
                    const uint32_t lo = words[w] & 0x0F0F0F0Fu, hi = (words[w] >> 4) & 0x0F0F0F0Fu;
                    uint32_t ph[4], pl[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        // 2^23 + code as a float (byte permute), minus 2^23 + 8: code - 8 exactly
                        const float e = (__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + i)) - 8388616.0f) * sc;
                        const float o = (__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + i)) - 8388616.0f) * sc;
                        ph[i] = bf16x2_rn(e, o);
                        if constexpr (SPLIT) pl[i] = bf16x2_rn(e - bf16_lo(ph[i]), o - bf16_hi(ph[i]));
                    }
                    const uint32_t off = static_cast<uint32_t>((w ^ (row & 7)) << 4);
                    *reinterpret_cast<uint4*>(at + off) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
                    if constexpr (SPLIT) *reinterpret_cast<uint4*>(at + C::kABytes + off) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
                }
                fence_async_smem();  // generic-proxy writes -> visible to the tensor cores
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&load_empty[s]);
                    mbar_arrive(&a_full[as]);
                }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
            const int n0 = (tile / mtiles) * kPgRows, m0 = (tile % mtiles) * NT;
            const uint32_t b = it & 1;
            ok = mbar_wait_bounded(&acc_full[b], (it >> 1) & 1, p.err, wait_ns);
            tc_fence_after();
            const int row = n0 + 32 * q + lane;
#pragma unroll 1
            for (int c = 0; c < NT / 32; ++c) {
                uint32_t r[32];
                tc_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * NT + 32 * c, r);
                if (row < p.N) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int t = m0 + 32 * c + j;
                        if (t < p.M) {
                            const size_t o = static_cast<size_t>(t) * p.ldy + row;
                            const float v = __uint_as_float(r[j]);
                            if (p.out_kind == kPgOutF32) p.y_f32[o] = v;
                            else if (p.out_kind == kPgOutAddF32) p.y_f32[o] += v;
                            else p.y_bf16[o] = __float2bfloat16_rn(v);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    return encode;
}

// 2-D tiled tensor map: inner extent `inner` elements, `outer` rows `stride_bytes` apart.
bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
               uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool SPLIT, int NT>
cudaError_t launch_t(const PgParams& p, int num_sms, cudaStream_t s) {
    using C = PgCfg<SPLIT, NT>;
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t attr_err = cudaSuccess;
    std::call_once(once[dev & 63], [&] {
        attr_err = cudaFuncSetAttribute(prefill_gemm_kernel<SPLIT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::kSmem);
    });
    if (attr_err != cudaSuccess) return attr_err;
    const int tiles = ((p.M + NT - 1) / NT) * ((p.N + kPgRows - 1) / kPgRows);
    const int grid = std::max(1, std::min(num_sms, tiles));
    prefill_gemm_kernel<SPLIT, NT><<<grid, kPgThreads, C::kSmem, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool launch_prefill_gemm(const DevMatrix& w, const __nv_bfloat16* x, const __nv_bfloat16* x_lo, int M, void* y,
                         int ldy, int out_kind, unsigned* err, int num_sms, cudaStream_t s, uint64_t wait_ns) {
    if (w.kind != 0 || w.group != 64 || !w.d_rows || w.cols % kPgKb != 0 || M <= 0 || !x || !y ||
        (w.row_stride % 16) != 0 || (w.meta_offset % 16) != 0 || ldy < w.rows ||
        (reinterpret_cast<uintptr_t>(x) & 15u) || (x_lo && (reinterpret_cast<uintptr_t>(x_lo) & 15u)) ||
        out_kind < kPgOutF32 || out_kind > kPgOutBF16) {
        set_last_error("prefill GEMM: needs a symmetric row-layout matrix (group 64), K a multiple of 64, 16-byte "
                       "aligned bf16 activations and ldy >= rows");
        return false;
    }
    PgParams p = {};
    const int K = w.cols;
    const bool split = x_lo != nullptr;
    const int NT = split ? 128 : 256;
    bool ok = encode_2d(&p.map_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, 2ull * K, kPgKb, NT,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
              (!split || encode_2d(&p.map_x_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x_lo, K, M, 2ull * K, kPgKb, NT,
                                   CU_TENSOR_MAP_SWIZZLE_128B)) &&
              encode_2d(&p.map_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.d_rows, w.row_stride, w.rows, w.row_stride, 32,
                        kPgRows, CU_TENSOR_MAP_SWIZZLE_NONE) &&
              encode_2d(&p.map_scales, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.d_rows, w.row_stride, w.rows, w.row_stride,
                        16, kPgRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ok) {
        set_last_error("prefill GEMM: tensor map encoding failed");
        return false;
    }
    p.M = M;
    p.N = w.rows;
    p.K = K;
    p.meta_offset = w.meta_offset;
    p.ldy = ldy;
    p.out_kind = out_kind;
    p.y_f32 = static_cast<float*>(y);
    p.y_bf16 = static_cast<__nv_bfloat16*>(y);
    p.err = err;
    p.wait_ns = wait_ns;
    const cudaError_t e = split ? launch_t<true, 128>(p, num_sms, s) : launch_t<false, 256>(p, num_sms, s);
    if (e != cudaSuccess) {
        set_last_error(std::string("prefill GEMM launch failed: ") + cudaGetErrorString(e));
        return false;
    }
    return true;
}

}  // namespace xqb
