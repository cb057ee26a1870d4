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
//   warp 1      allocates tensor memory; one elected lane issues tcgen05.mma (M = 128, N = NT,
//               K = 16, four per K block) and tcgen05.commit to the mbarriers;
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
#include <cstdlib>
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
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
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

// The issuing roles (TMA producer, MMA) run their loops with the whole warp in uniform control
// flow and let one elected lane issue each instruction (elect.sync inside the same asm
// statement): the descriptors and coordinates stay warp-uniform, which a loop run by a single
// divergent lane does not give, and a single lane issuing tcgen05.mma measured about 4x slower
// per instruction at small N (about 155 vs 40 cycles) and 20 % slower at N = 256.
__device__ __forceinline__ void tma_2d_elect(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "{ .reg .pred e; elect.sync _|e, 0xffffffff; @e cp.async.bulk.tensor.2d.shared::cluster.global.tile."
        "mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4]; }" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void expect_tx_elect(uint64_t* bar, uint32_t bytes) {
    asm volatile("{ .reg .pred e; elect.sync _|e, 0xffffffff; @e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1; }" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void tc_mma_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p, e; setp.ne.b32 p, %4, 0; elect.sync _|e, 0xffffffff; "
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T (A: 128 lanes = rows, 8 columns of bf16 pairs = K 16).
__device__ __forceinline__ void tc_mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p, e; setp.ne.b32 p, %4, 0; elect.sync _|e, 0xffffffff; "
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit_elect(uint64_t* bar) {
    asm volatile(
        "{ .reg .pred e; elect.sync _|e, 0xffffffff; "
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0]; }" ::"r"(smem_u32(bar))
        : "memory");
}
// A bounded wait by every lane of a warp, made warp-uniform (all lanes continue only if all saw
// the phase complete), so the warp's loop never diverges.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned* err, uint64_t limit_ns) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, err, limit_ns));
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

// tcgen05.ld of N consecutive accumulator columns of this thread's TMEM lane (no wait).
template <int N>
__device__ __forceinline__ void tc_ld_cols(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tc_ld_cols<8>(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
template <>
__device__ __forceinline__ void tc_ld_cols<16>(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 consecutive columns of this thread's TMEM lane from registers (no wait).
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- thread-block cluster helpers (small-M split-K) -----------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
// Arrive on an mbarrier of CTA `rank`, releasing this thread's earlier writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(dsmem_addr(bar, rank))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (the arrivals come from other CTAs of the cluster).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned* err, uint64_t limit_ns) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (!wait_budget_left(t0, i, err, limit_ns)) return false;
    }
}
// As mbar_wait_cluster, independent of the error bit (the exit path after an error).
__device__ __forceinline__ void mbar_drain_cluster(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait_cluster(bar, parity))
        if (global_ns() - t0 > kWaitLimitNs) return;
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
        // ---------------- producer (whole warp, one elected lane issues) ----------------
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int n0 = (tile / mtiles) * kPgRows, m0 = (tile % mtiles) * NT;
            for (int kb = 0; kb < kblocks; ++kb, ++g) {
                const int s = g % kPgLoadStages;
                if (g >= kPgLoadStages && !warp_wait(&load_empty[s], ((g / kPgLoadStages) - 1) & 1, p.err, wait_ns))
                    goto producer_done;
                uint8_t* xs = smem + C::kOffX + s * C::kXStage;
                uint8_t* ws = smem + C::kOffW + s * C::kWStage;
                expect_tx_elect(&load_full[s], C::kXStage + C::kWStage);
                tma_2d_elect(xs, &p.map_x, kb * kPgKb, m0, &load_full[s]);
                if constexpr (SPLIT) tma_2d_elect(xs + C::kXBytes, &p.map_x_lo, kb * kPgKb, m0, &load_full[s]);
                tma_2d_elect(ws, &p.map_codes, kb * 32, n0, &load_full[s]);
                tma_2d_elect(ws + kPgCodeBytes, &p.map_scales, p.meta_offset + 16 * (kb >> 3), n0, &load_full[s]);
            }
        }
    producer_done:
        // every issued copy lands before the CTA can exit (bounded, independent of errors)
        for (uint32_t k = g > kPgLoadStages ? g - kPgLoadStages : 0; k < g; ++k)
            mbar_wait_drain(&load_full[k % kPgLoadStages], (k / kPgLoadStages) & 1);
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (whole warp, one elected lane issues) ----------------
        constexpr uint32_t idesc = f16_idesc(kPgRows, NT);
        uint32_t g = 0, ga = 0, it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
            const uint32_t b = it & 1;
            if (it >= 2) ok = warp_wait(&acc_empty[b], ((it >> 1) - 1) & 1, p.err, wait_ns);
            tc_fence_after();
            const uint32_t d = tmem + b * NT;
            for (int kb = 0; kb < kblocks && ok; ++kb, ++g, ++ga) {
                const int s = g % kPgLoadStages, as = ga % C::kAStages;
                ok = warp_wait(&load_full[s], (g / kPgLoadStages) & 1, p.err, wait_ns) &&
                     warp_wait(&a_full[as], (ga / C::kAStages) & 1, p.err, wait_ns);
                if (!ok) break;
                tc_fence_after();
                const uint32_t xa = smem_u32(smem + C::kOffX + s * C::kXStage);
                const uint32_t aa = smem_u32(smem + C::kOffA + as * C::kAStage);
#pragma unroll
                for (int k = 0; k < kPgKb / 16; ++k) {  // 32 bytes of K per MMA
                    tc_mma_elect(d, sw128_desc(aa + 32 * k), sw128_desc(xa + 32 * k), idesc, (kb | k) != 0);
                    if constexpr (SPLIT) {
                        tc_mma_elect(d, sw128_desc(aa + C::kABytes + 32 * k), sw128_desc(xa + 32 * k), idesc, 1u);
                        tc_mma_elect(d, sw128_desc(aa + 32 * k), sw128_desc(xa + C::kXBytes + 32 * k), idesc, 1u);
                    }
                }
                tc_commit_elect(&load_empty[s]);
                tc_commit_elect(&a_empty[as]);
            }
            tc_commit_elect(&acc_full[b]);
        }
        // the last commit tracks every MMA the elected lane issued: wait for it before the
        // accumulators are freed
        if (it > 0) mbar_wait_drain(&acc_full[(it - 1) & 1], ((it - 1) >> 1) & 1);
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

// ---- small M (batched decode, short prefill chunks) ------------------------------------------
// With few tokens the kernel above is bound by its dequantisation (fp32 scale math per weight,
// plus the bf16 residual in split mode) and by its MMA width (N = 128 for a handful of tokens),
// and a 4096-row matrix gives it 32 tiles for 148 SMs. Here:
//   * A holds the exact integers (code - 8) as bf16, built with byte permutes and one bf16x2
//     subtract per weight pair, and lives in tensor memory (tcgen05.st by the converter warps,
//     MMA with A from TMEM): a bf16 A tile in shared memory (written once, read once by the
//     tensor cores) would cost 4 bytes of shared-memory traffic per weight and bound the kernel
//     at the shared-memory bandwidth; no scale is applied to A;
//   * each 64-column K block (one quantisation group) is multiplied into its own TMEM
//     accumulator; the accumulator warps fold it into fp32 registers as
//     acc += scale(row, group) * (W X_hi + W X_lo), so W is exact and the error is X's split;
//   * X_hi and X_lo sit in one B tile of 2 NT rows: one MMA (M = 128, N = 2 NT, K = 16) per
//     16 columns computes both products;
//   * the pipeline moves several K blocks per step (four at NT = 16, else two; one wait and one
//     commit per barrier per step): the barrier operations of a step cost the issuing warp about
//     as much as eight MMAs, so they are amortised over 16 (or 8) MMAs;
//   * split-K over a thread-block cluster of S CTAs: CTA r of the cluster takes steps
//     [r steps / S, (r + 1) steps / S) of the cluster's row tiles; the partial tiles meet in
//     distributed shared memory and CTA r sums rows [r 128 / S, (r + 1) 128 / S) over the S
//     partials in rank order (deterministic; no global workspace, no atomics).
// Roles (19 warps): warp 0 TMA (X tiles + raw codes), warps 1 and 18 MMA issue (even and odd
// steps: one warp's barrier waits and commits overlap the other's MMAs; warp 1 also owns the
// tensor memory), warps 2-9 code conversion (warp w: TMEM lanes = rows 32 (w % 4) .., K blocks
// (w - 2) / 4, + 2, .. of the step), warps 10-17 accumulation (warp w: TMEM lanes 32 (w % 4) .., token
// half (w - 10) / 4) and the tile's output.
constexpr int kDgThreads = 608;  // 19 warps
constexpr int kDgConvWarps = 8;
constexpr int kDgAccWarps = 8;
constexpr int kDgTmemCols = 512;   // the whole tensor memory: accumulators + A stages

template <int NT>
struct DgCfg {
    // K blocks per pipeline step: four at NT = 16 (the barrier waits and commits of a step,
    // ~500 cycles, spread over 16 MMAs), two where four would not leave two steps in TMEM
    static constexpr int kKb = NT == 16 ? 4 : 2;
    static constexpr int kACols = kKb * 32;  // one A stage in TMEM: 128 lanes x kKb K blocks of bf16 pairs
    static constexpr int kAccBufs = NT == 64 ? 1 : 2;  // steps whose accumulators are in TMEM at once
    static constexpr int kAccCols = kAccBufs * kKb * 2 * NT;
    static constexpr int kAStages = (kDgTmemCols - kAccCols) / kACols;
    static constexpr int kLoadStages = NT == 64 ? 4 : 6;
    static constexpr int kXBytes = NT * 128;                    // one bf16 [NT][64] tile
    static constexpr int kXStage = 2 * kKb * kXBytes;          // [hi kb0 | lo kb0 | hi kb1 | lo kb1 | ..]
    static constexpr int kCodeStage = kKb * kPgCodeBytes;       // [kb][128 rows][32 bytes]
    static constexpr int kOffX = 0;
    static constexpr int kOffW = kOffX + kLoadStages * kXStage;
    static constexpr int kOffRed = kOffW + kLoadStages * kCodeStage;
    static constexpr int kRedBytes = kPgRows * NT * 4;          // [NT][128] fp32 partial tile
    static constexpr int kOffBar = kOffRed + kRedBytes;
    static constexpr int kSmem = kOffBar + 512 + 1024;
    static_assert(kSmem <= 227 * 1024, "small-M GEMM shared memory");
    static_assert(kXBytes % 1024 == 0, "swizzle atoms");
    static_assert(kAStages >= 2 && kAccCols + kAStages * kACols <= kDgTmemCols, "tensor memory budget");
};

// bf16x2 (128 + c0, 128 + c1) - (136, 136) = (c0 - 8, c1 - 8), exact.
__device__ __forceinline__ uint32_t bf16x2_sub136(uint32_t v) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&v);
    x = __hsub2(x, __floats2bfloat162_rn(136.0f, 136.0f));
    return *reinterpret_cast<uint32_t*>(&x);
}
// fp16 scale i (0..7) of a 16-byte group of eight.
__device__ __forceinline__ float scale_at(const uint4& v, int i) {
    const uint32_t w = (i & 4) ? ((i & 2) ? v.w : v.z) : ((i & 2) ? v.y : v.x);
    const unsigned short h = static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xFFFFu));
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ void pg_store(const PgParams& p, int t, int n, float v) {
    const size_t o = static_cast<size_t>(t) * p.ldy + n;
    if (p.out_kind == kPgOutF32) p.y_f32[o] = v;
    else if (p.out_kind == kPgOutAddF32) p.y_f32[o] += v;
    else p.y_bf16[o] = __float2bfloat16_rn(v);
}

template <int NT>
__global__ void __launch_bounds__(kDgThreads, 1) decode_gemm_kernel(const __grid_constant__ PgParams p) {
    using C = DgCfg<NT>;
    constexpr int LS = C::kLoadStages, AS = C::kAStages, RB = C::kAccBufs, NH = NT / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* code_full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);  // raw codes of a load stage
    uint64_t* x_full = code_full + LS;                                       // its X tiles
    uint64_t* load_empty = x_full + LS;
    uint64_t* a_full = load_empty + LS;
    uint64_t* a_empty = a_full + AS;
    uint64_t* acc_full = a_empty + AS;
    uint64_t* acc_empty = acc_full + RB;
    uint64_t* red_full = acc_empty + RB;
    uint64_t* red_free = red_full + 1;
    uint64_t* exit_bar = red_free + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(exit_bar + 1);
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t wait_ns = p.wait_ns ? p.wait_ns : kWaitLimitNs;
    const uint32_t S = cluster_size(), rank = cluster_rank();
    const int cid = static_cast<int>(cluster_id()), ncl = static_cast<int>(cluster_count());
    const int mtiles = (p.M + NT - 1) / NT;
    const int tiles = mtiles * ((p.N + kPgRows - 1) / kPgRows);
    const int kblocks = p.K / kPgKb;
    constexpr int KB = C::kKb;
    const int steps = kblocks / KB;
    const int st0 = static_cast<int>(rank * steps / S), st1 = static_cast<int>((rank + 1) * steps / S);
    const bool split = p.split != 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < LS; ++s) {
            mbar_init(&code_full[s], 1);
            mbar_init(&x_full[s], 1);
            mbar_init(&load_empty[s], kDgConvWarps + 1);  // converter warps + the MMA commit
        }
        for (int s = 0; s < AS; ++s) {
            mbar_init(&a_full[s], kDgConvWarps);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < RB; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kDgAccWarps);
        }
        mbar_init(red_full, kDgAccWarps * 32 * S);  // every accumulator thread of every CTA
        mbar_init(red_free, kDgAccWarps * 32 * S);
        mbar_init(exit_bar, kDgAccWarps * 32 * S);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kDgTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (S > 1) cluster_sync_all();  // the peers' barriers are initialised before any remote arrive
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();  // the next kernel may be scheduled; it waits for this one itself

    if (warp == 0) {
        // ---------------- producer (whole warp, one elected lane issues) ----------------
        // The weight codes do not depend on the previous kernel in the stream: the first load
        // stages' codes are requested before waiting for it (programmatic dependent launch), so
        // the weight stream and the code conversion start during its tail; X only after.
        const int per_tile = st1 - st0;
        const int my_tiles = cid < tiles ? (tiles - 1 - cid) / ncl + 1 : 0;
        const uint32_t total = static_cast<uint32_t>(per_tile * my_tiles);
        const uint32_t xbytes = KB * (split ? 2 : 1) * C::kXBytes;
        auto tile_of = [&](uint32_t g) { return cid + static_cast<int>(g / per_tile) * ncl; };
        auto step_of = [&](uint32_t g) { return st0 + static_cast<int>(g % per_tile); };
        auto issue_codes = [&](uint32_t g) {
            const int s = g % LS, n0 = (tile_of(g) / mtiles) * kPgRows, st = step_of(g);
            expect_tx_elect(&code_full[s], C::kCodeStage);
#pragma unroll
            for (int j = 0; j < KB; ++j)
                tma_2d_elect(smem + C::kOffW + s * C::kCodeStage + j * kPgCodeBytes, &p.map_codes, (st * KB + j) * 32,
                             n0, &code_full[s]);
        };
        auto issue_x = [&](uint32_t g) {
            const int s = g % LS, m0 = (tile_of(g) % mtiles) * NT, st = step_of(g);
            uint8_t* xs = smem + C::kOffX + s * C::kXStage;
            expect_tx_elect(&x_full[s], xbytes);
#pragma unroll
            for (int j = 0; j < KB; ++j) {
                const int kb = st * KB + j;
                tma_2d_elect(xs + 2 * j * C::kXBytes, &p.map_x, kb * kPgKb, m0, &x_full[s]);
                if (split) tma_2d_elect(xs + (2 * j + 1) * C::kXBytes, &p.map_x_lo, kb * kPgKb, m0, &x_full[s]);
            }
        };
        const uint32_t pre = total < static_cast<uint32_t>(LS) ? total : static_cast<uint32_t>(LS);
        for (uint32_t g = 0; g < pre; ++g) issue_codes(g);
        pdl_wait();
        uint32_t gc = pre, gx = 0;
        for (uint32_t g = 0; g < total; ++g) {
            if (g >= pre) {
                if (g >= static_cast<uint32_t>(LS) && !warp_wait(&load_empty[g % LS], ((g / LS) - 1) & 1, p.err, wait_ns))
                    break;
                issue_codes(g);
                gc = g + 1;
            }
            issue_x(g);
            gx = g + 1;
        }
        // every issued copy lands before the CTA can exit (bounded, independent of errors)
        for (uint32_t q = gc > static_cast<uint32_t>(LS) ? gc - LS : 0; q < gc; ++q)
            mbar_wait_drain(&code_full[q % LS], (q / LS) & 1);
        for (uint32_t q = gx > static_cast<uint32_t>(LS) ? gx - LS : 0; q < gx; ++q)
            mbar_wait_drain(&x_full[q % LS], (q / LS) & 1);
        __syncwarp();
    } else if (warp == 1 || warp == 2 + kDgConvWarps + kDgAccWarps) {
        // ---------------- MMA issuers (whole warp, one elected lane issues) ----------------
        // warp 1 issues the even steps, the last warp the odd ones; each commits (and so tracks)
        // only its own MMAs.
        // With a single accumulator buffer one issuer could wait on acc_empty a full phase
        // ahead of the other, where a parity wait cannot tell the phases apart: warp 1 then
        // issues every step alone.
        constexpr bool kTwoIssuers = RB >= 2;
        const bool return_role = !kTwoIssuers && warp != 1;
        const uint32_t parity = warp == 1 ? 0u : 1u;
        const uint32_t idesc = f16_idesc(kPgRows, split ? 2 * NT : NT);
        uint32_t g = 0, last = 0;
        bool ok = true, any = false;
        for (int tile = cid; tile < tiles && ok; tile += ncl) {
            for (int st = st0; st < st1; ++st, ++g) {
                if (return_role || (kTwoIssuers && (g & 1u) != parity)) continue;
                const int s = g % LS, as = g % AS, b = g % RB;
                ok = warp_wait(&a_full[as], (g / AS) & 1, p.err, wait_ns) &&
                     warp_wait(&x_full[s], (g / LS) & 1, p.err, wait_ns) &&
                     (g < static_cast<uint32_t>(RB) || warp_wait(&acc_empty[b], ((g / RB) - 1) & 1, p.err, wait_ns));
                if (!ok) break;
                tc_fence_after();
                const uint32_t xa = smem_u32(smem + C::kOffX + s * C::kXStage);
                const uint32_t aa = tmem + static_cast<uint32_t>(C::kAccCols + as * C::kACols);
#pragma unroll
                for (int j = 0; j < KB; ++j) {
                    const uint32_t d = tmem + static_cast<uint32_t>((b * KB + j) * 2 * NT);
#pragma unroll
                    for (int k = 0; k < kPgKb / 16; ++k)  // 16 K = 8 TMEM columns of A
                        tc_mma_ts_elect(d, aa + j * 32 + 8 * k, sw128_desc(xa + 2 * j * C::kXBytes + 32 * k), idesc,
                                        k != 0);
                }
                tc_commit_elect(&load_empty[s]);
                tc_commit_elect(&a_empty[as]);
                tc_commit_elect(&acc_full[b]);
                last = g;
                any = true;
            }
        }
        if (any) mbar_wait_drain(&acc_full[last % RB], (last / RB) & 1);
        __syncwarp();
    } else if (warp < 2 + kDgConvWarps) {
        // ---------------- code conversion (into the TMEM A stage) ----------------
        const int q = warp & 3, j0 = (warp - 2) >> 2;  // TMEM lane quarter, first K block of the step
        const int row = 32 * q + lane;
        uint32_t g = 0;
        bool ok = true;
        for (int tile = cid; tile < tiles && ok; tile += ncl) {
            for (int st = st0; st < st1; ++st, ++g) {
                const int s = g % LS, as = g % AS;
                ok = mbar_wait_bounded(&code_full[s], (g / LS) & 1, p.err, wait_ns) &&
                     (g < static_cast<uint32_t>(AS) || mbar_wait_bounded(&a_empty[as], ((g / AS) - 1) & 1, p.err, wait_ns));
                if (!ok) break;
                tc_fence_after();  // the MMAs that read this A stage have completed (a_empty)
#pragma unroll 1
                for (int j = j0; j < KB; j += 2) {
                const uint8_t* cs = smem + C::kOffW + s * C::kCodeStage + j * kPgCodeBytes + row * 32;
                const uint4 c0 = *reinterpret_cast<const uint4*>(cs);
                const uint4 c1 = *reinterpret_cast<const uint4*>(cs + 16);
                const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                uint32_t a[32];  // TMEM column m = bf16 pair of K columns 2m, 2m + 1
#pragma unroll
                for (int w = 0; w < 8; ++w) {  // word w: columns 8w .. 8w + 7, byte i = columns 2i, 2i + 1
                    const uint32_t lo = words[w] & 0x0F0F0F0Fu, hi = (words[w] >> 4) & 0x0F0F0F0Fu;
                    const uint32_t c03 = __byte_perm(lo, hi, 0x5140);  // codes of columns 0..3 as bytes
                    const uint32_t c47 = __byte_perm(lo, hi, 0x7362);  // columns 4..7
                    // bf16 (128 + c) = 0x4300 | c: one byte permute per pair, then - 136
                    a[4 * w] = bf16x2_sub136(__byte_perm(c03, 0x43434343u, 0x4140));
                    a[4 * w + 1] = bf16x2_sub136(__byte_perm(c03, 0x43434343u, 0x4342));
                    a[4 * w + 2] = bf16x2_sub136(__byte_perm(c47, 0x43434343u, 0x4140));
                    a[4 * w + 3] = bf16x2_sub136(__byte_perm(c47, 0x43434343u, 0x4342));
                }
                tc_st32(tmem + (static_cast<uint32_t>(32 * q) << 16) +
                            static_cast<uint32_t>(C::kAccCols + as * C::kACols + j * 32),
                        a);
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&load_empty[s]);
                    mbar_arrive(&a_full[as]);
                }
            }
        }
    } else {
        // ---------------- accumulation + output ----------------
        pdl_wait();  // y (added into, or overwritten) may be the previous kernel's
        const int q = warp & 3, hcol = (warp - 2 - kDgConvWarps) >> 2;
        const int rl = 32 * q + lane;  // tile row of this thread
        const int at = threadIdx.x - 32 * (2 + kDgConvWarps);  // 0..255
        uint32_t g = 0, it = 0;
        bool ok = true;
        // with a cluster, every CTA runs the exchange for every tile, after an error too, so that
        // the barrier phases stay aligned and no peer is left waiting on this CTA
        for (int tile = cid; tile < tiles && (ok || S > 1); tile += ncl, ++it) {
            const int n0 = (tile / mtiles) * kPgRows, m0 = (tile % mtiles) * NT;
            const int n = n0 + rl;
            const uint8_t* meta = p.w_rows + static_cast<size_t>(min(n, p.N - 1)) * p.row_stride + p.meta_offset;
            const int last_grp = (kblocks - 1) >> 3;
            float acc[NH];
#pragma unroll
            for (int j = 0; j < NH; ++j) acc[j] = 0.0f;
            int gcur = (st0 * KB) >> 3;
            uint4 vcur = __ldg(reinterpret_cast<const uint4*>(meta + 16 * gcur));
            uint4 vnxt = __ldg(reinterpret_cast<const uint4*>(meta + 16 * min(gcur + 1, last_grp)));
            for (int st = st0; st < st1; ++st, ++g) {
                const int b = g % RB;
                ok = ok && mbar_wait_bounded(&acc_full[b], (g / RB) & 1, p.err, wait_ns);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < KB; ++j) {
                    const int kb = st * KB + j;
                    if ((kb >> 3) != gcur) {  // next 8 groups' scales; the following 8 prefetched
                        gcur = kb >> 3;
                        vcur = vnxt;
                        vnxt = __ldg(reinterpret_cast<const uint4*>(meta + 16 * min(gcur + 1, last_grp)));
                    }
                    const float sc = scale_at(vcur, kb & 7);
                    const uint32_t ta = tmem + (static_cast<uint32_t>(32 * q) << 16) +
                                        static_cast<uint32_t>((b * KB + j) * 2 * NT + hcol * NH);
                    constexpr int CH = NH > 16 ? 16 : NH;  // columns per TMEM load (register budget)
#pragma unroll
                    for (int c0 = 0; c0 < NH; c0 += CH) {
                        uint32_t vh[CH], vl[CH];
                        tc_ld_cols<CH>(ta + c0, vh);
                        if (split) tc_ld_cols<CH>(ta + NT + c0, vl);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            const float v = split ? __uint_as_float(vh[i]) + __uint_as_float(vl[i]) : __uint_as_float(vh[i]);
                            acc[c0 + i] = fmaf(sc, v, acc[c0 + i]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[b]);
            }
            if (S == 1) {
                if (ok && n < p.N) {
#pragma unroll
                    for (int j = 0; j < NH; ++j) {
                        const int t = m0 + hcol * NH + j;
                        if (t < p.M) pg_store(p, t, n, acc[j]);
                    }
                }
                continue;
            }
            // split-K: partial tile -> shared memory, then rows [rank 128/S, (rank+1) 128/S) summed
            // over the S CTAs' partials in rank order
            if (it > 0) ok = mbar_wait_cluster(red_free, (it - 1) & 1, p.err, wait_ns) && ok;
#pragma unroll
            for (int j = 0; j < NH; ++j) red[(hcol * NH + j) * kPgRows + rl] = acc[j];
            for (uint32_t r = 0; r < S; ++r) mbar_arrive_cluster(red_full, r);
            const bool full = mbar_wait_cluster(red_full, it & 1, p.err, wait_ns);
            if (full && ok) {
                const int r0 = static_cast<int>(rank * kPgRows / S), r1 = static_cast<int>((rank + 1) * kPgRows / S);
                const int rows = r1 - r0;
                for (int e = at; e < rows * NT; e += kDgAccWarps * 32) {
                    const int t = e / rows, row_l = r0 + e % rows;
                    const float* src = red + t * kPgRows + row_l;
                    float v = 0.0f;
                    for (uint32_t r = 0; r < S; ++r) v += ld_dsmem_f32(dsmem_addr(src, r));
                    if (n0 + row_l < p.N && m0 + t < p.M) pg_store(p, m0 + t, n0 + row_l, v);
                }
            }
            ok = ok && full;
            for (uint32_t r = 0; r < S; ++r) mbar_arrive_cluster(red_free, r);
        }
        // no CTA leaves while a peer may still read its partial tile or arrive on its barriers:
        // the exit barrier's single phase completes after every peer's last remote access
        if (S > 1) {
            for (uint32_t r = 0; r < S; ++r) mbar_arrive_cluster(exit_bar, r);
            mbar_drain_cluster(exit_bar, 0);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kDgTmemCols) : "memory");
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

int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

constexpr int kDgSplits[] = {1, 2, 3, 4, 6, 8};

// Small-M launch: the cluster size S (split-K factor) minimises waves x (steps per CTA + a
// per-tile overhead of about two steps) over the clusters that fit at once.
template <int NT>
cudaError_t launch_dg(const PgParams& p, int num_sms, cudaStream_t s) {
    using C = DgCfg<NT>;
    static std::once_flag once[64];
    static int fit[64][9];    // co-resident clusters per cluster size (0: unknown)
    static cudaError_t attr_err[64];
    int dev = 0;
    cudaGetDevice(&dev);
    dev &= 63;
    std::call_once(once[dev], [&] {
        attr_err[dev] = cudaFuncSetAttribute(decode_gemm_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        for (int S : kDgSplits) {
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = S;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.gridDim = dim3(S * std::max(1, num_sms / S));
            cfg.blockDim = dim3(kDgThreads);
            cfg.dynamicSmemBytes = C::kSmem;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            fit[dev][S] = (attr_err[dev] == cudaSuccess &&
                           cudaOccupancyMaxActiveClusters(&n, decode_gemm_kernel<NT>, &cfg) == cudaSuccess)
                              ? n
                              : 0;
        }
        cudaGetLastError();  // a refused query leaves no sticky error behind
    });
    if (attr_err[dev] != cudaSuccess) return attr_err[dev];
    const int tiles = ((p.M + NT - 1) / NT) * ((p.N + kPgRows - 1) / kPgRows);
    const int steps = p.K / (kPgKb * C::kKb);
    static const int forced = env_int("XQ_GEMM_KSPLIT", 0);
    int best_s = 1, best_cl = std::max(1, fit[dev][1] ? fit[dev][1] : num_sms);
    long best = -1;
    for (int S : kDgSplits) {
        if (forced > 0 && S != forced) continue;
        if (S > 1 && steps < 2 * S) continue;
        const int cl = fit[dev][S] > 0 ? fit[dev][S] : num_sms / S;
        if (cl < 1) continue;
        const long cost = static_cast<long>((tiles + cl - 1) / cl) * ((steps + S - 1) / S + 2);
        if (best < 0 || cost < best) {
            best = cost;
            best_s = S;
            best_cl = cl;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = best_s;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // weight codes before the wait
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(best_s * std::min(tiles, best_cl));
    cfg.blockDim = dim3(kDgThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = s;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, decode_gemm_kernel<NT>, p);
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
    static const bool small_m_kernel = env_int("XQ_GEMM_SMALL_M", 1) != 0;
    // widest token tile of the small-M kernel (16, 32 or 64); a narrower one covers M in several
    // token tiles whose CTAs share each weight tile through L2
    // (32 by default: at M = 64 two 32-token tiles with two accumulators in flight measured up to
    // 1.3x faster per layer matrix than one 64-token tile, which has room for one)
    static const int small_nt_max = env_int("XQ_GEMM_SMALL_NT_MAX", 32);
    const int small_nt = (!small_m_kernel || K % (kPgKb * 4) != 0) ? 0
                         : M <= 16                                     ? 16
                         : M <= 32 || (small_nt_max < 64 && M <= 64)   ? std::min(32, std::max(16, small_nt_max))
                         : M <= 64                                     ? 64
                                                                       : 0;
    const int NT = small_nt ? small_nt : split ? 128 : 256;
    bool ok = encode_2d(&p.map_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, 2ull * K, kPgKb, NT,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
              (!split || encode_2d(&p.map_x_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x_lo, K, M, 2ull * K, kPgKb, NT,
                                   CU_TENSOR_MAP_SWIZZLE_128B)) &&
              encode_2d(&p.map_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.d_rows, w.row_stride, w.rows, w.row_stride,
                        32, kPgRows, CU_TENSOR_MAP_SWIZZLE_NONE) &&
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
    p.w_rows = w.d_rows;
    p.row_stride = w.row_stride;
    p.split = split ? 1 : 0;
    const cudaError_t e = small_nt == 16   ? launch_dg<16>(p, num_sms, s)
                          : small_nt == 32 ? launch_dg<32>(p, num_sms, s)
                          : small_nt == 64 ? launch_dg<64>(p, num_sms, s)
                          : split          ? launch_t<true, 128>(p, num_sms, s)
                                           : launch_t<false, 256>(p, num_sms, s);
    if (e != cudaSuccess) {
        set_last_error(std::string("prefill GEMM launch failed: ") + cudaGetErrorString(e));
        return false;
    }
    return true;
}

}  // namespace xqb
