// Persistent decode-step kernel (see stepper.cuh).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "gemv.hpp"
#include "mma_gemv.hpp"
#include "ops_device.cuh"
#include "stepper.cuh"

namespace xqb {

namespace {

// Shared-memory layout (bytes):
//   [0, 128)      full mbarriers       [128, 256)    empty mbarriers
//   [256, 384)    warp sums            [384, 416)    activation / constant / 2 descriptor mbarriers
//   [512, 4608)   row sums: dp4a path [2][16][32]; tensor-core path [3 teams][2][4 warps][16]
//   [4608, 6912)  attention scratch    [6912, 8192)  3 DeltaNet scratches
//   [8192, 8704)  argmax scratch       [8704, 9728)  two phase descriptors
//   [10240, +48K) activation area: a GEMV phase's x and its second vector (norm weights or
//                 gate) as 128-byte rows with 128-byte swizzle (the tensor-core path then writes
//                 x's digit table over them), or an attention phase's q / scores
//   [.., +4K)     epilogue inputs of this block's rows (residual, conv weights and state)
//   then the weight ring (slot size StepParams::slot_bytes).
constexpr int kOffFull = 0, kOffEmpty = 128, kOffWsum = 256, kOffXBar = 384, kOffCBar = 392, kOffDBar = 400,
              kOffRed = 512, kOffAttn = 4608, kOffDelta = 6912, kOffArg = 8192, kOffDesc = kStepHeaderBytes;
constexpr int kDescBytes = 512;
constexpr int kMmaStepTeams = 3, kMmaStepWarpsPerTeam = 4;  // tensor-core phases: 12 consumer warps
static_assert(kMmaStepTeams * kMmaStepWarpsPerTeam * 32 == kStepConsumers, "tensor-core teams");
static_assert(kMmaStepSlotBytes % kMmaUnitBytes == 0, "tensor-core ring slot");
constexpr int kOffAct = 10240;  // 1024-byte aligned: 128-byte swizzled tensor copies land here
constexpr int kOffEpi = kOffAct + kStepActBytes;
constexpr int kOffRing = kOffEpi + 4 * kStepEpiFloats;
static_assert(sizeof(AttnScratch) <= kOffDelta - kOffAttn, "attention scratch");
static_assert(3 * sizeof(DeltaScratch) <= kOffArg - kOffDelta, "delta scratch");
static_assert(sizeof(PhaseDesc) % 16 == 0 && sizeof(PhaseDesc) <= kDescBytes, "phase descriptor copy");
static_assert(kStepAttnDynBytes <= kStepActBytes, "attention scratch aliases the activation area");
static_assert(kOffRing % 128 == 0, "ring alignment");
static_assert(kOffDesc + 2 * kDescBytes <= kOffAct && kOffAct % 1024 == 0, "activation area");

struct ArgScratch {
    float v[32];
    int i[32];
    int last;
    int token;
};
static_assert(sizeof(ArgScratch) <= kStepHeaderBytes - kOffArg, "argmax scratch");

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct Ctx {
    uint8_t* base;  // dynamic shared memory
    uint64_t* full;
    uint64_t* empty;
    uint64_t* xbar;  // activation copies of the current phase (completes once per phase)
    uint64_t* cbar;  // constant copies of the current phase (completes once per phase)
    float* wsum;
    float* red;
    float* act;
    float* epi;
    uint8_t* ring;
    int nslots;
    int slot_bytes;
    int tid, lane, warp;
    int gbase;   // chunks this block consumed in earlier phases
    uint32_t parity;  // of xbar / cbar in the current phase
    uint64_t wait_ns;  // limit of every bounded wait in this launch
};

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// This block's rows of a GEMV phase and the number of ring chunks they stream in. Tensor-core
// tiles: contiguous 16-row tiles (r_end clamped to the matrix), mma_pairs / mma_ppc chunks each.
__device__ __forceinline__ void block_rows(const GemvParams& p, int* r_begin, int* r_end, int* nchunks) {
    if (p.mma_pairs > 0) {
        const int tiles = (p.rows + 15) >> 4;
        const int t0 = static_cast<int>((long long)tiles * blockIdx.x / gridDim.x);
        const int t1 = static_cast<int>((long long)tiles * (blockIdx.x + 1) / gridDim.x);
        *r_begin = 16 * t0;
        *r_end = min(p.rows, 16 * t1);
        *nchunks = (t1 - t0) * (p.mma_pairs / p.mma_ppc);
        return;
    }
    const int units = p.rows / p.unit;
    *r_begin = static_cast<int>((long long)units * blockIdx.x / gridDim.x) * p.unit;
    *r_end = static_cast<int>((long long)units * (blockIdx.x + 1) / gridDim.x) * p.unit;
    *nchunks = (*r_end - *r_begin + p.rows_per_chunk - 1) / p.rows_per_chunk;
}

// The contiguous weight bytes of this block's rows, streamed in chunks of `cstride` bytes (the
// last one may be short in the row layout).
__device__ __forceinline__ void block_span(const GemvParams& p, int r_begin, int r_end, const uint8_t** base,
                                           size_t* cstride, size_t* len) {
    if (p.mma_pairs > 0) {
        const size_t unit = static_cast<size_t>(p.mma_pairs) * kMmaUnitBytes;  // one 16-row tile
        *base = p.w + static_cast<size_t>(r_begin >> 4) * unit;
        *cstride = static_cast<size_t>(p.mma_ppc) * kMmaUnitBytes;
        *len = static_cast<size_t>(((r_end + 15) >> 4) - (r_begin >> 4)) * unit;
        return;
    }
    *base = p.w + static_cast<size_t>(r_begin) * p.row_stride;
    *cstride = static_cast<size_t>(p.rows_per_chunk) * p.row_stride;
    *len = static_cast<size_t>(r_end - r_begin) * p.row_stride;
}

// Rows of this block whose epilogue inputs are staged in shared memory: [r0, r1), widened to
// multiples of 4 rows so that every copy starts and ends on a 16-byte boundary. `ok` is false
// (inputs read from global memory instead) when they do not fit the staging area.
struct EpiWindow {
    int r0, r1;
    bool ok;
};
__device__ __forceinline__ EpiWindow epi_window(const GemvParams& p, int epi, int r_begin, int r_end) {
    EpiWindow w{0, 0, false};
    if (r_begin >= r_end) return w;
    if (epi == kEpiResidual) {
        w.r0 = r_begin & ~3;
        w.r1 = min(p.rows, (r_end + 3) & ~3);
        w.ok = (p.rows & 3) == 0 && w.r1 - w.r0 <= kStepEpiFloats;
    } else if (epi == kEpiConv && r_begin < p.conv_channels) {
        w.r0 = r_begin & ~3;
        w.r1 = min(p.conv_channels, (r_end + 3) & ~3);
        w.ok = p.conv_k == 4 && (p.conv_channels & 3) == 0 && 7 * (w.r1 - w.r0) <= kStepEpiFloats;
    }
    return w;
}

// n fp32 values (n / 32 rows of 128 bytes) into dst by 2-D tensor copies of up to 32 rows;
// 128-byte swizzle: the 16-byte chunk j of row r lands at chunk j ^ (r & 7).
__device__ __forceinline__ void tma_vector(float* dst, const void* tmap, int n, uint64_t* bar, int lane = 0,
                                           int lanes = 1) {
    const int rows = n >> 5;
    const int box = min(32, rows);
    for (int r = lane * box; r < rows; r += lanes * box)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
            "[%4];" ::"r"(smem_u32(dst + 32 * r)),
            "l"(tmap), "r"(0), "r"(r), "r"(smem_u32(bar))
            : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- attention phase -----------------------------------------------------------------
// One (kv head, split) item per block (blocks beyond nkv * kAttnSplits idle), on all 12 consumer
// warps. Split sp covers positions [t0, t1) of the context 0 .. pos. Shared layout in the
// activation area: q [group][hd] fp32, then scores [group][chunk] fp32.
// (Staging the split's K / V rows into shared memory before the grid barrier was measured: the
// phase took 17.5 instead of 21.6 us, but the extra bulk copies slowed every GEMV loop of the
// step by 3-5 % and the step as a whole by 2 %, so the rows are read from global memory here.)
struct AttnLayout {
    int pos, t0, t1, n, chunk;
};
__device__ __forceinline__ AttnLayout attn_layout(const AttnParams& a, int split) {
    AttnLayout l;
    l.pos = a.pos_ptr ? __ldcg(a.pos_ptr) : a.pos_const;
    const int L = l.pos + 1;
    l.chunk = (L + kAttnSplits - 1) / kAttnSplits;
    l.t0 = min(L, split * l.chunk);
    l.t1 = min(L, l.t0 + l.chunk);
    l.n = l.t1 - l.t0;
    return l;
}

// The item (kv head kh, split): the arithmetic of attention_item (custom_model.cpp:740-753,
// 871-946) with the scores spread over all 12 warps, 8 V rows per memory round trip, and a merge
// by the last split of each kv head that requests every partial at once. Out of line: it runs
// 8 times per step and must not shape the register allocation of the inlined GEMV loops.
template <typename KV>
__device__ __noinline__ void attention_item_step(const AttnParams& p, int kh, int split, int tid, uint8_t* act,
                                                 AttnScratch* sh, unsigned* err, unsigned long long* ts) {
    constexpr int kThreads = kStepConsumers, kWarps = kThreads / 32;
    const int lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd, group = p.nq / p.nkv;
    const AttnLayout l = attn_layout(p, split);
    float* qs = reinterpret_cast<float*>(act);  // [group][hd]
    float* sc = qs + group * hd;                // [group][chunk]
    KV* kc = static_cast<KV*>(p.k_cache);
    KV* vc = static_cast<KV*>(p.v_cache);
    const float2* rope_row = p.rope + static_cast<size_t>(p.rope_stride) * l.pos;
    const bool has_new = l.pos >= l.t0 && l.pos < l.t1;
    // bounds of everything this item touches; on failure record it and skip the whole item
    {
        const bool bad = l.pos < 0 || l.pos >= p.capacity || l.t1 > p.capacity ||
                         4 * group * hd + 4 * group * l.chunk > kStepActBytes || l.n > l.chunk ||
                         group > kAttnMaxGroup || hd != kAttnThreads;
        if (bad) {
            if (tid == 0 && err) atomicOr(err, kErrAttnIndex);
            return;
        }
    }
    if (warp < group) {  // query head kh*group + warp: [query | gate] split, head norm, RoPE
        const float* src = p.qkv + static_cast<size_t>(kh * group + warp) * 2 * hd;
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = __ldcg(src + lane + 32 * m);
        norm_rope_head(v, p.q_norm, hd, p.eps, lane, rope_row);
#pragma unroll
        for (int m = 0; m < 8; ++m) qs[warp * hd + lane + 32 * m] = v[m];
    } else if (warp == kWarps - 1 && has_new) {  // appendKv: normed + rotated k and raw v at pos
        const float* kq = p.qkv + static_cast<size_t>(p.nq) * 2 * hd + kh * hd;
        const float* vq = kq + static_cast<size_t>(p.nkv) * hd;
        float nk[8], nv[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            nk[m] = __ldcg(kq + lane + 32 * m);
            nv[m] = __ldcg(vq + lane + 32 * m);
        }
        norm_rope_head(nk, p.k_norm, hd, p.eps, lane, rope_row);
        KV* kd = kc + (static_cast<size_t>(l.pos) * p.nkv + kh) * hd;
        KV* vd = vc + (static_cast<size_t>(l.pos) * p.nkv + kh) * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            kv_st(kd + lane + 32 * m, nk[m]);
            kv_st(vd + lane + 32 * m, nv[m]);
        }
    }
    if (ts && tid == 0) ts[3] = global_ns();
    __threadfence_block();
    named_bar(1, kThreads);

    // scores s = q . k / sqrt(hd) (custom_model.cpp:871-885), row j on warp j % 12
    const float rs = sqrtf(static_cast<float>(hd));
    for (int j = warp; j < l.n; j += kWarps) {
        const KV* kr = kc + (static_cast<size_t>(l.t0 + j) * p.nkv + kh) * hd;
        float kv[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) kv[m] = kv_ld(kr + lane + 32 * m);
        for (int g = 0; g < group; ++g) {
            float d = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; ++m) d += qs[g * hd + lane + 32 * m] * kv[m];
            d = warp_sum(d);
            if (lane == 0) sc[g * l.chunk + j] = d / rs;
        }
    }
    named_bar(1, kThreads);
    if (ts && tid == 0) ts[5] = global_ns();
    if (warp < group) {  // local max-subtracted exponentials (custom_model.cpp:890-905)
        float mx = -INFINITY;
        for (int j = lane; j < l.n; j += 32) mx = fmaxf(mx, sc[warp * l.chunk + j]);
        mx = warp_max(mx);
        float s_ = 0.0f;
        for (int j = lane; j < l.n; j += 32) {
            const float e = expf(sc[warp * l.chunk + j] - mx);
            sc[warp * l.chunk + j] = e;
            s_ += e;
        }
        s_ = warp_sum(s_);
        if (lane == 0) {
            sh->m[warp] = mx;
            sh->l[warp] = s_;
        }
    }
    named_bar(1, kThreads);
    float* pp = p.part + static_cast<size_t>(kh * kAttnSplits + split) * group * (hd + 2);
    if (tid < hd) {  // V reduction (custom_model.cpp:910-928), thread = dimension
        float o[kAttnMaxGroup];
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g) o[g] = 0.0f;
        for (int j0 = 0; j0 < l.n; j0 += 8) {  // 8 rows per round trip
            float vb[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                vb[u] = j0 + u < l.n ? kv_ld(vc + (static_cast<size_t>(l.t0 + j0 + u) * p.nkv + kh) * hd + tid) : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j0 + u < l.n) {
#pragma unroll
                    for (int g = 0; g < kAttnMaxGroup; ++g)
                        if (g < group) o[g] += sc[g * l.chunk + j0 + u] * vb[u];
                }
        }
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g)
            if (g < group) pp[g * (hd + 2) + tid] = o[g];
    }
    if (tid < group) {
        pp[tid * (hd + 2) + hd] = sh->m[tid];
        pp[tid * (hd + 2) + hd + 1] = sh->l[tid];
    }
    // Thread 0's acq_rel add publishes the block's partials (ordered before it by the block
    // barrier) and, for the last split of the kv head, acquires the other splits' partials.
    named_bar(1, kThreads);
    if (tid == 0) {
        unsigned old;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.counters + kh) : "memory");
        sh->last = old == kAttnSplits - 1 ? 1 : 0;
    }
    named_bar(1, kThreads);
    if (ts && tid == 0) ts[6] = global_ns();
    if (!sh->last) return;
    // Merge: (max, sum) of every (split, head) pair, one rescale weight per pair, then each
    // (head, dimension) output sums its partials over the splits, all of them in flight at once.
    const float* base = p.part + static_cast<size_t>(kh * kAttnSplits) * group * (hd + 2);
    if (tid < kAttnSplits * group) {
        const float* ps = base + tid * (hd + 2);  // tid = split * group + g
        sh->pm[tid] = __ldcg(ps + hd);
        sh->pl[tid] = __ldcg(ps + hd + 1);
    }
    float v32[kAttnSplits];  // this thread's first output's partials, requested with the pairs
    {
        const int e = tid < group * hd ? tid : 0, g = e / hd, d = e - g * hd;
#pragma unroll
        for (int u = 0; u < kAttnSplits; ++u) v32[u] = __ldcg(base + (u * group + g) * (hd + 2) + d);
    }
    named_bar(1, kThreads);
    if (tid < group) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < kAttnSplits; ++s2) M = fmaxf(M, sh->pm[s2 * group + tid]);
        float Ls = 0.0f;
        for (int s2 = 0; s2 < kAttnSplits; ++s2) Ls += sh->pl[s2 * group + tid] * expf(sh->pm[s2 * group + tid] - M);
        sh->M[tid] = M;
        sh->invL[tid] = Ls > 0.0f ? 1.0f / Ls : 0.0f;
    }
    named_bar(1, kThreads);
    if (tid < kAttnSplits * group) sh->pm[tid] = expf(sh->pm[tid] - sh->M[tid % group]);
    named_bar(1, kThreads);
    for (int e = tid; e < group * hd; e += kThreads) {  // output (g, d), over all consumer threads
        const int g = e / hd, d = e - g * hd;
        if (e != tid) {
#pragma unroll
            for (int u = 0; u < kAttnSplits; ++u) v32[u] = __ldcg(base + (u * group + g) * (hd + 2) + d);
        }
        float O = 0.0f;
#pragma unroll
        for (int u = 0; u < kAttnSplits; ++u) O += v32[u] * sh->pm[u * group + g];
        const float gate = __ldcg(p.qkv + static_cast<size_t>(kh * group + g) * 2 * hd + hd + d);
        p.out[(kh * group + g) * hd + d] = (O * sh->invL[g]) * dsigmoid(gate);  // output gate, :944-946
    }
    if (tid == 0) p.counters[kh] = 0u;
}

// Inputs of a GEMV phase that do not depend on the phase just before it, issued by thread 0
// right after this block arrives at the grid barrier that closes that phase: norm weights, conv
// weights and this block's conv state (which only this block writes), the gate of a gated
// prologue (written by the in_proj two phases earlier) and this block's residual rows (the
// hidden state, last written two or more phases earlier and not written by the phase in
// between). This block passed the barrier that closed those writers' phase, and this thread
// acquired it; the proxy fence orders those writes before the bulk copies. Also warms the
// descriptor of x's tensor map. Always arms cbar once.
__device__ __forceinline__ void issue_constants(const PhaseDesc& D, Ctx& c) {
    fence_proxy_async_smem();  // the areas were last read by generic loads
    fence_proxy_async_global();
    uint32_t bytes = 0;
    const void* src[3] = {nullptr, nullptr, nullptr};
    void* dst[3] = {nullptr, nullptr, nullptr};
    uint32_t len[3] = {0, 0, 0};
    int vec_n = 0, vec_map = 0, gate_n = 0;
    float* vec_dst = nullptr;
    if (D.kind == kPhaseGemv) {
        const GemvParams& p = D.g;
        prefetch_tensormap(D.tmap[0]);
        if (D.pro == kProRms) {
            vec_n = p.cols, vec_map = 1, vec_dst = c.act + p.cols;
        } else if (D.pro == kProGatedRms) {
            vec_n = p.head_dim, vec_map = 2, vec_dst = c.act + 2 * p.cols;
            gate_n = p.cols;
        }
        int r_begin, r_end, nchunks;
        block_rows(p, &r_begin, &r_end, &nchunks);
        if (D.epi == kEpiConv) {
            const EpiWindow w = epi_window(p, kEpiConv, r_begin, r_end);
            if (w.ok) {
                const int n = w.r1 - w.r0;
                src[1] = p.conv_w + static_cast<size_t>(w.r0) * 4, dst[1] = c.epi, len[1] = 16u * n;
                src[2] = p.conv_state + static_cast<size_t>(w.r0) * 3, dst[2] = c.epi + 4 * n, len[2] = 12u * n;
            }
        } else if (D.epi == kEpiResidual) {
            const EpiWindow w = epi_window(p, kEpiResidual, r_begin, r_end);
            if (w.ok) src[0] = p.out + w.r0, dst[0] = c.epi, len[0] = 4u * (w.r1 - w.r0);
        }
    }
    // DeltaNet phase: each team's state slice ([dk][kDeltaCols], 8 KB at dk = 128) into the
    // activation area (the recurrent state was last written one step earlier).
    int delta_items = 0;
    if (D.kind == kPhaseDelta && D.tmap[0]) {
        const int nslice = D.d.dv / kDeltaCols, items = D.d.nv * nslice;
        for (int t = 0; t < 3; ++t)
            if (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x) < items) ++delta_items;
    }
    for (int k = 0; k < 3; ++k) bytes += len[k];
    mbar_expect_tx(c.cbar, bytes + 4u * (vec_n + gate_n) + delta_items * 4u * kDeltaCols * D.d.dk);
    for (int t = 0; t < delta_items; ++t) {
        const int i = blockIdx.x + t * gridDim.x, nslice = D.d.dv / kDeltaCols;
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
            "[%4];" ::"r"(smem_u32(c.act + t * kDeltaCols * D.d.dk)),
            "l"(D.tmap[0]), "r"((i % nslice) * kDeltaCols), "r"((i / nslice) * D.d.dk), "r"(smem_u32(c.cbar))
            : "memory");
    }
    if (vec_n) tma_vector(vec_dst, D.tmap[vec_map], vec_n, c.cbar);
    if (gate_n) tma_vector(c.act + D.g.cols, D.tmap[1], gate_n, c.cbar);
    for (int k = 0; k < 3; ++k)
        if (len[k]) bulk_g2s(dst[k], src[k], len[k], c.cbar);
}

// x of a GEMV phase (the previous phase's output): issued right after the grid barrier that
// opens the phase, whose acquire makes the other blocks' stores visible; the proxy fence extends
// that to the tensor copies. Always arms xbar once. Called by all 32 lanes of warp 0: lane 0
// arms xbar, then lanes 0-15 issue the boxes in parallel (a 48 KB x is 12 boxes).
__device__ __forceinline__ void issue_activations(const PhaseDesc& D, Ctx& c, int lane) {
    fence_proxy_async_global();
    fence_proxy_async_smem();
    if (D.kind != kPhaseGemv) {
        if (lane == 0) mbar_expect_tx(c.xbar, 0);
        return;
    }
    const GemvParams& p = D.g;
    const uint32_t ss_bytes =
        D.pro == kProHeadScale ? 4u * static_cast<uint32_t>(p.cols / p.head_dim * p.head_ss_slices) : 0u;
    if (lane == 0) mbar_expect_tx(c.xbar, 4u * p.cols + ss_bytes);
    __syncwarp();
    if (lane < 16) tma_vector(c.act, D.tmap[0], p.cols, c.xbar, lane, 16);
    if (lane == 16 && ss_bytes) bulk_g2s(c.act + p.cols, p.head_ss, ss_bytes, c.xbar);
}

// One output row's epilogue with its inputs from the staging area when `w.ok`.
template <int EPI>
__device__ __forceinline__ void step_epilogue_row(const GemvParams& p, int r, float y, const EpiWindow& w,
                                                  const float* epi) {
    if constexpr (EPI == kEpiResidual) {
        const float res = w.ok ? epi[r - w.r0] : __ldcg(p.out + r);
        p.out[r] = res + y;  // addResidual, custom_model.cpp:294-299
    } else if constexpr (EPI == kEpiConv) {
        if (r < p.conv_channels && w.ok) {
            // causal conv + SiLU + state shift, custom_model.cpp:985-1006 (conv_k = 4)
            const int n = w.r1 - w.r0;
            const float4 cw = *reinterpret_cast<const float4*>(epi + 4 * (r - w.r0));
            const float* stc = epi + 4 * n + 3 * (r - w.r0);
            const float s0 = stc[0], s1 = stc[1], s2 = stc[2];
            float acc = 0.0f;
            acc += s0 * cw.x;
            acc += s1 * cw.y;
            acc += s2 * cw.z;
            acc += y * cw.w;
            p.out[r] = dsilu(acc);
            float* st = p.conv_state + static_cast<size_t>(r) * 3;
            st[0] = s1;
            st[1] = s2;
            st[2] = y;
        } else {
            gemv_epilogue_row<EPI>(p, r, y);
        }
    } else {
        gemv_epilogue_row<EPI>(p, r, y);
    }
}

// Thread t's 32 consecutive values of a staged vector (row t of the swizzled [n/32][32] copy).
__device__ __forceinline__ void staged_row(const float* base, int row, float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 a = *reinterpret_cast<const float4*>(base + 32 * row + 4 * (i ^ (row & 7)));
        v[4 * i] = a.x;
        v[4 * i + 1] = a.y;
        v[4 * i + 2] = a.z;
        v[4 * i + 3] = a.w;
    }
}

// 16-byte chunk `chunk` of row `row` of a staged [n/32][32] vector (128-byte swizzle).
__device__ __forceinline__ float4* staged_chunk(float* base, int row, int chunk) {
    return reinterpret_cast<float4*>(base + 32 * row + 4 * (chunk ^ (row & 7)));
}

// Gated head-RMS prologue (applyGatedHeadRms, custom_model.cpp:329-349), spread over all
// consumers: one thread per 32-column row sums its squares and the head's lanes combine them
// (inverse norms of the <= 32 heads in wsum), then every consumer thread normalises 16-byte
// chunks in place, x * inv * w * silu(z) in that order. The expf work of a head lands on twelve
// warps instead of the four that own the rows.
__device__ __forceinline__ void gated_prologue(const GemvParams& p, Ctx& c) {
    const int nrows = p.cols >> 5;
    const int tph = p.head_dim >> 5;  // rows of one head: consecutive threads of one warp
    const int tid = c.tid;
    float ss = 0.0f;
    if (tid < nrows) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 a = *staged_chunk(c.act, tid, i);
            ss += a.x * a.x;
            ss += a.y * a.y;
            ss += a.z * a.z;
            ss += a.w * a.w;
        }
    }
    for (int o = 1; o < tph; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (tid < nrows && tid % tph == 0) c.wsum[tid / tph] = 1.0f / sqrtf(ss / static_cast<float>(p.head_dim) + p.eps);
    named_bar(1, kStepConsumers);
    for (int q = tid; q < nrows * 8; q += kStepConsumers) {
        const int row = q >> 3, i = q & 7;
        const float inv = c.wsum[row / tph];
        float4 a = *staged_chunk(c.act, row, i);
        const float4 z = *staged_chunk(c.act + p.cols, row, i);
        const float4 g = *staged_chunk(c.act + 2 * p.cols, row % tph, i);
        a.x = a.x * inv * g.x * dsilu(z.x);
        a.y = a.y * inv * g.y * dsilu(z.y);
        a.z = a.z * inv * g.z * dsilu(z.z);
        a.w = a.w * inv * g.w * dsilu(z.w);
        *staged_chunk(c.act, row, i) = a;
    }
    named_bar(1, kStepConsumers);  // the normalised x is visible to every team; wsum free again
}

// gemv_load_x's arithmetic on the staged copies (same operations in the same order); a gated
// prologue has normalised x in place already (gated_prologue).
template <int PRO>
__device__ __forceinline__ void staged_prologue(const GemvParams& p, const float* act, int t, int lane, int warp,
                                                int team, int wpt, int team_bar, int team_size, float* wsum,
                                                float (&xv)[32]) {
    staged_row(act, t, xv);
    if constexpr (PRO == kProRms) {
        // rmsnormReference (ref_rmsnorm.cpp:8-17): x * (1/sqrt(mean(x^2)+eps)) * w
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) ss += xv[i] * xv[i];
        ss = warp_sum(ss);
        if (lane == 0) wsum[warp] = ss;
        named_bar(team_bar, team_size);
        float tot = 0.0f;
        for (int w = 0; w < wpt; ++w) tot += wsum[team * wpt + w];
        const float inv = 1.0f / sqrtf(tot / static_cast<float>(p.cols) + p.eps);
        float g[32];
        staged_row(act + p.cols, t, g);
#pragma unroll
        for (int i = 0; i < 32; ++i) xv[i] = xv[i] * inv * g[i];
        named_bar(team_bar, team_size);  // wsum may be reused by the next phase
    }
}

// Partial dot products of RPT rows of a ring slot for thread t (same arithmetic as
// gemv_chunk_partials). No row clamp: RPT rows always lie inside the slot, and the sums of rows
// past a short last chunk are never stored.
template <int META, int RPT>
__device__ __forceinline__ void step_partials(const uint8_t* sb, int row_stride, int meta_offset, int t,
                                              const XLimbs& L, float (&part)[RPT]) {
    const uint8_t* cp = sb + 16 * t;
    const uint8_t* mp = sb + meta_offset + (META == kMetaSym16 ? 2 : 8) * (t >> 1);
    uint4 wv[RPT];
    float sc[RPT], off[RPT];
#pragma unroll
    for (int jj = 0; jj < RPT; ++jj) {
        wv[jj] = ld_shared_v4(cp + jj * row_stride);
        if constexpr (META == kMetaSym16) {
            sc[jj] = __half2float(*reinterpret_cast<const __half*>(mp + jj * row_stride));
            off[jj] = 0.0f;
        } else {
            const float2 sbv = *reinterpret_cast<const float2*>(mp + jj * row_stride);
            sc[jj] = sbv.x;
            off[jj] = sbv.y;
        }
    }
#pragma unroll
    for (int jj = 0; jj < RPT; ++jj) {
        const uint32_t ws[4] = {wv[jj].x, wv[jj].y, wv[jj].z, wv[jj].w};
        int ae[3], ao[3];
        {
            const uint32_t lw = ws[0] & 0x0F0F0F0Fu, hw = ws[0] & 0xF0F0F0F0u;
#pragma unroll
            for (int l = 0; l < 3; ++l) {
                ae[l] = dp4a_us(lw, L.le[0][l], L.acc_init[l]);
                ao[l] = dp4a_us(hw, L.lo[0][l], 0);
            }
        }
#pragma unroll
        for (int i = 1; i < 4; ++i) {
            const uint32_t lw = ws[i] & 0x0F0F0F0Fu, hw = ws[i] & 0xF0F0F0F0u;
#pragma unroll
            for (int l = 0; l < 3; ++l) {
                ae[l] = dp4a_us(lw, L.le[i][l], ae[l]);
                ao[l] = dp4a_us(hw, L.lo[i][l], ao[l]);
            }
        }
        const float d2 = static_cast<float>(ae[2] * 16 + ao[2]);
        const float d1 = static_cast<float>(ae[1] * 16 + ao[1]);
        const float d0 = static_cast<float>(ae[0] * 16 + ao[0]);
        const float dot = d2 * 65536.0f + (d1 * 256.0f + d0);
        if constexpr (META == kMetaSym16)
            part[jj] = dot * (sc[jj] * L.down) + L.nan_or_zero;
        else
            part[jj] = dot * (sc[jj] * L.down) + off[jj] * L.xsum + L.nan_or_zero;
    }
}

// End of an argmax phase: block result, then the last block merges all blocks, samples the
// token and loads its embedding row (gemvW4A16ArgmaxNeon :309-336, loadEmbeddingRow
// custom_model.cpp:569-608).
__device__ __forceinline__ void argmax_tail(const GemvParams& p, Ctx& c, float best_v, int best_i) {
    const int tid = c.tid, lane = c.lane, warp = c.warp;
    ArgScratch* a = reinterpret_cast<ArgScratch*>(c.base + kOffArg);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        argmax_merge(best_v, best_i, ov, oi);
    }
    if (lane == 0) {
        a->v[warp] = best_v;
        a->i[warp] = best_i;
    }
    named_bar(1, kStepConsumers);
    if (tid == 0) {
        for (int w = 1; w < kStepConsumers / 32; ++w) argmax_merge(best_v, best_i, a->v[w], a->i[w]);
        p.part_val[blockIdx.x] = best_v;
        p.part_idx[blockIdx.x] = best_i;
        __threadfence();
        a->last = (atomicAdd(p.counter, 1u) == gridDim.x - 1) ? 1 : 0;
    }
    named_bar(1, kStepConsumers);
    if (a->last) {
        __threadfence();
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int b = tid; b < static_cast<int>(gridDim.x); b += kStepConsumers)
            argmax_merge(bv, bi, __ldcg(p.part_val + b), __ldcg(p.part_idx + b));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, ov, oi);
        }
        named_bar(1, kStepConsumers);
        if (lane == 0) {
            a->v[warp] = bv;
            a->i[warp] = bi;
        }
        named_bar(1, kStepConsumers);
        if (tid == 0) {
            for (int w = 1; w < kStepConsumers / 32; ++w) argmax_merge(bv, bi, a->v[w], a->i[w]);
            if (bi < 0 || bi >= p.rows) bi = 0;
            a->token = bi;
            if (p.token_out) *p.token_out = bi;
            if (p.value_out) *p.value_out = bv;
            if (p.ring) {
                const int k = *p.ring_ctr;
                p.ring[k % p.ring_cap] = bi;
                *p.ring_ctr = k + 1;
            }
            if (p.pos) {
                const int np = *p.next_pos;
                *p.pos = np;
                *p.next_pos = np + 1;
            }
            *p.counter = 0u;
        }
        named_bar(1, kStepConsumers);
        if (p.emb) {
            const uint16_t* e = p.emb + static_cast<size_t>(a->token) * p.hidden;
            for (int k = tid; k < p.hidden; k += kStepConsumers) p.hidden_out[k] = bf16_to_f32(e[k]);
        }
    }
}

// One GEMV phase. The prologue and epilogue kinds are runtime values (uniform branches): the
// kernel then holds a single copy of the chunk loop, which keeps the instruction working set
// of a step small (every phase switch would otherwise fetch a new unrolled loop).
template <int META, int RPT>
__device__ __forceinline__ void gemv_phase(const GemvParams& p, const int pro, const int epi, Ctx& c,
                                        unsigned long long* ts) {
    int r_begin, r_end, nchunks;
    block_rows(p, &r_begin, &r_end, &nchunks);
    const int R = p.rows_per_chunk;
    const int team_size = p.cols >> 5;
    const int teams = kStepConsumers / team_size;
    const int tid = c.tid, lane = c.lane, warp = c.warp;
    float best_v = -INFINITY;
    int best_i = (tid == 0) ? r_begin : 0x7fffffff;
    const EpiWindow ew = epi_window(p, epi, r_begin, r_end);
    mbar_wait_bounded(c.cbar, c.parity, p.err, c.wait_ns);
    if (ts && tid == 0) ts[7] = global_ns();
    mbar_wait_bounded(c.xbar, c.parity, p.err, c.wait_ns);
    if (ts && tid == 0) ts[10] = global_ns();
    if (pro == kProGatedRms) gated_prologue(p, c);
    if (tid < teams * team_size) {
        const int team = tid / team_size;
        const int t = tid - team * team_size;
        const int wpt = team_size >> 5;
        const int team_bar = 2 + team;
        XLimbs L;
        {
            float xv[32];
            if (pro == kProRms)
                staged_prologue<kProRms>(p, c.act, t, lane, warp, team, wpt, team_bar, team_size, c.wsum, xv);
            else
                staged_row(c.act, t, xv);  // plain, or already normalised by gated_prologue
            if (ts && tid == 0) ts[3] = global_ns() + (xv[0] != xv[0]);
            gemv_make_limbs<META>(xv, L);
        }
        if (ts && tid == 0) ts[4] = global_ns();
        int it = 0;
        unsigned long long full_wait = 0;
        // ring slot and fill parity of chunk gbase + team, advanced by `teams` chunks per step
        // (no division in the loop)
        int s = (c.gbase + team) % c.nslots;
        uint32_t par = static_cast<uint32_t>(((c.gbase + team) / c.nslots) & 1);
        for (int ci = team; ci < nchunks; ci += teams, ++it) {
            const int row0 = r_begin + ci * R;
            const int nr = min(R, r_end - row0);
            if (ts && tid == 0) {
                const unsigned long long w0 = global_ns();
                mbar_wait_bounded(&c.full[s], par, p.err, c.wait_ns);
                const unsigned long long w1 = global_ns();
                full_wait += w1 - w0;
                if (it == 0) ts[5] = w1;
            } else {
                mbar_wait_bounded(&c.full[s], par, p.err, c.wait_ns);
            }
            float part[RPT];
            step_partials<META, RPT>(c.ring + static_cast<size_t>(s) * c.slot_bytes, p.row_stride, p.meta_offset,
                                     t, L, part);
            const float v = reduce_rows<RPT>(part, lane);
            float* rbuf = c.red + (it & 1) * (kMaxRowsPerChunk * 32);
            if ((lane & (32 / RPT - 1)) == 0) {
                const int j = lane / (32 / RPT);
                if (j < nr) rbuf[j * 32 + warp] = v;
            }
            named_bar(team_bar, team_size);
            if (t == 0) mbar_arrive(&c.empty[s]);
            s += teams;
            while (s >= c.nslots) {
                s -= c.nslots;
                par ^= 1u;
            }
            const int w0 = team * wpt;
            if (epi == kEpiSwiglu) {
                if (t < (nr >> 1)) {
                    float gsum = 0.0f, u = 0.0f;
                    for (int w = 0; w < wpt; ++w) {
                        gsum += rbuf[(2 * t) * 32 + w0 + w];
                        u += rbuf[(2 * t + 1) * 32 + w0 + w];
                    }
                    p.out[(row0 >> 1) + t] = dsilu(gsum) * u;  // custom_model.cpp:1226-1230
                }
            } else {
                if (t < nr) {
                    float y = 0.0f;
                    for (int w = 0; w < wpt; ++w) y += rbuf[t * 32 + w0 + w];
                    if (epi == kEpiArgmax)
                        argmax_merge(best_v, best_i, y, row0 + t);
                    else if (epi == kEpiResidual)
                        step_epilogue_row<kEpiResidual>(p, row0 + t, y, ew, c.epi);
                    else if (epi == kEpiConv)
                        step_epilogue_row<kEpiConv>(p, row0 + t, y, ew, c.epi);
                    else
                        step_epilogue_row<kEpiStore>(p, row0 + t, y, ew, c.epi);
                }
            }
        }
        if (ts && tid == 0) ts[8] = full_wait;  // a duration, not a timestamp
    }
    if (ts && tid == 0) ts[6] = global_ns();
    c.gbase += nchunks;
    if (epi == kEpiArgmax) argmax_tail(p, c, best_v, best_i);
}

// ---- tensor-core GEMV phase (kMetaMma) -------------------------------------------------
// x as three signed 8-bit digits of a 22-bit fixed-point mantissa per 64-column group
// (x ~ m * 2^-S), laid out for the B fragments of mma.sync m16n8k32 in the activation area:
// digit row d (d = 0..2) at byte d * (K + 16) (the 16-byte pad puts the three rows on
// different banks), then per pair of groups 8 start values (int: -8 * the group's digit sum,
// the symmetric zero; columns 0-2 first group, 3-5 second, 6-7 zero) and 8 column weights
// (float: 256^d * 2^-S, NaN for a group holding a non-finite x, 0 for columns 6-7).
__device__ __forceinline__ int mma_digit_stride(int K) { return K + 16; }
__device__ __forceinline__ int* mma_cinit(uint8_t* act, int K) {
    return reinterpret_cast<int*>(act + 3 * mma_digit_stride(K));
}
__device__ __forceinline__ float* mma_wtab(uint8_t* act, int K) {
    return reinterpret_cast<float*>(act + 3 * mma_digit_stride(K)) + K / 16;
}

// Digits of thread t's E columns (E = 16 or 32; the 64 / E consecutive lanes of one 64-column
// group share the group's exponent and digit sums).
template <int E>
struct XDigits {
    uint32_t w[3][E / 4];  // digit d of columns 4k .. 4k + 3 (byte j = column 4k + j)
    int zs[3];             // digit sums of the whole group
    int S;
    bool finite;
};
template <int E>
__device__ __forceinline__ void mma_make_digits(const float (&xv)[E], XDigits<E>& X) {
    float amax = 0.0f;
    int bad = 0;  // fmaxf drops NaN operands: test every value
#pragma unroll
    for (int i = 0; i < E; ++i) {
        amax = fmaxf(amax, fabsf(xv[i]));
        bad |= !isfinite(xv[i]);
    }
#pragma unroll
    for (int o = 1; o < 64 / E; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    X.finite = !bad;
    // As gemv_make_limbs: amax = f * 2^ex, f in [0.5, 1); m = round_to_nearest_even(x * 2^S)
    // with |m| < 2^22 sits in the low bits of x * 2^S + 1.5 * 2^23, and m + 0x808080 has the
    // digits + 128 as its bytes.
    const int ex = ((__float_as_int(amax) >> 23) & 0xff) - 126;
    X.S = max(-100, min(100, 22 - ex));
    const float up = __int_as_float((X.S + 127) << 23);
    int z0 = 0, z1 = 0, z2 = 0;
#pragma unroll
    for (int k = 0; k < E / 4; ++k) {
        uint32_t u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            u[j] = static_cast<uint32_t>(__float_as_int(fmaf(xv[4 * k + j], up, 12582912.0f))) +
                   (0x808080u - 0x4B400000u);
        const uint32_t lo = __byte_perm(u[0], u[1], 0x5140), hi = __byte_perm(u[2], u[3], 0x5140);
        const uint32_t lo2 = __byte_perm(u[0], u[1], 0x0062), hi2 = __byte_perm(u[2], u[3], 0x0062);
        X.w[0][k] = __byte_perm(lo, hi, 0x5410) ^ 0x80808080u;
        X.w[1][k] = __byte_perm(lo, hi, 0x7632) ^ 0x80808080u;
        X.w[2][k] = __byte_perm(lo2, hi2, 0x5410) ^ 0x80808080u;
        z0 = __dp4a(static_cast<int>(X.w[0][k]), 0x01010101, z0);
        z1 = __dp4a(static_cast<int>(X.w[1][k]), 0x01010101, z1);
        z2 = __dp4a(static_cast<int>(X.w[2][k]), 0x01010101, z2);
    }
#pragma unroll
    for (int o = 1; o < 64 / E; o <<= 1) {
        z0 += __shfl_xor_sync(0xffffffffu, z0, o);
        z1 += __shfl_xor_sync(0xffffffffu, z1, o);
        z2 += __shfl_xor_sync(0xffffffffu, z2, o);
    }
    X.zs[0] = z0;
    X.zs[1] = z1;
    X.zs[2] = z2;
}
template <int E>
__device__ __forceinline__ void mma_store_digits(const XDigits<E>& X, int t, int K, uint8_t* act) {
#pragma unroll
    for (int d = 0; d < 3; ++d) {
        uint4* dst = reinterpret_cast<uint4*>(act + d * mma_digit_stride(K) + E * t);
#pragma unroll
        for (int k = 0; k < E / 16; ++k)
            dst[k] = make_uint4(X.w[d][4 * k], X.w[d][4 * k + 1], X.w[d][4 * k + 2], X.w[d][4 * k + 3]);
    }
    constexpr int kTpg = 64 / E;  // threads per group
    if (t % kTpg == 0) {
        const int g = t / kTpg, base = 8 * (g >> 1), n0 = (g & 1) * 3;
        int* ci = mma_cinit(act, K);
        float* wt = mma_wtab(act, K);
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            ci[base + n0 + d] = -8 * X.zs[d];
            wt[base + n0 + d] = X.finite ? __int_as_float((127 - X.S + 8 * d) << 23) : __int_as_float(0x7fc00000);
        }
        if (g & 1) {
            ci[base + 6] = ci[base + 7] = 0;
            wt[base + 6] = wt[base + 7] = 0.0f;
        }
    }
}

// Prologue of a tensor-core phase over K / E threads, thread t owning columns [E t, E t + E) of
// the staged x: RMSNorm (rmsnormReference, ref_rmsnorm.cpp:8-17: x * (1 / sqrt(mean(x^2) +
// eps)) * w) when asked (a gated prologue has already normalised x in place), then the digit
// table, written over the staged x once every thread has read its columns.
template <int E>
__device__ __forceinline__ void mma_prologue(const GemvParams& p, const int pro, Ctx& c, unsigned long long* ts) {
    const int K = p.cols, nth = K / E;
    const int tid = c.tid, lane = c.lane, warp = c.warp;
    XDigits<E> X;
    if (tid < nth) {
        const int row = (E * tid) >> 5, ch0 = ((E * tid) & 31) >> 2;
        float xv[E];
#pragma unroll
        for (int i = 0; i < E / 4; ++i) {
            const float4 a = *staged_chunk(c.act, row, ch0 + i);
            xv[4 * i] = a.x;
            xv[4 * i + 1] = a.y;
            xv[4 * i + 2] = a.z;
            xv[4 * i + 3] = a.w;
        }
        if (pro == kProRms) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < E; ++i) ss += xv[i] * xv[i];
            ss = warp_sum(ss);
            if (lane == 0) c.wsum[warp] = ss;
            named_bar(2, nth);
            float tot = 0.0f;
            for (int w = 0; w < (nth >> 5); ++w) tot += c.wsum[w];
            const float inv = 1.0f / sqrtf(tot / static_cast<float>(K) + p.eps);
#pragma unroll
            for (int i = 0; i < E / 4; ++i) {
                const float4 g = *staged_chunk(c.act + K, row, ch0 + i);
                xv[4 * i] = xv[4 * i] * inv * g.x;
                xv[4 * i + 1] = xv[4 * i + 1] * inv * g.y;
                xv[4 * i + 2] = xv[4 * i + 2] * inv * g.z;
                xv[4 * i + 3] = xv[4 * i + 3] * inv * g.w;
            }
        }
        if (pro == kProHeadScale) {
            // the gated head norm's 1 / sqrt(mean(o^2) + eps) of this thread's head (applyGatedHeadRms,
            // custom_model.cpp:329-349; x holds o * w * silu(z) already)
            const int h = (E * tid) / p.head_dim, ns = p.head_ss_slices;
            const float* ss = c.act + K + h * ns;
            float tot = 0.0f;
            for (int j = 0; j < ns; ++j) tot += ss[j];
            const float inv = 1.0f / sqrtf(tot / static_cast<float>(p.head_dim) + p.eps);
#pragma unroll
            for (int i = 0; i < E; ++i) xv[i] *= inv;
        }
        if (ts && tid == 0) ts[3] = global_ns() + (xv[0] != xv[0]);
        mma_make_digits<E>(xv, X);
    }
    named_bar(1, kStepConsumers);  // every staged x read (and wsum): the digit table may overwrite it
    if (tid < nth) mma_store_digits<E>(X, tid, K, reinterpret_cast<uint8_t*>(c.act));
    named_bar(1, kStepConsumers);
}

// One GEMV phase on the tensor cores. Three teams of four warps take this block's 16-row tiles
// in turn; a team streams a tile's chunks (mma_ppc pairs of groups each) and every warp takes a
// quarter of each chunk's pairs: per pair four mma.sync (one per 32-column slab) into one
// accumulator whose N columns carry the digits of both groups, then the group scales.
__device__ __forceinline__ void gemv_phase_mma(const GemvParams& p, const int pro, const int epi, Ctx& c,
                                               unsigned long long* ts) {
    int r_begin, r_end, nchunks;
    block_rows(p, &r_begin, &r_end, &nchunks);
    const int K = p.cols;
    const int tid = c.tid, lane = c.lane, warp = c.warp;
    uint8_t* act = reinterpret_cast<uint8_t*>(c.act);
    float best_v = -INFINITY;
    int best_i = (tid == 0) ? r_begin : 0x7fffffff;
    const EpiWindow ew = epi_window(p, epi, r_begin, r_end);
    mbar_wait_bounded(c.cbar, c.parity, p.err, c.wait_ns);
    if (ts && tid == 0) ts[7] = global_ns();
    mbar_wait_bounded(c.xbar, c.parity, p.err, c.wait_ns);
    if (ts && tid == 0) ts[10] = global_ns();
    if (pro == kProGatedRms) gated_prologue(p, c);
    // 16 columns per thread while K / 16 threads fit the consumers (K <= 6144), else 32
    if (K / 16 <= kStepConsumers)
        mma_prologue<16>(p, pro, c, ts);
    else
        mma_prologue<32>(p, pro, c, ts);
    if (ts && tid == 0) ts[4] = global_ns();

    const int tau = warp / kMmaStepWarpsPerTeam, wt = warp % kMmaStepWarpsPerTeam;
    const int q = lane & 3, r = lane >> 2;
    // B fragment of this lane: column n = r; slabs 0-1 (first group) use digit n for n < 3,
    // slabs 2-3 (second group) digit n - 3 for 3 <= n < 6; other lanes load a valid address
    // and mask the value to zero.
    const uint32_t mask_a = r < 3 ? 0xffffffffu : 0u, mask_b = (r >= 3 && r < 6) ? 0xffffffffu : 0u;
    const uint8_t* dig_a = act + (r < 3 ? r : 0) * mma_digit_stride(K) + 4 * q;
    const uint8_t* dig_b = act + ((r >= 3 && r < 6) ? r - 3 : 0) * mma_digit_stride(K) + 4 * q;
    const int* cinit = mma_cinit(act, K);
    const float* wtab = mma_wtab(act, K);
    const int ppc = p.mma_ppc, cpt = p.mma_pairs / ppc, pw = ppc / kMmaStepWarpsPerTeam;
    const int t_begin = r_begin >> 4, t_end = (r_end + 15) >> 4;
    unsigned long long full_wait = 0;
    int it = 0;
    for (int tile = t_begin + tau; tile < t_end; tile += kMmaStepTeams, ++it) {
        float acc0 = 0.0f, acc1 = 0.0f;  // rows r and r + 8 of the tile, this lane's columns
        for (int cc = 0; cc < cpt; ++cc) {
            const int gi = c.gbase + (tile - t_begin) * cpt + cc;
            const int s = gi % c.nslots;
            const uint32_t par = static_cast<uint32_t>((gi / c.nslots) & 1);
            if (ts && tid == 0) {
                const unsigned long long w0 = global_ns();
                mbar_wait_bounded(&c.full[s], par, p.err, c.wait_ns);
                const unsigned long long w1 = global_ns();
                full_wait += w1 - w0;
                if (it == 0 && cc == 0) ts[5] = w1;
            } else {
                mbar_wait_bounded(&c.full[s], par, p.err, c.wait_ns);
            }
            const uint8_t* base = c.ring + static_cast<size_t>(s) * c.slot_bytes;
            // two pairs per iteration (pw is even): two independent accumulator chains
            for (int k = 0; k < pw; k += 2) {
                const int pl = wt * pw + k, pg = cc * ppc + pl;
                const uint8_t* pb = base + pl * kMmaUnitBytes;
                const int2 ci0 = *reinterpret_cast<const int2*>(cinit + 8 * pg + 2 * q);
                const int2 ci1 = *reinterpret_cast<const int2*>(cinit + 8 * (pg + 1) + 2 * q);
                int d0[4] = {ci0.x, ci0.y, ci0.x, ci0.y};
                int d1[4] = {ci1.x, ci1.y, ci1.x, ci1.y};
#pragma unroll
                for (int sl = 0; sl < 4; ++sl) {
                    const uint2 a0 = *reinterpret_cast<const uint2*>(pb + sl * 256 + 8 * lane);
                    const uint2 a1 = *reinterpret_cast<const uint2*>(pb + kMmaUnitBytes + sl * 256 + 8 * lane);
                    const uint8_t* db = (sl < 2 ? dig_a : dig_b) + 128 * pg + 32 * sl;
                    const uint32_t m = sl < 2 ? mask_a : mask_b;
                    const uint32_t b00 = *reinterpret_cast<const uint32_t*>(db) & m;
                    const uint32_t b01 = *reinterpret_cast<const uint32_t*>(db + 16) & m;
                    const uint32_t b10 = *reinterpret_cast<const uint32_t*>(db + 128) & m;
                    const uint32_t b11 = *reinterpret_cast<const uint32_t*>(db + 144) & m;
                    mma_u8s8(d0, a0.x & 0x0F0F0F0Fu, (a0.x >> 4) & 0x0F0F0F0Fu, a0.y & 0x0F0F0F0Fu,
                             (a0.y >> 4) & 0x0F0F0F0Fu, b00, b01);
                    mma_u8s8(d1, a1.x & 0x0F0F0F0Fu, (a1.x >> 4) & 0x0F0F0F0Fu, a1.y & 0x0F0F0F0Fu,
                             (a1.y >> 4) & 0x0F0F0F0Fu, b10, b11);
                }
                // fp16 scales [row r: g0, g1 | row r + 8: g0, g1]; column 2q belongs to the second
                // group iff q >= 2, column 2q + 1 iff q >= 1.
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int* d = e ? d1 : d0;
                    const uint2 sh = *reinterpret_cast<const uint2*>(pb + e * kMmaUnitBytes + 1024 + 8 * r);
                    const float2 s_r = __half22float2(*reinterpret_cast<const __half2*>(&sh.x));
                    const float2 s_r8 = __half22float2(*reinterpret_cast<const __half2*>(&sh.y));
                    const float2 w = *reinterpret_cast<const float2*>(wtab + 8 * (pg + e) + 2 * q);
                    const float sa0 = q >= 2 ? s_r.y : s_r.x, sb0 = q >= 1 ? s_r.y : s_r.x;
                    const float sa1 = q >= 2 ? s_r8.y : s_r8.x, sb1 = q >= 1 ? s_r8.y : s_r8.x;
                    acc0 += static_cast<float>(d[0]) * (w.x * sa0) + static_cast<float>(d[1]) * (w.y * sb0);
                    acc1 += static_cast<float>(d[2]) * (w.x * sa1) + static_cast<float>(d[3]) * (w.y * sb1);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&c.empty[s]);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        // row sums [team][tile parity][warp][16]: the buffer of tile i is rewritten at tile i + 2,
        // after the team barrier of tile i + 1
        float* rb = c.red + ((tau * 2 + (it & 1)) * kMmaStepWarpsPerTeam) * 16;
        if (q == 0) {
            rb[wt * 16 + r] = acc0;
            rb[wt * 16 + r + 8] = acc1;
        }
        named_bar(2 + tau, 32 * kMmaStepWarpsPerTeam);
        const int tt = tid - tau * 32 * kMmaStepWarpsPerTeam;
        const int row0 = 16 * tile;
        if (epi == kEpiSwiglu) {
            if (tt < 8 && row0 + 2 * tt + 1 < p.rows) {
                const int j = 2 * tt;
                const float gsum = ((rb[j] + rb[16 + j]) + rb[32 + j]) + rb[48 + j];
                const float u = ((rb[j + 1] + rb[17 + j]) + rb[33 + j]) + rb[49 + j];
                p.out[(row0 >> 1) + tt] = dsilu(gsum) * u;  // custom_model.cpp:1226-1230
            }
        } else if (tt < 16 && row0 + tt < p.rows) {
            const float y = ((rb[tt] + rb[16 + tt]) + rb[32 + tt]) + rb[48 + tt];
            const int row = row0 + tt;
            if (epi == kEpiArgmax)
                argmax_merge(best_v, best_i, y, row);
            else if (epi == kEpiResidual)
                step_epilogue_row<kEpiResidual>(p, row, y, ew, c.epi);
            else if (epi == kEpiConv)
                step_epilogue_row<kEpiConv>(p, row, y, ew, c.epi);
            else
                step_epilogue_row<kEpiStore>(p, row, y, ew, c.epi);
        }
    }
    if (ts && tid == 0) {
        ts[8] = full_wait;
        ts[6] = global_ns();
    }
    c.gbase += nchunks;
    if (epi == kEpiArgmax) argmax_tail(p, c, best_v, best_i);
}

template <int META>
__device__ __forceinline__ void gemv_dispatch(const PhaseDesc& D, Ctx& c, unsigned long long* ts) {
    const int pro = D.pro, epi = D.epi;
    const bool known = (pro == kProRms && (epi == kEpiConv || epi == kEpiSwiglu || epi == kEpiStore ||
                                           epi == kEpiArgmax)) ||
                       (pro == kProGatedRms && epi == kEpiResidual) || (pro == kProPlain && epi == kEpiResidual);
    if constexpr (META == kMetaMma) {
        const bool head_scale = pro == kProHeadScale && epi == kEpiResidual && D.g.head_dim >= 32 &&
                                D.g.head_dim % 32 == 0 && D.g.head_ss_slices > 0 &&
                                (D.g.cols / D.g.head_dim) * D.g.head_ss_slices <= 1024;
        if ((known || head_scale) && D.g.mma_pairs > 0 && D.g.mma_ppc > 0 && D.g.mma_ppc % 8 == 0 &&
            D.g.mma_pairs % D.g.mma_ppc == 0 && D.g.mma_ppc * kMmaUnitBytes <= c.slot_bytes &&
            D.g.cols >> 5 <= kStepConsumers)
            gemv_phase_mma(D.g, pro, epi, c, ts);
        else if (c.tid == 0)
            atomicOr(D.g.err, kErrBadShape);
        return;
    }
    // Chunks of 8 rows (K = 4096) or 4 rows (K = 12288): the partials loop matches the chunk.
    if (known && D.g.rows_per_chunk == 8)
        gemv_phase<META, 8>(D.g, pro, epi, c, ts);
    else if (known && D.g.rows_per_chunk == 4)
        gemv_phase<META, 4>(D.g, pro, epi, c, ts);
    else if (c.tid == 0)
        atomicOr(D.g.err, kErrBadShape);
}

template <int META, typename KV>
// 13 warps: registers are allocated for 16 warps, so 128 per thread is the most one block gets.
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Ctx c;
    c.base = smem;
    c.full = reinterpret_cast<uint64_t*>(smem + kOffFull);
    c.empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
    c.xbar = reinterpret_cast<uint64_t*>(smem + kOffXBar);
    c.cbar = reinterpret_cast<uint64_t*>(smem + kOffCBar);
    uint64_t* dbar = reinterpret_cast<uint64_t*>(smem + kOffDBar);  // [2]
    c.wsum = reinterpret_cast<float*>(smem + kOffWsum);
    c.red = reinterpret_cast<float*>(smem + kOffRed);
    c.act = reinterpret_cast<float*>(smem + kOffAct);
    c.epi = reinterpret_cast<float*>(smem + kOffEpi);
    c.ring = smem + kOffRing;
    c.nslots = P.nslots;
    c.slot_bytes = P.slot_bytes;
    c.tid = threadIdx.x;
    c.lane = c.tid & 31;
    c.warp = c.tid >> 5;
    c.gbase = 0;
    c.parity = 0;
    c.wait_ns = P.wait_ns ? P.wait_ns : kWaitLimitNs;
    if (c.tid == 0) {
        for (int s = 0; s < c.nslots; ++s) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], META == kMetaMma ? kMmaStepWarpsPerTeam : 1);
        }
        mbar_init(c.xbar, 1);
        mbar_init(c.cbar, 1);
        mbar_init(&dbar[0], 1);
        mbar_init(&dbar[1], 1);
        fence_mbar_init();
        if (smem_u32(c.act) & 1023u) atomicOr(P.err, kErrBadShape);  // swizzled copies need 1024-byte alignment
    }
    __syncthreads();

    if (c.warp == kStepConsumers / 32) {
        // Producer: stream this block's rows of every GEMV phase, in phase order.
        if (c.lane == 0) {
            const int G = static_cast<int>(gridDim.x);
            const uint64_t pol = l2_evict_first_policy();
            int g = 0;  // chunks issued into the ring
            bool stop = false;
            for (int ph = 0; ph < P.nphases && !stop; ++ph) {
                const PhaseDesc& D = P.phases[ph];
                if (D.kind != kPhaseGemv) continue;
                int r_begin, r_end, nchunks;
                block_rows(D.g, &r_begin, &r_end, &nchunks);
                if (P.l2_prefetch) {
                    // Warm L2 with the phase's constant inputs well before the consumers stage them.
                    const GemvParams& g = D.g;
                    if (D.pro == kProRms && blockIdx.x == ph % G) prefetch_l2(g.norm_w, 4u * g.cols);
                    if (D.pro == kProGatedRms && blockIdx.x == ph % G) prefetch_l2(g.norm_w, 4u * g.head_dim);
                    if (D.epi == kEpiConv) {
                        const EpiWindow w = epi_window(g, kEpiConv, r_begin, r_end);
                        if (w.ok) {
                            prefetch_l2(g.conv_w + static_cast<size_t>(w.r0) * 4, 16u * (w.r1 - w.r0));
                            prefetch_l2(g.conv_state + static_cast<size_t>(w.r0) * 3, 12u * (w.r1 - w.r0));
                        }
                    }
                }
                // L2 prefetch A chunks ahead of the ring within the phase: the ring alone holds
                // too few bytes in flight for the loaded HBM latency.
                const int A = P.l2_ahead;
                const uint8_t* wbase;
                size_t cstride, wend;
                block_span(D.g, r_begin, r_end, &wbase, &cstride, &wend);
                for (int ci = 0; ci < min(A, nchunks); ++ci)
                    prefetch_l2(wbase + ci * cstride, static_cast<uint32_t>(min(cstride, wend - ci * cstride)));
                for (int ci = 0; ci < nchunks; ++ci) {
                    const int s = g % c.nslots;
                    if (ci + A < nchunks)
                        prefetch_l2(wbase + (ci + A) * cstride,
                                    static_cast<uint32_t>(min(cstride, wend - (ci + A) * cstride)));
                    if (g >= c.nslots) {
                        const unsigned long long w0 = P.trace && blockIdx.x == 0 ? global_ns() : 0;
                        if (!mbar_wait_bounded(&c.empty[s], static_cast<uint32_t>(((g / c.nslots) - 1) & 1), P.err,
                                               c.wait_ns)) {
                            stop = true;
                            break;
                        }
                        if (P.trace && blockIdx.x == 0) P.trace[kStepTraceSlots * ph + 9] += global_ns() - w0;
                    }
                    // Keep at most `inflight` copies outstanding: more only lengthens the
                    // memory queues that the consumers' activation loads wait in. Chunk
                    // g - inflight is the newest copy in its slot (inflight <= nslots), so
                    // the parity test below is unambiguous.
                    const int old = g - P.inflight;
                    if (old >= 0 && !mbar_wait_bounded(&c.full[old % c.nslots],
                                                       static_cast<uint32_t>((old / c.nslots) & 1), P.err, c.wait_ns)) {
                        stop = true;
                        break;
                    }
                    const size_t off = static_cast<size_t>(ci) * cstride;
                    const uint32_t bytes = static_cast<uint32_t>(min(cstride, wend - off));
                    mbar_expect_tx(&c.full[s], bytes);
                    if (D.g.evict_first)
                        bulk_g2s_hint(c.ring + static_cast<size_t>(s) * c.slot_bytes, wbase + off, bytes, &c.full[s],
                                      pol);
                    else
                        bulk_g2s(c.ring + static_cast<size_t>(s) * c.slot_bytes, wbase + off, bytes, &c.full[s]);
                    ++g;
                }
            }
            // Every issued copy has landed before this block can exit.
            for (int k = max(0, g - c.nslots); k < g; ++k)
                mbar_wait_drain(&c.full[k % c.nslots], static_cast<uint32_t>((k / c.nslots) & 1));
        }
        return;
    }

    AttnScratch* ash = reinterpret_cast<AttnScratch*>(smem + kOffAttn);
    DeltaScratch* dsh = reinterpret_cast<DeltaScratch*>(smem + kOffDelta);
    float* attn_dyn = c.act;
    PhaseDesc* desc = reinterpret_cast<PhaseDesc*>(smem + kOffDesc);  // [2], phase ph in desc[ph & 1]
    const unsigned G = gridDim.x;
    // Descriptor of phase ph into desc[ph & 1]; dbar[ph & 1] completes once per copy, so the
    // copy of phase ph is its (ph >> 1)-th completion.
    auto request_desc = [&](int ph) {
        mbar_expect_tx(&dbar[ph & 1], static_cast<uint32_t>(sizeof(PhaseDesc)));
        bulk_g2s(desc + (ph & 1), P.phases + ph, static_cast<uint32_t>(sizeof(PhaseDesc)), &dbar[ph & 1]);
    };
    auto wait_desc = [&](int ph) {
        mbar_wait_bounded(&dbar[ph & 1], static_cast<uint32_t>((ph >> 1) & 1), P.err, c.wait_ns);
    };
    if (c.tid == 0) {
        request_desc(0);
        if (P.nphases > 1) request_desc(1);
        wait_desc(0);
        issue_constants(desc[0], c);
    }
    if (c.warp == 0) {
        __syncwarp();
        wait_desc(0);
        issue_activations(desc[0], c, c.lane);  // written before this launch
    }
    for (int ph = 0; ph < P.nphases; ++ph) {
        c.parity = static_cast<uint32_t>(ph & 1);
        if (ph > 0 && c.warp == 0) {  // every phase consumes the previous phase's output
            if (c.lane == 0) {
                const unsigned target = static_cast<unsigned>(ph) * G + (ph == 1 ? P.barrier_extra : 0u);
                if (ld_acquire(P.grid_bar) < target) {
                    const uint64_t t0 = global_ns();
                    for (uint32_t n = 1; ld_acquire(P.grid_bar) < target; ++n)
                        if (!wait_budget_left(t0, n, P.err, c.wait_ns)) break;
                }
                if (P.trace && blockIdx.x == 0) P.trace[kStepTraceSlots * ph + 11] = global_ns();
            }
            __syncwarp();
            issue_activations(desc[ph & 1], c, c.lane);  // descriptor waited for at the end of phase ph - 1
            if (P.trace && blockIdx.x == 0 && c.lane == 0) P.trace[kStepTraceSlots * ph + 12] = global_ns();
        }
        named_bar(1, kStepConsumers);
        wait_desc(ph);
        const PhaseDesc& D = desc[ph & 1];
        if (P.trace && blockIdx.x == 0 && c.tid == 0) P.trace[kStepTraceSlots * ph] = global_ns();
        if (D.kind == kPhaseGemv) {
            gemv_dispatch<META>(D, c, (P.trace && blockIdx.x == 0) ? P.trace + kStepTraceSlots * ph : nullptr);
        } else if (D.kind == kPhaseDelta) {
            const int nslice = D.d.dv / kDeltaCols;
            const int items = D.d.nv * nslice;
            const int dteam = c.tid >> 7;  // 3 teams of 128 threads
            const bool staged = D.tmap[0] != nullptr;
            if (staged) mbar_wait_bounded(c.cbar, c.parity, P.err, c.wait_ns);  // state slices landed
            for (int i = blockIdx.x + dteam * G, r = 0; i < items; i += 3 * G, ++r)
                delta_item(D.d, i / nslice, i % nslice, c.tid & 127, 2 + dteam, dsh + dteam,
                           staged && r == 0 ? c.act + dteam * kDeltaCols * D.d.dk : nullptr);
        } else if (D.kind == kPhaseAttn) {
            const int items = D.a.nkv * kAttnSplits;
            // one item per block (the host launches the step kernel only when nkv * kAttnSplits
            // items fit the grid), its rows staged before the barrier
            if (static_cast<int>(blockIdx.x) < items)
                attention_item_step<KV>(D.a, blockIdx.x / kAttnSplits, blockIdx.x % kAttnSplits, c.tid,
                                        reinterpret_cast<uint8_t*>(attn_dyn), ash, P.err,
                                        (P.trace && blockIdx.x == 0) ? P.trace + kStepTraceSlots * ph : nullptr);
            else if (items > static_cast<int>(G) && c.tid == 0)
                atomicOr(P.err, kErrBadShape);
        } else if (D.kind == kPhaseEmbed) {
            // loadEmbeddingRow for prompt[next_pos] (custom_model.cpp:569-608, ids folded :573-575)
            if (blockIdx.x == 0) {
                int* tok = reinterpret_cast<int*>(smem + kOffArg);
                if (c.tid == 0) {
                    const int np = __ldcg(P.next_pos);
                    long long t = P.prompt[np];
                    if (t < 0 || t >= P.vocab) t = (t < 0 ? -t : t) % (P.vocab > 1 ? P.vocab : 1);
                    *tok = static_cast<int>(t);
                    *P.pos = np;
                    *P.next_pos = np + 1;
                }
                named_bar(1, kStepConsumers);
                const uint16_t* e = P.emb + static_cast<size_t>(*tok) * P.hidden_size;
                for (int k = c.tid; k < P.hidden_size; k += kStepConsumers) P.hidden[k] = bf16_to_f32(e[k]);
            }
        }
        named_bar(1, kStepConsumers);
        if (c.tid == 0) {
            if (P.trace && blockIdx.x == 0) P.trace[kStepTraceSlots * ph + 1] = global_ns();
            if (P.block_done) P.block_done[static_cast<size_t>(ph) * G + blockIdx.x] = global_ns();
            // Arrive first (the named barrier above ordered the block's work before this
            // thread's release; only the last phase, and a traced step, need the counter value
            // back), then stage the next phase's constants and descriptor while others finish.
            if (ph == P.nphases - 1 || P.trace) {
                unsigned old;
                asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(P.grid_bar) : "memory");
                if (P.trace && old == static_cast<unsigned>(ph + 1) * G - 1)
                    P.trace[kStepTraceSlots * ph + 2] = global_ns();
                if (ph == P.nphases - 1 && old == static_cast<unsigned>(P.nphases) * G - 1)
                    atomicExch(P.grid_bar, 0u);  // everybody has arrived; nobody waits any more
            } else {
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.grid_bar) : "memory");
            }
            if (ph + 1 < P.nphases) {
                wait_desc(ph + 1);
                issue_constants(desc[(ph + 1) & 1], c);
                if (ph + 2 < P.nphases) {
                    fence_proxy_async_smem();
                    request_desc(ph + 2);
                }
            }
        }
    }
    // Copies this block issued have landed before it exits (bounded waits).
    if (c.tid == 0 && P.nphases > 0) {
        const int last = P.nphases - 1;
        mbar_wait_drain(c.xbar, static_cast<uint32_t>(last & 1));
        mbar_wait_drain(c.cbar, static_cast<uint32_t>(last & 1));
    }
}

template <int META, typename KV>
cudaError_t launch_one(const StepParams& p, int num_sms, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = step_smem_bytes(p.nslots, p.slot_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_step_kernel<META, KV>, p);
}

template <int META, typename KV>
cudaError_t set_attr() {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return cudaFuncSetAttribute(decode_step_kernel<META, KV>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
}

}  // namespace

size_t step_smem_bytes(int nslots, int slot_bytes) {
    return static_cast<size_t>(kOffRing) + static_cast<size_t>(nslots) * slot_bytes;
}

int step_max_slots(int slot_bytes) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int avail = optin - kOffRing - 1024;
    return std::max(2, std::min(kStepMaxSlots, avail / slot_bytes));
}

cudaError_t step_init_device() {
    cudaError_t e;
    if ((e = set_attr<kMetaSym16, float>()) != cudaSuccess) return e;
    if ((e = set_attr<kMetaSym16, __half>()) != cudaSuccess) return e;
    if ((e = set_attr<kMetaAff32, float>()) != cudaSuccess) return e;
    if ((e = set_attr<kMetaAff32, __half>()) != cudaSuccess) return e;
    if ((e = set_attr<kMetaMma, float>()) != cudaSuccess) return e;
    return set_attr<kMetaMma, __half>();
}

bool encode_state_tmap(void* out, const float* ptr, int rows, int cols, int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    if (!encode || rows <= 0 || cols % kDeltaCols != 0 || box_rows <= 0 || box_rows > 256 ||
        (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0)
        return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t boxdim[2] = {kDeltaCols, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return encode(static_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims,
                  strides, boxdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int step_kernel_binary_version() {
    cudaFuncAttributes a = {};
    if (cudaFuncGetAttributes(&a, decode_step_kernel<kMetaMma, float>) != cudaSuccess) return 0;
    return a.binaryVersion;
}

bool encode_vector_tmap(void* out, const float* ptr, int n) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    const int rows = n / 32;
    const int box = std::min(32, rows);
    if (!encode || n <= 0 || n % 32 != 0 || rows % box != 0 || (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0)
        return false;
    const cuuint64_t dims[2] = {32, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t boxdim[2] = {32, static_cast<cuuint32_t>(box)};
    const cuuint32_t estr[2] = {1, 1};
    return encode(static_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims,
                  strides, boxdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_decode_step(const StepParams& p, int meta_kind, bool kv_fp16, int num_sms, cudaStream_t s) {
    if (meta_kind == kMetaSym16)
        return kv_fp16 ? launch_one<kMetaSym16, __half>(p, num_sms, s) : launch_one<kMetaSym16, float>(p, num_sms, s);
    if (meta_kind == kMetaMma)
        return kv_fp16 ? launch_one<kMetaMma, __half>(p, num_sms, s) : launch_one<kMetaMma, float>(p, num_sms, s);
    return kv_fp16 ? launch_one<kMetaAff32, __half>(p, num_sms, s) : launch_one<kMetaAff32, float>(p, num_sms, s);
}

}  // namespace xqb
