// W4A16 group-64 dequantising GEMV for sm_100a, with fused prologues / epilogues.
//
// Math (reference: computeRowImpl, xq_gemv_w4a16_neon.cpp:234-255):
//   y[r] = sum_g s[r,g] * (sum_{c in g} code[r,c] * x[c]) + b[r,g] * (sum_{c in g} x[c])
// with b = -zero*scale for XQ4 v1 and b = zero for XQ4 v2; for the symmetric layout
// (zero = 8) the kernel folds the zero into the integer sum instead.
//
// Device row layout (one row, 16-byte multiple): [K/2 bytes of nibbles, reference order:
// even column in the low nibble][group metadata: fp16 scale per group (kMetaSym16) or a
// float2 {scale, offset} per group (kMetaAff32)].
//
// Work split: a "team" of K/32 threads covers one row; thread t owns columns
// [32t, 32t+32) = nibble bytes [16t, 16t+16) and half of group t/2. x never changes while
// rows stream past, so each thread keeps its 32 x values in registers as three signed
// 8-bit limbs of a 22-bit fixed-point mantissa (scale 2^S per thread chunk); the code * x
// products then run as exact integer dp4a sums, converted to fp32 once per row. A producer
// warp streams row chunks into a `stages`-deep shared-memory ring with 1-D bulk async copies
// (cp.async.bulk + full/empty mbarriers); it never waits on the previous kernel
// (griddepcontrol.wait is only in the consumers), so with programmatic dependent launch the
// weight streaming of a kernel overlaps the tail of the one before it.
#pragma once

#include "common.cuh"

namespace xqb {

// kMetaMma: the symmetric layout's 16-row tensor-core tiles (mma_gemv.hpp), step kernel only.
enum MetaKind : int { kMetaSym16 = 0, kMetaAff32 = 1, kMetaMma = 2 };
// kProHeadScale (tensor-core step kernel only): x already holds o * w * silu(z) of the gated
// head norm (written by the DeltaNet phase); each head's values are multiplied by
// 1 / sqrt(sum(o^2) / head_dim + eps) from head_ss, the per-slice sums of o^2.
enum Prologue : int { kProPlain = 0, kProRms = 1, kProGatedRms = 2, kProHeadScale = 3 };
enum Epilogue : int { kEpiStore = 0, kEpiResidual = 1, kEpiSwiglu = 2, kEpiConv = 3, kEpiArgmax = 4 };

constexpr int kMaxStages = 16;
constexpr int kMaxRowsPerChunk = 16;
constexpr int kMaxRowsPerTeam = 8;
constexpr int kMaxBlock = 544;           // K = 16384: one 512-thread team + the producer warp
constexpr int kTargetBlock = 256;       // consumer threads per block (plus one producer warp)
constexpr int kStageTargetBytes = 32 * 1024;
constexpr int kRingBudgetBytes = 96 * 1024;
constexpr int kGemvHeaderBytes = 4608;  // full/empty mbarriers, warp sums, double-buffered row sums

struct GemvParams {
    const uint8_t* w;  // device rows
    int rows, cols, row_stride, meta_offset;
    int rows_per_chunk;  // R, even
    int stages;          // depth of the shared-memory ring, <= kMaxStages
    int unit;            // CTA row ranges are multiples of this (2 for gate/up pairs)
    int evict_first;     // stream the rows with the L2 evict-first policy
    // Tensor-core tiles (w points at them when mma_pairs > 0): 128-column pairs per 16-row tile,
    // and pairs per streamed chunk (a divisor of mma_pairs, a multiple of 8).
    int mma_pairs, mma_ppc;
    // prologue
    const float* x;
    const float* norm_w;  // kProRms: [cols]; kProGatedRms: [head_dim]
    const float* gate_z;  // kProGatedRms: [cols]
    float eps;
    int head_dim;  // kProGatedRms, kProHeadScale
    const float* head_ss;  // kProHeadScale: [cols / head_dim][head_ss_slices]
    int head_ss_slices;
    // epilogue
    float* out;
    float* out2;           // kEpiConv: rows >= conv_channels go here
    const float* conv_w;   // kEpiConv: [conv_channels][conv_k]
    float* conv_state;     // kEpiConv: [conv_channels][conv_k - 1]
    int conv_channels, conv_k;
    // kEpiArgmax (block partials, completion counter, outputs)
    float* part_val;
    int* part_idx;
    unsigned* counter;
    int* token_out;        // may be null
    float* value_out;      // may be null
    // optional follow-up work of the last block (decode step head)
    const uint16_t* emb;   // bf16 [vocab][hidden] -> hidden_out = emb[token]
    float* hidden_out;
    int hidden;
    int* pos;              // *pos = *next_pos; ++*next_pos
    int* next_pos;
    int* ring;             // ring[*ring_ctr % ring_cap] = token; ++*ring_ctr
    int* ring_ctr;
    int ring_cap;
    unsigned* err;
};

// Transpose-reduce N (power of two, <= 32) per-lane values across a warp: afterwards the
// lanes with (lane % (32 / N)) == 0 hold the warp total of value lane / (32 / N). Each
// halving step exchanges half of the remaining values (N - 1 shuffles), then the survivors
// finish with log2(32 / N) butterfly steps.
template <int N>
__device__ __forceinline__ float reduce_rows(const float (&p)[N], int lane) {
    float v[N];
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = p[i];
#pragma unroll
    for (int n = N, off = 16; n > 1; n >>= 1, off >>= 1) {
        const bool hi = lane & off;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float keep = hi ? v[n / 2 + i] : v[i];
            const float send = hi ? v[i] : v[n / 2 + i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float r = v[0];
#pragma unroll
    for (int off = 16 / N; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
    return r;
}

__device__ __forceinline__ void argmax_merge(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// x of one thread (32 columns) as three signed 8-bit limbs of round(x * 2^S).
struct XLimbs {
    uint32_t le[4][3], lo[4][3];  // even / odd columns of word i, limb l
    int acc_init[3];              // symmetric layout: -8 * sum of limbs (zero folded in)
    float down;                   // 2^(-S-4)
    float xsum;                   // sum of the 32 x values (affine layout offset term)
    float nan_or_zero;            // NaN when x holds a non-finite value (propagates like fp32)
};

// Load this thread's 32 x values and apply the prologue. Inter-phase activations are read
// with ld.global.cg (L2) so a persistent kernel never sees a stale L1 line.
template <int PRO>
__device__ __forceinline__ void gemv_load_x(const GemvParams& p, int t, int lane, int warp, int team, int wpt,
                                            int team_bar, int team_size, float* wsum, float (&xv)[32]) {
    // Every global load of the prologue is issued before the first use: under a saturated
    // memory system each dependent round trip costs microseconds.
    const float4* src = reinterpret_cast<const float4*>(p.x + 32 * t);
    float4 a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = __ldcg(src + i);
    if constexpr (PRO == kProRms) {
        const float4* wn = reinterpret_cast<const float4*>(p.norm_w + 32 * t);
#pragma unroll
        for (int i = 0; i < 8; ++i) b[i] = __ldg(wn + i);
    }
    float4 z[8];
    if constexpr (PRO == kProGatedRms) {
        const float4* gz = reinterpret_cast<const float4*>(p.gate_z + 32 * t);
#pragma unroll
        for (int i = 0; i < 8; ++i) z[i] = __ldcg(gz + i);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        xv[4 * i] = a[i].x;
        xv[4 * i + 1] = a[i].y;
        xv[4 * i + 2] = a[i].z;
        xv[4 * i + 3] = a[i].w;
    }
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
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            xv[4 * i] = xv[4 * i] * inv * b[i].x;
            xv[4 * i + 1] = xv[4 * i + 1] * inv * b[i].y;
            xv[4 * i + 2] = xv[4 * i + 2] * inv * b[i].z;
            xv[4 * i + 3] = xv[4 * i + 3] * inv * b[i].w;
        }
        named_bar(team_bar, team_size);  // wsum may be reused by the next phase
    } else if constexpr (PRO == kProGatedRms) {
        // applyGatedHeadRms (custom_model.cpp:329-349): per head of head_dim columns,
        // out = in * inv * w * silu(z); head_dim/32 consecutive lanes share one head.
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) ss += xv[i] * xv[i];
        const int tph = p.head_dim >> 5;
        for (int o = 1; o < tph; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(p.head_dim) + p.eps);
        // norm_w has head_dim entries shared by every head: an L1 hit for all but one warp.
        const float4* wn = reinterpret_cast<const float4*>(p.norm_w + (32 * t) % p.head_dim);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            b[i] = __ldg(wn + i);
            xv[4 * i] = xv[4 * i] * inv * b[i].x * dsilu(z[i].x);
            xv[4 * i + 1] = xv[4 * i + 1] * inv * b[i].y * dsilu(z[i].y);
            xv[4 * i + 2] = xv[4 * i + 2] * inv * b[i].z * dsilu(z[i].z);
            xv[4 * i + 3] = xv[4 * i + 3] * inv * b[i].w * dsilu(z[i].w);
        }
    }
}

template <int META>
__device__ __forceinline__ void gemv_make_limbs(const float (&xv)[32], XLimbs& L) {
    float amax = 0.0f, xsum = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        amax = fmaxf(amax, fabsf(xv[i]));
        xsum += xv[i];
    }
    const bool finite = isfinite(amax) && isfinite(xsum);
    // Block exponent: amax = f * 2^ex with f in [0.5, 1) (frexpf) for normal amax. A zero or
    // subnormal amax takes the clamp S = 100; every scaled value then rounds to the same
    // integer as with frexpf's exponent (zero stays zero, subnormals already clamp).
    const int ex = ((__float_as_int(amax) >> 23) & 0xff) - 126;
    const int S = max(-100, min(100, 22 - ex));
    const float up = __int_as_float((S + 127) << 23);       // 2^S
    L.down = __int_as_float((127 - S - 4) << 23);           // 2^(-S-4): undoes 2^S and the x16 of the high nibbles
    L.xsum = xsum;
    L.nan_or_zero = finite ? 0.0f : __int_as_float(0x7fc00000);
    // m = round_to_nearest_even(x * 2^S), |m| < 2^22, as the low mantissa bits of
    // x * 2^S + 1.5 * 2^23 (one rounding, in the fma). Its signed base-256 digits
    // (d0 + 256 d1 + 65536 d2, each in [-128, 127]) are the bytes of m + 0x808080 with the top
    // bit of each byte flipped. A non-finite x gives garbage digits; the NaN term replaces the
    // row result then.
    uint32_t u[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        u[i] = static_cast<uint32_t>(__float_as_int(fmaf(xv[i], up, 12582912.0f))) + (0x808080u - 0x4B400000u);
    int zs[3] = {0, 0, 0};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int odd = 0; odd < 2; ++odd) {
            // columns 8i + odd + {0, 2, 4, 6} -> bytes 0..3 of each limb word
            const uint32_t a = u[8 * i + odd], b = u[8 * i + 2 + odd], cc = u[8 * i + 4 + odd],
                           d = u[8 * i + 6 + odd];
            const uint32_t ab01 = __byte_perm(a, b, 0x5140), cd01 = __byte_perm(cc, d, 0x5140);
            const uint32_t ab2 = __byte_perm(a, b, 0x0062), cd2 = __byte_perm(cc, d, 0x0062);
            const uint32_t w0 = __byte_perm(ab01, cd01, 0x5410) ^ 0x80808080u;
            const uint32_t w1 = __byte_perm(ab01, cd01, 0x7632) ^ 0x80808080u;
            const uint32_t w2 = __byte_perm(ab2, cd2, 0x5410) ^ 0x80808080u;
            if (odd) {
                L.lo[i][0] = w0;
                L.lo[i][1] = w1;
                L.lo[i][2] = w2;
            } else {
                L.le[i][0] = w0;
                L.le[i][1] = w1;
                L.le[i][2] = w2;
            }
            if constexpr (META == kMetaSym16) {
                zs[0] = __dp4a(static_cast<int>(w0), 0x01010101, zs[0]);
                zs[1] = __dp4a(static_cast<int>(w1), 0x01010101, zs[1]);
                zs[2] = __dp4a(static_cast<int>(w2), 0x01010101, zs[2]);
            }
        }
    }
#pragma unroll
    for (int l = 0; l < 3; ++l) L.acc_init[l] = (META == kMetaSym16) ? -8 * zs[l] : 0;
}

// Partial dot products of this thread's 32 columns for the first nr (<= RPT) rows of a
// chunk in shared memory. Branch-free over rows (clamped index, predicated result) so the
// shared loads and dp4a chains of all RPT rows overlap.
template <int META, int RPT>
__device__ __forceinline__ void gemv_chunk_partials(const uint8_t* sb, int row_stride, int meta_offset, int t,
                                                    int nr, const XLimbs& L, float (&part)[RPT]) {
    uint4 wv[RPT];
    float sc[RPT], off[RPT];
    // Rows jj >= nr repeat row nr - 1 (the stage may hold fewer than RPT rows); their sums only
    // reach reduction slots of their own row index, which are never stored.
#pragma unroll
    for (int jj = 0; jj < RPT; ++jj) {
        const uint8_t* row = sb + min(jj, nr - 1) * row_stride;
        wv[jj] = ld_shared_v4(row + 16 * t);
        if constexpr (META == kMetaSym16) {
            sc[jj] = __half2float(*reinterpret_cast<const __half*>(row + meta_offset + 2 * (t >> 1)));
            off[jj] = 0.0f;
        } else {
            const float2 sbv = *reinterpret_cast<const float2*>(row + meta_offset + 8 * (t >> 1));
            sc[jj] = sbv.x;
            off[jj] = sbv.y;
        }
    }
#pragma unroll
    for (int jj = 0; jj < RPT; ++jj) {
        const uint32_t ws[4] = {wv[jj].x, wv[jj].y, wv[jj].z, wv[jj].w};
        int ae[3] = {L.acc_init[0], L.acc_init[1], L.acc_init[2]};
        int ao[3] = {0, 0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lw = ws[i] & 0x0F0F0F0Fu;
            const uint32_t hw = ws[i] & 0xF0F0F0F0u;
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
        float val;
        if constexpr (META == kMetaSym16)
            val = dot * (sc[jj] * L.down) + L.nan_or_zero;
        else
            val = dot * (sc[jj] * L.down) + off[jj] * L.xsum + L.nan_or_zero;
        part[jj] = val;
    }
}

// Epilogue of one finished row (everything except argmax and the SwiGLU pair).
template <int EPI>
__device__ __forceinline__ void gemv_epilogue_row(const GemvParams& p, int r, float y) {
    if constexpr (EPI == kEpiStore) {
        p.out[r] = y;
    } else if constexpr (EPI == kEpiResidual) {
        p.out[r] = __ldcg(p.out + r) + y;  // addResidual, custom_model.cpp:294-299
    } else if constexpr (EPI == kEpiConv) {
        if (r < p.conv_channels) {
            // causal conv + SiLU + state shift, custom_model.cpp:985-1006
            const int h = p.conv_k - 1;
            const float* cw = p.conv_w + static_cast<size_t>(r) * p.conv_k;
            float* st = p.conv_state + static_cast<size_t>(r) * h;
            float acc = 0.0f;
            for (int k = 0; k < h; ++k) acc += st[k] * cw[k];
            acc += y * cw[h];
            p.out[r] = dsilu(acc);
            for (int k = 0; k + 1 < h; ++k) st[k] = st[k + 1];
            if (h > 0) st[h - 1] = y;
        } else {
            p.out2[r - p.conv_channels] = y;
        }
    }
}

// Block = `teams` consumer teams of K/32 threads + one producer warp (the last warp).
// The producer streams this block's row chunks into a ring of shared-memory stages with
// 1-D bulk copies (full[s] completes when a stage has landed, empty[s] when its team has
// read it). Consumer team `t` owns chunks t, t + teams, ... and synchronises only within
// the team (named barrier 2 + t), so teams never wait for each other.
template <int META, int PRO, int EPI, int RPT>
__global__ void __launch_bounds__(kMaxBlock, 1) gemv_w4a16_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    float* wsum = reinterpret_cast<float*>(smem + 256);  // one float per warp
    float* red = reinterpret_cast<float*>(smem + 512);   // [2][kMaxRowsPerChunk][32 warps]
    uint8_t* stages = smem + kGemvHeaderBytes;

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int consumers = blockDim.x - 32;
    const int team_size = p.cols >> 5;
    const int teams = consumers / team_size;
    const int R = p.rows_per_chunk;
    const int nst = p.stages;
    const int stage_bytes = R * p.row_stride;

    const int units = p.rows / p.unit;
    const int r_begin = static_cast<int>((long long)units * blockIdx.x / gridDim.x) * p.unit;
    const int r_end = static_cast<int>((long long)units * (blockIdx.x + 1) / gridDim.x) * p.unit;
    const int nchunks = (r_end - r_begin + R - 1) / R;

    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == (consumers >> 5)) {
        // Producer: weights never depend on the previous kernel, so no griddepcontrol.wait.
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int issued = 0;
            for (int ci = 0; ci < nchunks; ++ci) {
                const int s = ci % nst;
                if (ci >= nst && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((ci / nst) - 1) & 1), p.err))
                    break;
                const int row0 = r_begin + ci * R;
                const uint32_t bytes = static_cast<uint32_t>(min(R, r_end - row0) * p.row_stride);
                mbar_expect_tx(&full[s], bytes);
                if (p.evict_first)
                    bulk_g2s_hint(stages + s * stage_bytes, p.w + static_cast<size_t>(row0) * p.row_stride, bytes,
                                  &full[s], pol);
                else
                    bulk_g2s(stages + s * stage_bytes, p.w + static_cast<size_t>(row0) * p.row_stride, bytes,
                             &full[s]);
                ++issued;
            }
            // Every issued copy has landed before this block can exit.
            for (int k = max(0, issued - nst); k < issued; ++k)
                mbar_wait_drain(&full[k % nst], static_cast<uint32_t>((k / nst) & 1));
        }
        return;
    }

    const int team = tid / team_size;
    const int t = tid - team * team_size;
    const int wpt = team_size >> 5;
    const int team_bar = 2 + team;
    pdl_wait();

    XLimbs L;
    {
        float xv[32];
        gemv_load_x<PRO>(p, t, lane, warp, team, wpt, team_bar, team_size, wsum, xv);
        gemv_make_limbs<META>(xv, L);
    }
    float best_v = -INFINITY;
    int best_i = (tid == 0) ? r_begin : 0x7fffffff;

    // ---- stream this team's chunks ------------------------------------------------------
    int it = 0;
    for (int ci = team; ci < nchunks; ci += teams, ++it) {
        const int s = ci % nst;
        const int row0 = r_begin + ci * R;
        const int nr = min(R, r_end - row0);
        mbar_wait_bounded(&full[s], static_cast<uint32_t>((ci / nst) & 1), p.err);
        float part[RPT];
        gemv_chunk_partials<META, RPT>(stages + s * stage_bytes, p.row_stride, p.meta_offset, t, nr, L, part);
        const float v = reduce_rows<RPT>(part, lane);
        float* rbuf = red + (it & 1) * (kMaxRowsPerChunk * 32);
        if ((lane & (32 / RPT - 1)) == 0) {
            const int j = lane / (32 / RPT);
            if (j < nr) rbuf[j * 32 + warp] = v;
        }
        named_bar(team_bar, team_size);
        if (t == 0) mbar_arrive(&empty[s]);  // every thread of the team is done with stage s

        // ---- epilogue for the rows of this chunk (the team's first warp) -------------------
        const int w0 = team * wpt;
        if constexpr (EPI == kEpiSwiglu) {
            if (t < (nr >> 1)) {
                float g = 0.0f, u = 0.0f;
                for (int w = 0; w < wpt; ++w) {
                    g += rbuf[(2 * t) * 32 + w0 + w];
                    u += rbuf[(2 * t + 1) * 32 + w0 + w];
                }
                p.out[(row0 >> 1) + t] = dsilu(g) * u;  // custom_model.cpp:1226-1230
            }
        } else {
            if (t < nr) {
                float y = 0.0f;
                for (int w = 0; w < wpt; ++w) y += rbuf[t * 32 + w0 + w];
                if constexpr (EPI == kEpiArgmax)
                    argmax_merge(best_v, best_i, y, row0 + t);
                else
                    gemv_epilogue_row<EPI>(p, row0 + t, y);
            }
        }
    }

    if constexpr (EPI == kEpiArgmax) {
        // Block result (lowest index on ties, gemvW4A16ArgmaxNeon :309-336), then the last
        // block to finish merges all blocks and runs the optional decode-step head work.
        __shared__ int s_last, s_token;
        __shared__ float s_v[32];
        __shared__ int s_i[32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            argmax_merge(best_v, best_i, ov, oi);
        }
        if (lane == 0) {
            s_v[warp] = best_v;
            s_i[warp] = best_i;
        }
        named_bar(1, consumers);
        if (tid == 0) {
            for (int w = 1; w < (consumers >> 5); ++w) argmax_merge(best_v, best_i, s_v[w], s_i[w]);
            p.part_val[blockIdx.x] = best_v;
            p.part_idx[blockIdx.x] = best_i;
            __threadfence();
            const unsigned done = atomicAdd(p.counter, 1u);
            s_last = (done == gridDim.x - 1) ? 1 : 0;
        }
        named_bar(1, consumers);
        if (s_last) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int b = tid; b < static_cast<int>(gridDim.x); b += consumers)
                argmax_merge(bv, bi, __ldcg(p.part_val + b), __ldcg(p.part_idx + b));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                argmax_merge(bv, bi, ov, oi);
            }
            named_bar(1, consumers);  // s_v / s_i reuse
            if (lane == 0) {
                s_v[warp] = bv;
                s_i[warp] = bi;
            }
            named_bar(1, consumers);
            if (tid == 0) {
                for (int w = 1; w < (consumers >> 5); ++w) argmax_merge(bv, bi, s_v[w], s_i[w]);
                if (bi < 0 || bi >= p.rows) bi = 0;
                s_token = bi;
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
                *p.counter = 0u;  // re-arm for the next launch
            }
            named_bar(1, consumers);
            if (p.emb) {  // loadEmbeddingRow, custom_model.cpp:569-608 (bf16 -> fp32)
                const uint16_t* e = p.emb + static_cast<size_t>(s_token) * p.hidden;
                for (int k = tid; k < p.hidden; k += consumers) p.hidden_out[k] = bf16_to_f32(e[k]);
            }
        }
    }
}

// Generic GEMV for shapes the fused kernel does not serve (any K, any group size): one warp
// per row over the reference's own layout, fp32 dequantise-and-accumulate per group.
__global__ void gemv_generic_kernel(const uint8_t* packed, const float* scales, const float* zeros, int rows,
                                    int cols, int group, int version, const float* x, float* y);

}  // namespace xqb
