// Device implementations shared by the standalone kernels (ops.cu) and the persistent
// decode-step kernel (stepper.cu): Gated-DeltaNet work item, attention work item, helpers.
#pragma once

#include <cuda_fp16.h>

#include "ops.cuh"

namespace xqb {

// Transpose-reduce 16 per-lane values across a warp: lanes 2m and 2m+1 return the warp
// total of value m.
__device__ __forceinline__ float warp_reduce16(const float (&v)[16], int lane) {
    float a[8], b[4], c[2];
    bool h = lane & 16;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const float keep = h ? v[8 + m] : v[m];
        const float send = h ? v[m] : v[8 + m];
        a[m] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    h = lane & 8;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float keep = h ? a[4 + m] : a[m];
        const float send = h ? a[m] : a[4 + m];
        b[m] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    h = lane & 4;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const float keep = h ? b[2 + m] : b[m];
        const float send = h ? b[m] : b[2 + m];
        c[m] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    h = lane & 2;
    float d = (h ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, h ? c[0] : c[1], 2);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    return d;
}

__device__ __forceinline__ void bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// staged: this item's state slice already in shared memory ([dk][kDeltaCols] rows of 64 bytes),
// or null to read it from p.state.
__device__ __forceinline__ void delta_item(const DeltaParams& p, int vh, int slice, int i, int bar_id, DeltaScratch* sh,
                                           const float* staged = nullptr) {
    const int j0 = slice * kDeltaCols;
    const int lane = i & 31, warp = i >> 5;
    const int factor = max(1, p.nv / max(1, p.nk));
    const int kh = min(p.nk - 1, vh / factor);
    // Every global input of the item is requested before any of it is used: one memory round
    // trip instead of one per dependent step.
    float q = __ldcg(p.conv + kh * p.dk + i);
    float k = __ldcg(p.conv + p.nk * p.dk + kh * p.dk + i);
    const float b_in = __ldcg(p.ab + p.nv + vh);
    const float a_in = __ldcg(p.ab + vh);
    const float a_log = p.a_log[vh], dt_bias = p.dt_bias[vh];
    float4* sp = reinterpret_cast<float4*>(p.state + (static_cast<size_t>(vh) * p.dk + i) * p.dv + j0);
    const float4* src = staged ? reinterpret_cast<const float4*>(staged + i * kDeltaCols) : sp;
    const bool fuse = p.z != nullptr;
    const float zi = fuse && i < kDeltaCols ? __ldcg(p.z + vh * p.dv + j0 + i) : 0.0f;
    const float wi = fuse && i < kDeltaCols ? p.norm_w[j0 + i] : 0.0f;
    float s[kDeltaCols], t[kDeltaCols], vj[kDeltaCols];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float4 v = src[m];
        s[4 * m] = v.x;
        s[4 * m + 1] = v.y;
        s[4 * m + 2] = v.z;
        s[4 * m + 3] = v.w;
    }
    const float4* vv4 = reinterpret_cast<const float4*>(p.conv + 2 * p.nk * p.dk + vh * p.dv + j0);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float4 v = __ldcg(vv4 + m);
        vj[4 * m] = v.x;
        vj[4 * m + 1] = v.y;
        vj[4 * m + 2] = v.z;
        vj[4 * m + 3] = v.w;
    }
    float sq = warp_sum(q * q), sk = warp_sum(k * k);
    if (lane == 0) {
        sh->nrm[0][warp] = sq;
        sh->nrm[1][warp] = sk;
    }
    bar_sync(bar_id, 128);
    sq = (sh->nrm[0][0] + sh->nrm[0][1]) + (sh->nrm[0][2] + sh->nrm[0][3]);
    sk = (sh->nrm[1][0] + sh->nrm[1][1]) + (sh->nrm[1][2] + sh->nrm[1][3]);
    q *= 1.0f / sqrtf(sq + 1.0e-6f);
    k *= 1.0f / sqrtf(sk + 1.0e-6f);
    const float beta = dsigmoid(b_in);
    const float gate = -expf(a_log) * dsoftplus(a_in + dt_bias);
    const float decay = expf(gate);
#pragma unroll
    for (int j = 0; j < kDeltaCols; ++j) {
        s[j] *= decay;
        t[j] = s[j] * k;
    }
    float r = warp_reduce16(t, lane);
    if ((lane & 1) == 0) sh->red[warp][lane >> 1] = r;
    bar_sync(bar_id, 128);
    if (i < kDeltaCols) sh->bc[i] = (sh->red[0][i] + sh->red[1][i]) + (sh->red[2][i] + sh->red[3][i]);
    bar_sync(bar_id, 128);
    const float scale = 1.0f / sqrtf(static_cast<float>(p.dk));
#pragma unroll
    for (int j = 0; j < kDeltaCols; ++j) {
        const float delta = beta * (vj[j] - sh->bc[j]);
        s[j] += k * delta;
        t[j] = s[j] * q * scale;
    }
    r = warp_reduce16(t, lane);
    bar_sync(bar_id, 128);  // bc / red reuse
    if ((lane & 1) == 0) sh->red[warp][lane >> 1] = r;
#pragma unroll
    for (int m = 0; m < 4; ++m) sp[m] = make_float4(s[4 * m], s[4 * m + 1], s[4 * m + 2], s[4 * m + 3]);
    bar_sync(bar_id, 128);
    if (i < kDeltaCols) {
        const float o = (sh->red[0][i] + sh->red[1][i]) + (sh->red[2][i] + sh->red[3][i]);
        if (fuse) {
            p.out[vh * p.dv + j0 + i] = o * wi * dsilu(zi);
            float ss = o * o;  // lanes 0..15 of warp 0
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0x0000ffffu, ss, off);
            if (i == 0) p.head_ss[vh * (p.dv / kDeltaCols) + slice] = ss;
        } else {
            p.out[vh * p.dv + j0 + i] = o;
        }
    }
    bar_sync(bar_id, 128);  // the scratch may be reused by the next item
}

template <typename KV>
__device__ __forceinline__ float kv_ld(const KV* p);
template <>
__device__ __forceinline__ float kv_ld<float>(const float* p) {
    return __ldcg(p);
}
template <>
__device__ __forceinline__ float kv_ld<__half>(const __half* p) {
    return __half2float(__ldcg(p));
}
__device__ __forceinline__ void kv_st(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_st(__half* p, float v) { *p = __float2half_rn(v); }

// Head RMSNorm (applyHeadRms, custom_model.cpp:301-313: x *= inv * w) and partial NeoX
// RoPE (applyRopeVector, :351-370) on one head held as v[m] = x[lane + 32 m]. The rotated
// pairs (i, 32 + i), i < 32, are v[0], v[1] of lane i (rotary_dim = 64).
__device__ __forceinline__ void norm_rope_head(float (&v)[8], const float* w, int hd, float eps, int lane,
                                               const float2* rope_row) {
    float ss = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; ++m) ss += v[m] * v[m];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(hd) + eps);
#pragma unroll
    for (int m = 0; m < 8; ++m) v[m] *= inv * w[lane + 32 * m];
    const float2 cs = rope_row[lane];
    const float c = cs.x, s = cs.y;
    const float x0 = v[0], x1 = v[1];
    v[0] = x0 * c - x1 * s;
    v[1] = x1 * c + x0 * s;
}

// Split-K flash decode of one (kv head, split) item: score positions [t0, t1) of kv head kh
// for all its query heads, keep (max, sum, unnormalised output) per head; the last item of a
// kv head to finish merges the splits and applies the sigmoid output gate.
template <typename KV, int SPLITS = kAttnSplits>
__device__ __forceinline__ void attention_item(const AttnParams& p, int kh, int split, int tid, int bar_id, float* dyn,
                               AttnScratch* sh, __nv_bfloat16* out_hi = nullptr,
                               __nv_bfloat16* out_lo = nullptr) {
    const int lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd;
    const int group = p.nq / p.nkv;
    const int cmax = (p.capacity + SPLITS - 1) / SPLITS;
    float* qs = dyn;               // [group][hd]
    float* sc = dyn + group * hd;  // [group][cmax]
    KV* kc = static_cast<KV*>(p.k_cache);
    KV* vc = static_cast<KV*>(p.v_cache);

    const int pos = p.pos_ptr ? __ldcg(p.pos_ptr) : p.pos_const;
    const int L = pos + 1;
    const int chunk = (L + SPLITS - 1) / SPLITS;
    const int t0 = min(L, split * chunk);
    const int t1 = min(L, t0 + chunk);
    const int n = t1 - t0;
    const float2* rope_row = p.rope + static_cast<size_t>(p.rope_stride) * pos;

    if (warp < group) {  // query head kh*group + warp: [query | gate] split (custom_model.cpp:740-753)
        const float* src = p.qkv + static_cast<size_t>(kh * group + warp) * 2 * hd;
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = __ldcg(src + lane + 32 * m);
        norm_rope_head(v, p.q_norm, hd, p.eps, lane, rope_row);
#pragma unroll
        for (int m = 0; m < 8; ++m) qs[warp * hd + lane + 32 * m] = v[m];
    }
    if (pos >= t0 && pos < t1 && warp == kAttnThreads / 32 - 1) {
        // appendKv (custom_model.cpp:673-733): normed + rotated k and raw v at `pos`.
        const float* ks = p.qkv + static_cast<size_t>(p.nq) * 2 * hd + kh * hd;
        const float* vs = ks + static_cast<size_t>(p.nkv) * hd;
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = __ldcg(ks + lane + 32 * m);
        norm_rope_head(v, p.k_norm, hd, p.eps, lane, rope_row);
        KV* kd = kc + (static_cast<size_t>(pos) * p.nkv + kh) * hd;
        KV* vd = vc + (static_cast<size_t>(pos) * p.nkv + kh) * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            kv_st(kd + lane + 32 * m, v[m]);
            kv_st(vd + lane + 32 * m, __ldcg(vs + lane + 32 * m));
        }
        __threadfence_block();
    }
    bar_sync(bar_id, kAttnThreads);

    // scores s = q . k / sqrt(hd) (custom_model.cpp:871-885); warp w takes positions t0 + w,
    // t0 + w + 8, ..., loading three of its K rows per memory round trip
    const float rs = sqrtf(static_cast<float>(hd));
    constexpr int kNW = kAttnThreads / 32;
    for (int tb = t0 + warp; tb < t1; tb += 3 * kNW) {
        float kv[3][8];
#pragma unroll
        for (int u = 0; u < 3; ++u) {
            const int t = tb + u * kNW;
            const KV* kr = kc + (static_cast<size_t>(min(t, t1 - 1)) * p.nkv + kh) * hd;
#pragma unroll
            for (int m = 0; m < 8; ++m) kv[u][m] = t < t1 ? kv_ld(kr + lane + 32 * m) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 3; ++u) {
            const int t = tb + u * kNW;
            if (t >= t1) break;
            for (int g = 0; g < group; ++g) {
                float d = 0.0f;
#pragma unroll
                for (int m = 0; m < 8; ++m) d += qs[g * hd + lane + 32 * m] * kv[u][m];
                d = warp_sum(d);
                if (lane == 0) sc[g * cmax + (t - t0)] = d / rs;
            }
        }
    }
    bar_sync(bar_id, kAttnThreads);
    if (warp < group) {  // local max-subtracted exponentials (custom_model.cpp:890-905)
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[warp * cmax + j]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int j = lane; j < n; j += 32) {
            const float e = expf(sc[warp * cmax + j] - mx);
            sc[warp * cmax + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            sh->m[warp] = mx;
            sh->l[warp] = l;
        }
    }
    bar_sync(bar_id, kAttnThreads);
    float o[kAttnMaxGroup];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) o[g] = 0.0f;
    for (int j0 = 0; j0 < n; j0 += 24) {  // V reduction (custom_model.cpp:910-928), thread = dim
        float vb[24];                       // 24 requests in flight per round trip
#pragma unroll
        for (int u = 0; u < 24; ++u)
            vb[u] = j0 + u < n ? kv_ld(vc + (static_cast<size_t>(t0 + j0 + u) * p.nkv + kh) * hd + tid) : 0.0f;
#pragma unroll
        for (int u = 0; u < 24; ++u)
            if (j0 + u < n) {
#pragma unroll
                for (int g = 0; g < kAttnMaxGroup; ++g)
                    if (g < group) o[g] += sc[g * cmax + j0 + u] * vb[u];
            }
    }
    float* pp = p.part + static_cast<size_t>(kh * SPLITS + split) * group * (hd + 2);
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g)
        if (g < group) pp[g * (hd + 2) + tid] = o[g];
    if (tid < group) {
        pp[tid * (hd + 2) + hd] = sh->m[tid];
        pp[tid * (hd + 2) + hd + 1] = sh->l[tid];
    }
    __threadfence();
    bar_sync(bar_id, kAttnThreads);
    if (tid == 0) sh->last = (atomicAdd(&p.counters[kh], 1u) == SPLITS - 1) ? 1 : 0;
    bar_sync(bar_id, kAttnThreads);
    if (sh->last) {
        __threadfence();
        // Merge the splits in parallel: (max, sum) of every (split, head) pair to shared memory,
        // one rescale weight per pair, then thread d sums its dimension over the splits.
        const float* base = p.part + static_cast<size_t>(kh * SPLITS) * group * (hd + 2);
        float gate[kAttnMaxGroup];  // output gates, loaded with the (max, sum) pairs
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g)
            gate[g] = g < group ? __ldcg(p.qkv + static_cast<size_t>(kh * group + g) * 2 * hd + hd + tid) : 0.0f;
        if (tid < SPLITS * group) {
            const float* ps = base + tid * (hd + 2);  // tid = split * group + g
            sh->pm[tid] = __ldcg(ps + hd);
            sh->pl[tid] = __ldcg(ps + hd + 1);
        }
        bar_sync(bar_id, kAttnThreads);
        if (tid < group) {
            float M = -INFINITY;
            for (int s2 = 0; s2 < SPLITS; ++s2) M = fmaxf(M, sh->pm[s2 * group + tid]);
            float Ls = 0.0f;
            for (int s2 = 0; s2 < SPLITS; ++s2) Ls += sh->pl[s2 * group + tid] * expf(sh->pm[s2 * group + tid] - M);
            sh->M[tid] = M;
            sh->invL[tid] = Ls > 0.0f ? 1.0f / Ls : 0.0f;
        }
        bar_sync(bar_id, kAttnThreads);
        if (tid < SPLITS * group) sh->pm[tid] = expf(sh->pm[tid] - sh->M[tid % group]);
        bar_sync(bar_id, kAttnThreads);
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g) {
            if (g >= group) break;
            float part[SPLITS];  // every split of this head in flight in one round trip
#pragma unroll
            for (int u = 0; u < SPLITS; ++u) part[u] = __ldcg(base + (u * group + g) * (hd + 2) + tid);
            float O = 0.0f;
#pragma unroll
            for (int u = 0; u < SPLITS; ++u) O += part[u] * sh->pm[u * group + g];
            const int qh = kh * group + g;
            const float val = (O * sh->invL[g]) * dsigmoid(gate[g]);  // output gate, custom_model.cpp:944-946
            if (out_hi) {  // batched decode: the o_proj GEMM operands as a bf16 pair
                const __nv_bfloat16 h = __float2bfloat16_rn(val);
                out_hi[qh * hd + tid] = h;
                out_lo[qh * hd + tid] = __float2bfloat16_rn(val - __bfloat162float(h));
            } else {
                p.out[qh * hd + tid] = val;
            }
        }
        if (tid == 0) p.counters[kh] = 0u;
    }
    bar_sync(bar_id, kAttnThreads);  // scratch reuse by the caller's next item
}


}  // namespace xqb
