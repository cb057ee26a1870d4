// Generic-shape decode step: the per-token operations of CustomModel for any dimensions the
// package's manifest gives (head_dim, rotary_dim, key / value head dims, conv kernel, group
// size), for models the fused step kernels do not serve (for example the reference's tiny
// runtime-test model). Plain single-block kernels with the reference's loops and operation
// order; the GEMVs run on the generic-layout kernel (launch_gemv_generic). Slow on purpose-built
// shapes, exact in the reference's fp32 order where the reference is sequential.
#include <cuda_runtime.h>

#include <cmath>

#include "common.cuh"
#include "generic.hpp"

namespace xqb {

namespace {

// One block. Causal conv + SiLU + state shift (custom_model.cpp:985-1006, any kernel size),
// q / k l2 norm per key head (:315-327), gate math (:1075-1082) and the gated delta rule
// (ref_delta.cpp:8-41) per value head, then the gated head RMSNorm (:329-349). proj:
// [qkv (conv_dim) | z (nv*dv) | a (nv) | b (nv)]; conv scratch: conv_dim floats; out: nv*dv.
__global__ void generic_linear_attn_kernel(const float* proj, const float* conv_w, float* conv_state,
                                           const float* a_log, const float* dt_bias, float* rec_state,
                                           const float* norm_w, float eps, float* conv, float* out, int nk, int nv,
                                           int dk, int dv, int kconv) {
    const int conv_dim = 2 * nk * dk + nv * dv;
    const int hist = kconv > 1 ? kconv - 1 : 0;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int c = tid; c < conv_dim; c += nt) {
        float acc = 0.0f;
        for (int k = 0; k < hist; ++k) acc += conv_state[c * hist + k] * conv_w[c * kconv + k];
        acc += proj[c] * conv_w[c * kconv + hist];
        conv[c] = acc / (1.0f + expf(-acc));
        float* st = conv_state + c * hist;
        for (int k = 0; k + 1 < hist; ++k) st[k] = st[k + 1];
        if (hist > 0) st[hist - 1] = proj[c];
    }
    __syncthreads();
    for (int h = tid; h < 2 * nk; h += nt) {  // q heads then k heads
        float* base = conv + h * dk;
        float sum = 0.0f;
        for (int d = 0; d < dk; ++d) sum += base[d] * base[d];
        const float inv = 1.0f / sqrtf(sum + 1.0e-6f);
        for (int d = 0; d < dk; ++d) base[d] *= inv;
    }
    __syncthreads();
    const float* z = proj + conv_dim;
    const float* av = z + nv * dv;
    const float* bv = av + nv;
    const int factor = max(1, nv / max(1, nk));
    const float scale = 1.0f / sqrtf(static_cast<float>(dk));
    for (int vh = tid; vh < nv; vh += nt) {
        const int kh = min(nk - 1, vh / factor);
        const float* q = conv + kh * dk;
        const float* k = conv + nk * dk + kh * dk;
        const float* v = conv + 2 * nk * dk + vh * dv;
        const float bx = bv[vh];
        const float beta = bx >= 0.0f ? 1.0f / (1.0f + expf(-bx)) : expf(bx) / (1.0f + expf(bx));
        const float sx = av[vh] + dt_bias[vh];
        const float sp = sx > 20.0f ? sx : (sx < -20.0f ? expf(sx) : log1pf(expf(sx)));
        const float gate = -expf(a_log[vh]) * sp;
        const float decay = expf(gate);
        float* st = rec_state + static_cast<size_t>(vh) * dk * dv;
        for (int i = 0; i < dk * dv; ++i) st[i] *= decay;
        for (int j = 0; j < dv; ++j) {
            float pred = 0.0f;
            for (int i = 0; i < dk; ++i) pred += st[i * dv + j] * k[i];
            const float delta = beta * (v[j] - pred);
            for (int i = 0; i < dk; ++i) st[i * dv + j] += k[i] * delta;
        }
        float* o = out + vh * dv;
        for (int j = 0; j < dv; ++j) {
            float acc = 0.0f;
            for (int i = 0; i < dk; ++i) acc += st[i * dv + j] * q[i] * scale;
            o[j] = acc;
        }
        // applyGatedHeadRms: o * inv * w * silu(z)
        float sum = 0.0f;
        for (int d = 0; d < dv; ++d) sum += o[d] * o[d];
        const float inv = 1.0f / sqrtf(sum / static_cast<float>(dv) + eps);
        const float* zz = z + vh * dv;
        for (int d = 0; d < dv; ++d) o[d] = o[d] * inv * norm_w[d] * (zz[d] / (1.0f + expf(-zz[d])));
    }
}

// One block. Full attention at *pos (custom_model.cpp:735-946): [query | gate] split per head
// when q_proj carries both (else the gate is 0, sigmoid 0.5, as the reference does), head
// RMSNorm of q and k, partial RoPE from the (cos, sin) table, KV append, GQA softmax attention
// over positions 0..pos and the sigmoid output gate. proj: [q rows | k (nkv*hd) | v (nkv*hd)];
// scores: scratch [nq][capacity]; qbuf: nq*hd + nkv*hd floats; out: nq*hd.
__global__ void generic_attention_kernel(const float* proj, int q_rows, const float* q_norm, const float* k_norm,
                                         const float2* rope, int rope_stride, float* kc, float* vc, const int* pos_ptr,
                                         float* scores, float* qbuf, float* out, int nq, int nkv, int hd, int rotary,
                                         float eps) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const int pos = *pos_ptr;
    const int L = pos + 1;
    const bool gated = q_rows >= nq * 2 * hd;
    const float* kp = proj + q_rows;
    const float* vp = kp + nkv * hd;
    float* q = qbuf;
    float* k = qbuf + nq * hd;
    const int active = max(0, min(hd, rotary)), half = active / 2;
    const float2* rr = rope + static_cast<size_t>(rope_stride) * pos;
    for (int h = tid; h < nq + nkv; h += nt) {
        float* base = h < nq ? q + h * hd : k + (h - nq) * hd;
        const float* src = h < nq ? proj + (gated ? h * 2 * hd : h * hd) : kp + (h - nq) * hd;
        const float* w = h < nq ? q_norm : k_norm;
        float sum = 0.0f;
        for (int d = 0; d < hd; ++d) {
            base[d] = src[d];
            sum += base[d] * base[d];
        }
        const float inv = 1.0f / sqrtf(sum / static_cast<float>(hd) + eps);
        for (int d = 0; d < hd; ++d) base[d] *= inv * w[d];
        for (int i = 0; i < half; ++i) {
            const float c = rr[i].x, s = rr[i].y;
            const float x0 = base[i], x1 = base[half + i];
            base[i] = x0 * c - x1 * s;
            base[half + i] = x1 * c + x0 * s;
        }
    }
    __syncthreads();
    for (int e = tid; e < nkv * hd; e += nt) {  // appendKv at pos
        kc[static_cast<size_t>(pos) * nkv * hd + e] = k[e];
        vc[static_cast<size_t>(pos) * nkv * hd + e] = vp[e];
    }
    __syncthreads();
    const int group = max(1, nq / max(1, nkv));
    const float rs = sqrtf(static_cast<float>(hd));
    for (int h = tid; h < nq; h += nt) {
        const int kh = min(nkv - 1, h / group);
        const float* qv = q + h * hd;
        float* sc = scores + static_cast<size_t>(h) * L;
        float mx = -INFINITY;
        for (int t = 0; t < L; ++t) {
            const float* kv = kc + (static_cast<size_t>(t) * nkv + kh) * hd;
            float dot = 0.0f;
            for (int d = 0; d < hd; ++d) dot += qv[d] * kv[d];
            const float s = dot / rs;
            sc[t] = s;
            mx = fmaxf(mx, s);
        }
        float denom = 0.0f;
        for (int t = 0; t < L; ++t) {
            sc[t] = expf(sc[t] - mx);
            denom += sc[t];
        }
        const float inv = denom > 0.0f ? 1.0f / denom : 0.0f;
        for (int t = 0; t < L; ++t) sc[t] *= inv;
        float* o = out + h * hd;
        for (int d = 0; d < hd; ++d) o[d] = 0.0f;
        for (int t = 0; t < L; ++t) {
            const float* vv = vc + (static_cast<size_t>(t) * nkv + kh) * hd;
            for (int d = 0; d < hd; ++d) o[d] += sc[t] * vv[d];
        }
        for (int d = 0; d < hd; ++d) {
            const float g = gated ? proj[h * 2 * hd + hd + d] : 0.0f;
            const float sg = g >= 0.0f ? 1.0f / (1.0f + expf(-g)) : expf(g) / (1.0f + expf(g));
            o[d] *= sg;
        }
    }
}

// h[j] = silu(gu[2j]) * gu[2j+1] (interleaved gate / up rows, custom_model.cpp:1226-1230).
__global__ void generic_swiglu_kernel(const float* gu, float* h, int inter) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < inter; j += gridDim.x * blockDim.x) {
        const float g = gu[2 * j];
        h[j] = g / (1.0f + expf(-g)) * gu[2 * j + 1];
    }
}

// hidden += y (addResidual, custom_model.cpp:294-299).
__global__ void generic_add_kernel(float* hidden, const float* y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) hidden[i] += y[i];
}

// One block: greedy sample (argmax over the logits, ties to the lowest index, as
// gemvW4A16ArgmaxNeon), then load that token's embedding row and advance the positions
// (custom_model.cpp:1340-1356, 569-608); the token into token_out and the ring.
__global__ void generic_sample_kernel(const float* logits, int vocab, const uint16_t* emb, float* hidden, int H,
                                      int* pos, int* next_pos, int* token_out, int* ring, int* ring_ctr, int ring_cap) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int tok;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int k = threadIdx.x; k < vocab; k += blockDim.x)
        if (logits[k] > bv) {
            bv = logits[k];
            bi = k;
        }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        if (bi < 0 || bi >= vocab) bi = 0;
        tok = bi;
        if (token_out) *token_out = bi;
        if (ring) {
            const int k = *ring_ctr;
            ring[k % ring_cap] = bi;
            *ring_ctr = k + 1;
        }
        const int np = *next_pos;
        *pos = np;
        *next_pos = np + 1;
    }
    __syncthreads();
    const uint16_t* e = emb + static_cast<size_t>(tok) * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x) hidden[k] = bf16_to_f32(e[k]);
}

}  // namespace

cudaError_t generic_linear_attn(const GenericLinearArgs& a, cudaStream_t s) {
    generic_linear_attn_kernel<<<1, 256, 0, s>>>(a.proj, a.conv_w, a.conv_state, a.a_log, a.dt_bias, a.rec_state,
                                                 a.norm_w, a.eps, a.conv, a.out, a.nk, a.nv, a.dk, a.dv, a.kconv);
    return cudaGetLastError();
}

cudaError_t generic_attention(const GenericAttnArgs& a, cudaStream_t s) {
    generic_attention_kernel<<<1, 256, 0, s>>>(a.proj, a.q_rows, a.q_norm, a.k_norm, a.rope, a.rope_stride, a.k_cache,
                                               a.v_cache, a.pos, a.scores, a.qbuf, a.out, a.nq, a.nkv, a.hd, a.rotary,
                                               a.eps);
    return cudaGetLastError();
}

cudaError_t generic_swiglu(const float* gu, float* h, int inter, cudaStream_t s) {
    generic_swiglu_kernel<<<(inter + 255) / 256, 256, 0, s>>>(gu, h, inter);
    return cudaGetLastError();
}

cudaError_t generic_add(float* hidden, const float* y, int n, cudaStream_t s) {
    generic_add_kernel<<<(n + 255) / 256, 256, 0, s>>>(hidden, y, n);
    return cudaGetLastError();
}

cudaError_t generic_sample(const float* logits, int vocab, const uint16_t* emb, float* hidden, int H, int* pos,
                           int* next_pos, int* token_out, int* ring, int* ring_ctr, int ring_cap, cudaStream_t s) {
    generic_sample_kernel<<<1, 1024, 0, s>>>(logits, vocab, emb, hidden, H, pos, next_pos, token_out, ring, ring_ctr,
                                             ring_cap);
    return cudaGetLastError();
}

}  // namespace xqb
