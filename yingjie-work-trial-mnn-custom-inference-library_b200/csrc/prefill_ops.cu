// Batched prefill (prefill_kv_build over all prompt tokens at once): the per-token operations of
// CustomModel::prefill (custom_model.cpp:610-640) restated over a [tokens][width] batch, around
// the tensor-core GEMMs of prefill_gemm.cu. Each kernel keeps the per-element arithmetic (and
// order) of the decode path's kernels, so the batched prefill agrees with the token-serial one
// to fp32 rounding plus the GEMMs' split-bf16 error.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemv.hpp"
#include "ops_device.cuh"
#include "prefill_ops.hpp"

namespace xqb {

namespace {

// Every kernel of this file waits for its predecessor with griddepcontrol.wait before touching
// memory, so all are launched with the programmatic-dependent-launch attribute: the launch and
// block scheduling overlap the previous kernel's tail, and a following tensor-core GEMM can
// start streaming its weights.
template <typename Kernel, typename... Args>
cudaError_t pdl_launch(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    return launch_ex(kernel, grid, block, smem, s, pdl_enabled(), args...);
}

__device__ __forceinline__ void store_split(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    if (lo) lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
}

// H[t] = embedding row of ids[t] (ids folded by abs % vocab, custom_model.cpp:573-575).
__global__ void embed_rows_kernel(const int* ids, const uint16_t* emb, float* H, int hidden, int vocab) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    const int t = blockIdx.x;
    long long id = ids[t];
    if (id < 0 || id >= vocab) id = (id < 0 ? -id : id) % (vocab > 1 ? vocab : 1);
    const uint16_t* e = emb + static_cast<size_t>(id) * hidden;
    for (int k = threadIdx.x; k < hidden; k += blockDim.x) H[static_cast<size_t>(t) * hidden + k] = bf16_to_f32(e[k]);
}

// X[t] = rmsnorm(H[t]) * w as a bf16 pair (rmsnormReference, ref_rmsnorm.cpp:8-17). 256 threads.
__global__ void rmsnorm_split_kernel(const float* H, const float* w, int n, float eps, __nv_bfloat16* hi,
                                     __nv_bfloat16* lo) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    __shared__ float ws[8];
    const int t = blockIdx.x;
    const float* x = H + static_cast<size_t>(t) * n;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < n; k += blockDim.x) ss += x[k] * x[k];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += ws[i];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        store_split(hi, lo, static_cast<size_t>(t) * n + k, x[k] * inv * w[k]);
}

// The same for rows of at most 8192 floats (n % 4 == 0): every thread loads its float4s before
// any arithmetic, so a row is one memory round trip instead of one per loop iteration.
__global__ void __launch_bounds__(256) rmsnorm_split_vec_kernel(const float* H, const float* w, int n, float eps,
                                                                __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    constexpr int kV = 8;  // float4s per thread held in registers
    __shared__ float ws[8];
    const int t = blockIdx.x, n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(H + static_cast<size_t>(t) * n);
    float4 v[kV];
#pragma unroll
    for (int i = 0; i < kV; ++i) {
        const int k = threadIdx.x + i * 256;
        v[i] = k < n4 ? x4[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kV; ++i) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += ws[i];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
    for (int i = 0; i < kV; ++i) {
        const int k = threadIdx.x + i * 256;
        if (k >= n4) break;
        const float4 g = w4[k];
        const float o[4] = {v[i].x * inv * g.x, v[i].y * inv * g.y, v[i].z * inv * g.z, v[i].w * inv * g.w};
        __nv_bfloat16 h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = __float2bfloat16_rn(o[j]);
            l[j] = __float2bfloat16_rn(o[j] - __bfloat162float(h[j]));
        }
        const size_t e = static_cast<size_t>(t) * n + 4 * static_cast<size_t>(k);
        *reinterpret_cast<uint2*>(hi + e) = *reinterpret_cast<const uint2*>(h);
        if (lo) *reinterpret_cast<uint2*>(lo + e) = *reinterpret_cast<const uint2*>(l);
    }
}

// Causal conv1d + SiLU over the sequence, then the state shift (custom_model.cpp:985-1006,
// conv_k = 4): one thread per channel walks the tokens in order. Y: [n][ldy] projections (the
// first `channels` columns), out: [n][channels], state: [channels][3], updated in place.
// blockIdx.y = sequence: rows [y n, y n + n) with its own state at state + y * state_bstride
// (batched decode: n = 1 per sequence).
__global__ void conv_seq_kernel(const float* Y, int ldy, const float* w, float* state, float* out, int n, int channels,
                                size_t state_bstride) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    Y += static_cast<size_t>(blockIdx.y) * n * ldy;
    out += static_cast<size_t>(blockIdx.y) * n * channels;
    state += blockIdx.y * state_bstride;
    const float4 cw = *reinterpret_cast<const float4*>(w + static_cast<size_t>(c) * 4);
    float s0 = state[3 * c], s1 = state[3 * c + 1], s2 = state[3 * c + 2];
    for (int t = 0; t < n; ++t) {
        const float y = Y[static_cast<size_t>(t) * ldy + c];
        float acc = 0.0f;
        acc += s0 * cw.x;
        acc += s1 * cw.y;
        acc += s2 * cw.z;
        acc += y * cw.w;
        out[static_cast<size_t>(t) * channels + c] = dsilu(acc);
        s0 = s1;
        s1 = s2;
        s2 = y;
    }
    state[3 * c] = s0;
    state[3 * c + 1] = s1;
    state[3 * c + 2] = s2;
}

// The gated delta rule over the sequence for one (value head, 16-column slice): delta_item's
// arithmetic token after token with the state slice held in registers (thread i = key row i).
// q | k | v of token t: conv[t] (width 2*nk*dk + nv*dv); a, b: Y[t][ab_off + vh], [.. + nv + vh].
// The next token's inputs are loaded while the current one is processed.
// blockIdx.z = sequence: rows [z n, z n + n), its recurrent state at state + z * state_bstride.
__global__ void __launch_bounds__(128) delta_seq_kernel(const float* conv, int conv_ld, const float* Y, int ldy,
                                                        int ab_off, const float* a_log_p, const float* dt_bias_p,
                                                        float* state, float* out, int out_ld, int n, int nk, int nv,
                                                        int dk, int dv, size_t state_bstride) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    __shared__ DeltaScratch sh;
    conv += static_cast<size_t>(blockIdx.z) * n * conv_ld;
    Y += static_cast<size_t>(blockIdx.z) * n * ldy;
    out += static_cast<size_t>(blockIdx.z) * n * out_ld;
    state += blockIdx.z * state_bstride;
    const int vh = blockIdx.x, j0 = blockIdx.y * kDeltaCols;
    const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
    const int factor = max(1, nv / max(1, nk));
    const int kh = min(nk - 1, vh / factor);
    const float a_log = a_log_p[vh], dt_bias = dt_bias_p[vh];
    float4* sp = reinterpret_cast<float4*>(state + (static_cast<size_t>(vh) * dk + i) * dv + j0);
    float s[kDeltaCols], tt[kDeltaCols];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float4 v = sp[m];
        s[4 * m] = v.x;
        s[4 * m + 1] = v.y;
        s[4 * m + 2] = v.z;
        s[4 * m + 3] = v.w;
    }
    const float scale = 1.0f / sqrtf(static_cast<float>(dk));
    // inputs of token t
    auto load = [&](int t, float& q, float& k, float& a_in, float& b_in, float (&vj)[kDeltaCols]) {
        const float* c = conv + static_cast<size_t>(t) * conv_ld;
        q = c[kh * dk + i];
        k = c[nk * dk + kh * dk + i];
        a_in = Y[static_cast<size_t>(t) * ldy + ab_off + vh];
        b_in = Y[static_cast<size_t>(t) * ldy + ab_off + nv + vh];
        const float4* v4 = reinterpret_cast<const float4*>(c + 2 * nk * dk + vh * dv + j0);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float4 v = v4[m];
            vj[4 * m] = v.x;
            vj[4 * m + 1] = v.y;
            vj[4 * m + 2] = v.z;
            vj[4 * m + 3] = v.w;
        }
    };
    float q, k, a_in, b_in, vj[kDeltaCols];
    load(0, q, k, a_in, b_in, vj);
    for (int t = 0; t < n; ++t) {
        float nq_ = 0.0f, nk_ = 0.0f, na = 0.0f, nb = 0.0f, nv_[kDeltaCols];
        if (t + 1 < n) load(t + 1, nq_, nk_, na, nb, nv_);
        float sq = warp_sum(q * q), sk = warp_sum(k * k);
        if (lane == 0) {
            sh.nrm[0][warp] = sq;
            sh.nrm[1][warp] = sk;
        }
        __syncthreads();
        sq = (sh.nrm[0][0] + sh.nrm[0][1]) + (sh.nrm[0][2] + sh.nrm[0][3]);
        sk = (sh.nrm[1][0] + sh.nrm[1][1]) + (sh.nrm[1][2] + sh.nrm[1][3]);
        const float qn = q * (1.0f / sqrtf(sq + 1.0e-6f));
        const float kn = k * (1.0f / sqrtf(sk + 1.0e-6f));
        const float beta = dsigmoid(b_in);
        const float gate = -expf(a_log) * dsoftplus(a_in + dt_bias);
        const float decay = expf(gate);
#pragma unroll
        for (int j = 0; j < kDeltaCols; ++j) {
            s[j] *= decay;
            tt[j] = s[j] * kn;
        }
        float r = warp_reduce16(tt, lane);
        if ((lane & 1) == 0) sh.red[warp][lane >> 1] = r;
        __syncthreads();
        if (i < kDeltaCols) sh.bc[i] = (sh.red[0][i] + sh.red[1][i]) + (sh.red[2][i] + sh.red[3][i]);
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kDeltaCols; ++j) {
            const float delta = beta * (vj[j] - sh.bc[j]);
            s[j] += kn * delta;
            tt[j] = s[j] * qn * scale;
        }
        r = warp_reduce16(tt, lane);
        __syncthreads();  // bc / red reuse
        if ((lane & 1) == 0) sh.red[warp][lane >> 1] = r;
        __syncthreads();
        if (i < kDeltaCols)
            out[static_cast<size_t>(t) * out_ld + vh * dv + j0 + i] =
                (sh.red[0][i] + sh.red[1][i]) + (sh.red[2][i] + sh.red[3][i]);
        q = nq_;
        k = nk_;
        a_in = na;
        b_in = nb;
#pragma unroll
        for (int j = 0; j < kDeltaCols; ++j) vj[j] = nv_[j];
        // the next token's first shared write (nrm) is ordered after these reads by the barrier
        // that follows it; red is rewritten only after two more barriers
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) sp[m] = make_float4(s[4 * m], s[4 * m + 1], s[4 * m + 2], s[4 * m + 3]);
}

// Gated head RMSNorm (applyGatedHeadRms, custom_model.cpp:329-349: o * inv * w * silu(z), w
// without +1) of token t, head h, as a bf16 pair. One warp per (t, head), head_dim 128.
__global__ void gated_norm_split_kernel(const float* O, int o_ld, const float* Y, int ldy, int z_off, const float* w,
                                        int heads, int hd, float eps, int n, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (gw >= n * heads) return;
    const int t = gw / heads, h = gw % heads;
    const float* o = O + static_cast<size_t>(t) * o_ld + h * hd;
    const float* z = Y + static_cast<size_t>(t) * ldy + z_off + h * hd;
    float ss = 0.0f;
    for (int d = lane; d < hd; d += 32) ss += o[d] * o[d];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(hd) + eps);
    for (int d = lane; d < hd; d += 32)
        store_split(hi, lo, static_cast<size_t>(t) * heads * hd + h * hd + d, o[d] * inv * w[d] * dsilu(z[d]));
}

// Attention prologue of token t (position p0 + t): per query head the [query | gate] split,
// head RMSNorm and partial RoPE of the query (into Q [n][nq][hd]); per kv head the normed and
// rotated k and the raw v appended to the KV cache (appendKv, custom_model.cpp:673-733). One
// warp per (t, head) of nq + nkv; norm_rope_head is the decode path's arithmetic.
// pos_arr (batched decode): row t is sequence t at position pos_arr[t] with its KV cache at
// kc / vc + t * kv_bstride; null: one sequence, row t at position p0 + t.
template <typename KV>
__global__ void attn_prep_kernel(const float* Y, int ldy, const float* q_norm, const float* k_norm, const float2* rope,
                                 int rope_stride, float* Q, KV* kc, KV* vc, int p0, int n, int nq, int nkv, int hd,
                                 float eps, const int* pos_arr, size_t kv_bstride) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (gw >= n * (nq + nkv)) return;
    const int t = gw / (nq + nkv), h = gw % (nq + nkv);
    const int pos = pos_arr ? pos_arr[t] : p0 + t;
    if (pos_arr) {
        kc += t * kv_bstride;
        vc += t * kv_bstride;
    }
    const float* y = Y + static_cast<size_t>(t) * ldy;
    const float2* rope_row = rope + static_cast<size_t>(rope_stride) * pos;
    float v[8];
    if (h < nq) {
        const float* src = y + static_cast<size_t>(h) * 2 * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = src[lane + 32 * m];
        norm_rope_head(v, q_norm, hd, eps, lane, rope_row);
        float* dst = Q + (static_cast<size_t>(t) * nq + h) * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) dst[lane + 32 * m] = v[m];
    } else {
        const int kh = h - nq;
        const float* ks = y + static_cast<size_t>(nq) * 2 * hd + kh * hd;
        const float* vs = ks + static_cast<size_t>(nkv) * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = ks[lane + 32 * m];
        norm_rope_head(v, k_norm, hd, eps, lane, rope_row);
        KV* kd = kc + (static_cast<size_t>(pos) * nkv + kh) * hd;
        KV* vd = vc + (static_cast<size_t>(pos) * nkv + kh) * hd;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            kv_st(kd + lane + 32 * m, v[m]);
            kv_st(vd + lane + 32 * m, vs[lane + 32 * m]);
        }
    }
}

// Causal GQA attention of token t (custom_model.cpp:871-946) for the query heads of kv head kh:
// scores over positions 0 .. p0 + t, max-subtracted exponentials, the normalised V sum and the
// sigmoid output gate, written as a bf16 pair (the o_proj GEMM input). 256 threads (thread =
// head dimension in the V sum); dynamic shared memory: group * hd (queries) + group * L (scores).
template <typename KV>
__global__ void __launch_bounds__(256) attn_causal_kernel(const float* Q, const float* Y, int ldy, const KV* kc,
                                                          const KV* vc, int p0, int nq, int nkv, int hd,
                                                          __nv_bfloat16* hi, __nv_bfloat16* lo, const int* pos_arr,
                                                          size_t kv_bstride) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    extern __shared__ float dyn[];
    const int t = blockIdx.x, kh = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int group = nq / nkv;
    const int L = (pos_arr ? pos_arr[t] : p0 + t) + 1;
    if (pos_arr) {
        kc += t * kv_bstride;
        vc += t * kv_bstride;
    }
    float* qs = dyn;               // [group][hd]
    float* sc = dyn + group * hd;  // [group][L]
    __shared__ float red_m[kAttnMaxGroup], red_l[kAttnMaxGroup];
    for (int e = tid; e < group * hd; e += blockDim.x)
        qs[e] = Q[(static_cast<size_t>(t) * nq + kh * group) * hd + e];
    __syncthreads();
    const float rs = sqrtf(static_cast<float>(hd));
    for (int u = warp; u < L; u += 8) {  // scores (custom_model.cpp:871-885)
        const KV* kr = kc + (static_cast<size_t>(u) * nkv + kh) * hd;
        float kv[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) kv[m] = kv_ld(kr + lane + 32 * m);
        for (int g = 0; g < group; ++g) {
            float d = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; ++m) d += qs[g * hd + lane + 32 * m] * kv[m];
            d = warp_sum(d);
            if (lane == 0) sc[g * L + u] = d / rs;
        }
    }
    __syncthreads();
    if (warp < group) {  // softmax (custom_model.cpp:890-905)
        float mx = -INFINITY;
        for (int j = lane; j < L; j += 32) mx = fmaxf(mx, sc[warp * L + j]);
        mx = warp_max(mx);
        float l = 0.0f;
        for (int j = lane; j < L; j += 32) {
            const float e = expf(sc[warp * L + j] - mx);
            sc[warp * L + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            red_m[warp] = mx;
            red_l[warp] = l > 0.0f ? 1.0f / l : 0.0f;
        }
    }
    __syncthreads();
    float o[kAttnMaxGroup];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) o[g] = 0.0f;
    for (int j0 = 0; j0 < L; j0 += 16) {  // V sum (custom_model.cpp:910-928), thread = dimension
        float vb[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
            vb[u] = j0 + u < L ? kv_ld(vc + (static_cast<size_t>(j0 + u) * nkv + kh) * hd + tid) : 0.0f;
#pragma unroll
        for (int u = 0; u < 16; ++u)
            if (j0 + u < L) {
#pragma unroll
                for (int g = 0; g < kAttnMaxGroup; ++g)
                    if (g < group) o[g] += sc[g * L + j0 + u] * vb[u];
            }
    }
    const float* yq = Y + static_cast<size_t>(t) * ldy;
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g) {
        if (g >= group) break;
        const int qh = kh * group + g;
        const float gate = yq[static_cast<size_t>(qh) * 2 * hd + hd + tid];
        store_split(hi, lo, static_cast<size_t>(t) * nq * hd + qh * hd + tid, (o[g] * red_l[g]) * dsigmoid(gate));
    }
}

// SwiGLU of the interleaved gate/up rows (custom_model.cpp:1226-1230) as a bf16 pair.
__global__ void swiglu_split_kernel(const float* Y, int ldy, int inter, int n, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    const size_t e = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<size_t>(n) * inter) return;
    const size_t t = e / inter, j = e % inter;
    const float2 gu = *reinterpret_cast<const float2*>(Y + t * ldy + 2 * j);
    store_split(hi, lo, e, dsilu(gu.x) * gu.y);
}

// Row argmax, ties to the lowest index (gemvW4A16ArgmaxNeon, xq_gemv_w4a16_neon.cpp:315-318): one
// block of 1024 threads per row. A NaN never wins (as with the reference's `>` comparisons).
__global__ void __launch_bounds__(1024) row_argmax_kernel(const float* logits, int n, int* idx) {
    pdl_launch_dependents();  // launched with programmatic dependent launch: inputs only after
    pdl_wait();               // the previous kernel has finished
    __shared__ float sv[32];
    __shared__ int si[32];
    const float* x = logits + static_cast<size_t>(blockIdx.x) * n;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    // eight loads in flight per thread, then compared in increasing k: a later equal value never
    // replaces an earlier one
    constexpr int kU = 8;
    const int stride = blockDim.x;
    for (int k0 = threadIdx.x; k0 < n; k0 += kU * stride) {
        float v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) v[u] = k0 + u * stride < n ? x[k0 + u * stride] : -INFINITY;
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (v[u] > bv) {
                bv = v[u];
                bi = k0 + u * stride;
            }
    }
#pragma unroll
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
        idx[blockIdx.x] = (bi >= 0 && bi < n) ? bi : 0;
    }
}

}  // namespace

cudaError_t batch_argmax(const float* logits, int rows, int n, int* idx, cudaStream_t s) {
    pdl_launch(row_argmax_kernel, dim3(rows), dim3(1024), 0, s, logits, n, idx);
    return cudaGetLastError();
}

cudaError_t prefill_embed(const int* ids, const uint16_t* emb, float* H, int n, int hidden, int vocab, cudaStream_t s) {
    pdl_launch(embed_rows_kernel, dim3(n), dim3(256), 0, s, ids, emb, H, hidden, vocab);
    return cudaGetLastError();
}

cudaError_t prefill_rmsnorm_split(const float* H, const float* w, int n, int width, float eps, __nv_bfloat16* hi,
                                  __nv_bfloat16* lo, cudaStream_t s) {
    const bool vec = width % 4 == 0 && width <= 8 * 1024 && (reinterpret_cast<uintptr_t>(H) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && (reinterpret_cast<uintptr_t>(hi) & 7u) == 0 &&
                     (reinterpret_cast<uintptr_t>(lo) & 7u) == 0;
    if (vec)
        pdl_launch(rmsnorm_split_vec_kernel, dim3(n), dim3(256), 0, s, H, w, width, eps, hi, lo);
    else
        pdl_launch(rmsnorm_split_kernel, dim3(n), dim3(256), 0, s, H, w, width, eps, hi, lo);
    return cudaGetLastError();
}

cudaError_t prefill_conv(const float* Y, int ldy, const float* w, float* state, float* out, int n, int channels,
                         cudaStream_t s, int nseq, size_t state_bstride) {
    pdl_launch(conv_seq_kernel, dim3(dim3((channels + 127) / 128, nseq)), dim3(128), 0, s, Y, ldy, w, state, out, n, channels,
                                                                      state_bstride);
    return cudaGetLastError();
}

cudaError_t prefill_delta(const float* conv, int conv_ld, const float* Y, int ldy, int ab_off, const float* a_log,
                          const float* dt_bias, float* state, float* out, int out_ld, int n, int nk, int nv, int dk,
                          int dv, cudaStream_t s, int nseq, size_t state_bstride) {
    if (dk != 128 || dv % kDeltaCols != 0) return cudaErrorInvalidValue;
    pdl_launch(delta_seq_kernel, dim3(dim3(nv, dv / kDeltaCols, nseq)), dim3(128), 0, s, conv, conv_ld, Y, ldy, ab_off, a_log, dt_bias,
                                                                      state, out, out_ld, n, nk, nv, dk, dv,
                                                                      state_bstride);
    return cudaGetLastError();
}

cudaError_t prefill_gated_norm(const float* O, int o_ld, const float* Y, int ldy, int z_off, const float* w, int heads,
                               int hd, float eps, int n, __nv_bfloat16* hi, __nv_bfloat16* lo, cudaStream_t s) {
    const int warps = n * heads;
    pdl_launch(gated_norm_split_kernel, dim3((warps + 7) / 8), dim3(256), 0, s, O, o_ld, Y, ldy, z_off, w, heads, hd, eps, n, hi, lo);
    return cudaGetLastError();
}

cudaError_t prefill_attn_prep(const float* Y, int ldy, const float* q_norm, const float* k_norm, const float2* rope,
                              int rope_stride, float* Q, void* kc, void* vc, bool kv_fp16, int p0, int n, int nq,
                              int nkv, int hd, float eps, cudaStream_t s, const int* pos_arr, size_t kv_bstride) {
    if (hd != 256) return cudaErrorInvalidValue;
    const int warps = n * (nq + nkv);
    if (kv_fp16)
        pdl_launch(attn_prep_kernel<__half>, dim3((warps + 7) / 8), dim3(256), 0, s, Y, ldy, q_norm, k_norm, rope, rope_stride, Q,
                                                                static_cast<__half*>(kc), static_cast<__half*>(vc), p0,
                                                                n, nq, nkv, hd, eps, pos_arr, kv_bstride);
    else
        pdl_launch(attn_prep_kernel<float>, dim3((warps + 7) / 8), dim3(256), 0, s, Y, ldy, q_norm, k_norm, rope, rope_stride, Q,
                                                               static_cast<float*>(kc), static_cast<float*>(vc), p0, n,
                                                               nq, nkv, hd, eps, pos_arr, kv_bstride);
    return cudaGetLastError();
}

size_t prefill_attn_smem(int nq, int nkv, int hd, int max_len) {
    const int group = nq / nkv;
    return sizeof(float) * (static_cast<size_t>(group) * hd + static_cast<size_t>(group) * max_len);
}

cudaError_t prefill_attn(const float* Q, const float* Y, int ldy, const void* kc, const void* vc, bool kv_fp16, int p0,
                         int n, int nq, int nkv, int hd, __nv_bfloat16* hi, __nv_bfloat16* lo, cudaStream_t s,
                         const int* pos_arr, size_t kv_bstride, int max_len) {
    if (hd != 256 || nq % nkv != 0 || nq / nkv > kAttnMaxGroup) return cudaErrorInvalidValue;
    const size_t smem = prefill_attn_smem(nq, nkv, hd, pos_arr ? max_len : p0 + n);
    if (smem > kPrefillAttnMaxSmem) return cudaErrorInvalidValue;
    cudaError_t e;
    if (kv_fp16) {
        e = cudaFuncSetAttribute(attn_causal_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kPrefillAttnMaxSmem);
        if (e != cudaSuccess) return e;
        pdl_launch(attn_causal_kernel<__half>, dim3(dim3(n, nkv)), dim3(256), smem, s, Q, Y, ldy, static_cast<const __half*>(kc),
                                                                   static_cast<const __half*>(vc), p0, nq, nkv, hd, hi,
                                                                   lo, pos_arr, kv_bstride);
    } else {
        e = cudaFuncSetAttribute(attn_causal_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kPrefillAttnMaxSmem);
        if (e != cudaSuccess) return e;
        pdl_launch(attn_causal_kernel<float>, dim3(dim3(n, nkv)), dim3(256), smem, s, Q, Y, ldy, static_cast<const float*>(kc),
                                                                  static_cast<const float*>(vc), p0, nq, nkv, hd, hi,
                                                                  lo, pos_arr, kv_bstride);
    }
    return cudaGetLastError();
}

cudaError_t prefill_swiglu(const float* Y, int ldy, int inter, int n, __nv_bfloat16* hi, __nv_bfloat16* lo,
                           cudaStream_t s) {
    const size_t total = static_cast<size_t>(n) * inter;
    pdl_launch(swiglu_split_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, s, Y, ldy, inter, n, hi, lo);
    return cudaGetLastError();
}

}  // namespace xqb
