// Persistent decode-step kernel (see stepper.cuh).
#include <cuda_fp16.h>

#include <algorithm>

#include "gemv.hpp"
#include "ops_device.cuh"
#include "stepper.cuh"

namespace xqb {

namespace {

// Shared-memory layout (bytes):
//   [0, 128)     full mbarriers      [128, 256)   empty mbarriers
//   [256, 384)   warp sums           [512, 4608)  double-buffered row sums [2][16][32]
//   [4608, 6912) attention scratch   [6912, 8192) 3 DeltaNet scratches
//   [8192, 8704) argmax scratch      then kStepAttnDynBytes, then the weight ring.
constexpr int kOffFull = 0, kOffEmpty = 128, kOffWsum = 256, kOffRed = 512, kOffAttn = 4608, kOffDelta = 6912,
              kOffArg = 8192;
static_assert(sizeof(AttnScratch) <= kOffDelta - kOffAttn, "attention scratch");
static_assert(3 * sizeof(DeltaScratch) <= kOffArg - kOffDelta, "delta scratch");

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
    float* wsum;
    float* red;
    uint8_t* ring;
    int nslots;
    int tid, lane, warp;
    int gbase;  // chunks this block consumed in earlier phases
};

__device__ __forceinline__ void block_rows(const GemvParams& p, int* r_begin, int* r_end, int* nchunks) {
    const int units = p.rows / p.unit;
    *r_begin = static_cast<int>((long long)units * blockIdx.x / gridDim.x) * p.unit;
    *r_end = static_cast<int>((long long)units * (blockIdx.x + 1) / gridDim.x) * p.unit;
    *nchunks = (*r_end - *r_begin + p.rows_per_chunk - 1) / p.rows_per_chunk;
}

template <int META, int PRO, int EPI>
__device__ __forceinline__ void gemv_phase(const GemvParams& p, Ctx& c) {
    int r_begin, r_end, nchunks;
    block_rows(p, &r_begin, &r_end, &nchunks);
    const int R = p.rows_per_chunk;
    const int team_size = p.cols >> 5;
    const int teams = kStepConsumers / team_size;
    const int tid = c.tid, lane = c.lane, warp = c.warp;
    float best_v = -INFINITY;
    int best_i = (tid == 0) ? r_begin : 0x7fffffff;
    if (tid < teams * team_size) {
        const int team = tid / team_size;
        const int t = tid - team * team_size;
        const int wpt = team_size >> 5;
        const int team_bar = 2 + team;
        XLimbs L;
        {
            float xv[32];
            gemv_load_x<PRO>(p, t, lane, warp, team, wpt, team_bar, team_size, c.wsum, xv);
            gemv_make_limbs<META>(xv, L);
        }
        int it = 0;
        for (int ci = team; ci < nchunks; ci += teams, ++it) {
            const int g = c.gbase + ci;
            const int s = g % c.nslots;
            const int row0 = r_begin + ci * R;
            const int nr = min(R, r_end - row0);
            mbar_wait_bounded(&c.full[s], static_cast<uint32_t>((g / c.nslots) & 1), p.err);
            float part[kMaxRowsPerTeam];
            gemv_chunk_partials<META, kMaxRowsPerTeam>(c.ring + static_cast<size_t>(s) * kStepSlotBytes,
                                                       p.row_stride, p.meta_offset, t, nr, L, part);
            const float v = reduce_rows<kMaxRowsPerTeam>(part, lane);
            float* rbuf = c.red + (it & 1) * (kMaxRowsPerChunk * 32);
            if ((lane & (32 / kMaxRowsPerTeam - 1)) == 0) {
                const int j = lane / (32 / kMaxRowsPerTeam);
                if (j < nr) rbuf[j * 32 + warp] = v;
            }
            named_bar(team_bar, team_size);
            if (t == 0) mbar_arrive(&c.empty[s]);
            const int w0 = team * wpt;
            if constexpr (EPI == kEpiSwiglu) {
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
                    if constexpr (EPI == kEpiArgmax)
                        argmax_merge(best_v, best_i, y, row0 + t);
                    else
                        gemv_epilogue_row<EPI>(p, row0 + t, y);
                }
            }
        }
    }
    c.gbase += nchunks;
    if constexpr (EPI == kEpiArgmax) {
        // Block result, then the last block merges all blocks, samples the token and loads its
        // embedding row (gemvW4A16ArgmaxNeon :309-336, loadEmbeddingRow custom_model.cpp:569-608).
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
}

template <int META>
__device__ __forceinline__ void gemv_dispatch(const PhaseDesc& D, Ctx& c) {
    const int pro = D.pro, epi = D.epi;
    if (pro == kProRms && epi == kEpiConv)
        gemv_phase<META, kProRms, kEpiConv>(D.g, c);
    else if (pro == kProGatedRms && epi == kEpiResidual)
        gemv_phase<META, kProGatedRms, kEpiResidual>(D.g, c);
    else if (pro == kProRms && epi == kEpiSwiglu)
        gemv_phase<META, kProRms, kEpiSwiglu>(D.g, c);
    else if (pro == kProPlain && epi == kEpiResidual)
        gemv_phase<META, kProPlain, kEpiResidual>(D.g, c);
    else if (pro == kProRms && epi == kEpiStore)
        gemv_phase<META, kProRms, kEpiStore>(D.g, c);
    else if (pro == kProRms && epi == kEpiArgmax)
        gemv_phase<META, kProRms, kEpiArgmax>(D.g, c);
    else if (c.tid == 0)
        atomicOr(D.g.err, kErrBadShape);
}

template <int META, typename KV>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ctx c;
    c.base = smem;
    c.full = reinterpret_cast<uint64_t*>(smem + kOffFull);
    c.empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
    c.wsum = reinterpret_cast<float*>(smem + kOffWsum);
    c.red = reinterpret_cast<float*>(smem + kOffRed);
    float* attn_dyn = reinterpret_cast<float*>(smem + kStepHeaderBytes);
    c.ring = smem + kStepHeaderBytes + kStepAttnDynBytes;
    c.nslots = P.nslots;
    c.tid = threadIdx.x;
    c.lane = c.tid & 31;
    c.warp = c.tid >> 5;
    c.gbase = 0;
    if (c.tid == 0) {
        for (int s = 0; s < c.nslots; ++s) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (c.warp == kStepConsumers / 32) {
        // Producer: stream this block's rows of every GEMV phase, in phase order.
        if (c.lane == 0) {
            int g = 0;
            bool stop = false;
            for (int ph = 0; ph < P.nphases && !stop; ++ph) {
                const PhaseDesc& D = P.phases[ph];
                if (D.kind != kPhaseGemv) continue;
                int r_begin, r_end, nchunks;
                block_rows(D.g, &r_begin, &r_end, &nchunks);
                for (int ci = 0; ci < nchunks; ++ci) {
                    const int s = g % c.nslots;
                    if (g >= c.nslots &&
                        !mbar_wait_bounded(&c.empty[s], static_cast<uint32_t>(((g / c.nslots) - 1) & 1), P.err)) {
                        stop = true;
                        break;
                    }
                    const int row0 = r_begin + ci * D.g.rows_per_chunk;
                    const uint32_t bytes =
                        static_cast<uint32_t>(min(D.g.rows_per_chunk, r_end - row0) * D.g.row_stride);
                    mbar_expect_tx(&c.full[s], bytes);
                    bulk_g2s(c.ring + static_cast<size_t>(s) * kStepSlotBytes,
                             D.g.w + static_cast<size_t>(row0) * D.g.row_stride, bytes, &c.full[s]);
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
    const unsigned G = gridDim.x;
    for (int ph = 0; ph < P.nphases; ++ph) {
        const PhaseDesc& D = P.phases[ph];
        if (ph > 0) {  // every phase consumes the previous phase's output
            if (c.tid == 0) {
                const unsigned target = static_cast<unsigned>(ph) * G;
                if (ld_acquire(P.grid_bar) < target) {
                    const uint64_t t0 = global_ns();
                    for (uint32_t n = 1; ld_acquire(P.grid_bar) < target; ++n)
                        if (!wait_budget_left(t0, n, P.err)) break;
                }
            }
            named_bar(1, kStepConsumers);
        }
        if (P.trace && blockIdx.x == 0 && c.tid == 0) P.trace[3 * ph] = global_ns();
        if (D.kind == kPhaseGemv) {
            gemv_dispatch<META>(D, c);
        } else if (D.kind == kPhaseDelta) {
            const int nslice = D.d.dv / kDeltaCols;
            const int items = D.d.nv * nslice;
            const int dteam = c.tid >> 7;  // 3 teams of 128 threads
            for (int i = blockIdx.x + dteam * G; i < items; i += 3 * G)
                delta_item(D.d, i / nslice, i % nslice, c.tid & 127, 2 + dteam, dsh + dteam);
        } else if (D.kind == kPhaseAttn) {
            const int items = D.a.nkv * kAttnSplits;
            if (c.tid < kAttnThreads)
                for (int i = blockIdx.x; i < items; i += G)
                    attention_item<KV>(D.a, i / kAttnSplits, i % kAttnSplits, c.tid, 2, attn_dyn, ash);
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
            if (P.trace && blockIdx.x == 0) P.trace[3 * ph + 1] = global_ns();
            __threadfence();
            const unsigned old = atomicAdd(P.grid_bar, 1u);
            if (P.trace && old == static_cast<unsigned>(ph + 1) * G - 1) P.trace[3 * ph + 2] = global_ns();
            if (ph == P.nphases - 1 && old == static_cast<unsigned>(P.nphases) * G - 1)
                atomicExch(P.grid_bar, 0u);  // everybody has arrived; nobody waits any more
        }
    }
}

template <int META, typename KV>
cudaError_t launch_one(const StepParams& p, int num_sms, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = step_smem_bytes(p.nslots);
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
    return cudaFuncSetAttribute(decode_step_kernel<META, KV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(step_smem_bytes(step_max_slots())));
}

}  // namespace

size_t step_smem_bytes(int nslots) {
    return static_cast<size_t>(kStepHeaderBytes) + kStepAttnDynBytes + static_cast<size_t>(nslots) * kStepSlotBytes;
}

int step_max_slots() {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int avail = optin - kStepHeaderBytes - kStepAttnDynBytes - 1024;
    return std::max(2, std::min(kStepMaxSlots, avail / kStepSlotBytes));
}

cudaError_t step_init_device() {
    cudaError_t e;
    if ((e = set_attr<kMetaSym16, float>()) != cudaSuccess) return e;
    if ((e = set_attr<kMetaSym16, __half>()) != cudaSuccess) return e;
    if ((e = set_attr<kMetaAff32, float>()) != cudaSuccess) return e;
    return set_attr<kMetaAff32, __half>();
}

cudaError_t launch_decode_step(const StepParams& p, int meta_kind, bool kv_fp16, int num_sms, cudaStream_t s) {
    if (meta_kind == kMetaSym16)
        return kv_fp16 ? launch_one<kMetaSym16, __half>(p, num_sms, s) : launch_one<kMetaSym16, float>(p, num_sms, s);
    return kv_fp16 ? launch_one<kMetaAff32, __half>(p, num_sms, s) : launch_one<kMetaAff32, float>(p, num_sms, s);
}

}  // namespace xqb
