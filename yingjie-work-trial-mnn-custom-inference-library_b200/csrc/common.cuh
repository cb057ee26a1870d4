// Shared device helpers for the sm_100a kernels: error reporting, bulk async copies with
// mbarrier completion, programmatic dependent launch, warp reductions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace xqb {

// ------------------------------------------------------------------------------------
// Host-side error handling
// ------------------------------------------------------------------------------------
void set_last_error(const std::string& msg);
const char* last_error();

#define XQB_CUDA_OK(expr)                                                                        \
    do {                                                                                         \
        cudaError_t _e = (expr);                                                                 \
        if (_e != cudaSuccess) {                                                                 \
            ::xqb::set_last_error(std::string(#expr) + ": " + cudaGetErrorString(_e));           \
            return false;                                                                        \
        }                                                                                        \
    } while (0)

// Device-side error word bits (written with atomicOr, read by the host after a step).
enum DeviceError : unsigned {
    kErrBarrierTimeout = 1u,  // an mbarrier wait ran out of its iteration budget
    kErrBadShape = 2u,        // a kernel saw a configuration it does not support
    kErrAttnIndex = 4u,       // an attention item failed its bounds check (item skipped)
};

// Every spin-wait in these kernels is bounded in time: after its limit (kWaitLimitNs unless the
// launch passes another one) it records kErrBarrierTimeout in the error word and gives up, and
// every later wait in any block returns at once when it sees that bit, so a kernel that cannot
// make progress ends within seconds instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kSpinLimit = 1u << 30;         // poll cap on top of the time limit
#ifndef XQB_WAIT_SLEEP_NS
#define XQB_WAIT_SLEEP_NS 0
#endif
constexpr uint32_t kWaitSleepHintNs = XQB_WAIT_SLEEP_NS;  // longest sleep of one mbarrier poll (0: spin)

// ------------------------------------------------------------------------------------
// PTX wrappers
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue
// (launch_dependents), and wait until the previous kernel's results are visible (wait).
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// 1-D bulk copy global -> shared, completion counted on `bar`. dst, src 16-byte aligned,
// bytes a multiple of 16 (callers guarantee this by construction of the row layout).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// L2 policy for data read exactly once per step (the weight stream): its lines are the
// first to be evicted, so the small working set (activations, states, norm and conv
// weights, the step's phase list, code) stays resident in L2 across the step.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// bulk_g2s with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: a waiting thread may sleep up to `hint_ns` instead of
// spinning (it is woken when the phase completes), so waiting warps stop taking issue slots
// from the warps that do work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Slow path of every bounded wait: true while the caller may keep waiting.
__device__ __forceinline__ bool wait_budget_left(uint64_t t0, uint32_t i, unsigned* err,
                                                 uint64_t limit_ns = kWaitLimitNs) {
    if ((i & 255u) != 0u) return i < kSpinLimit;
    if (err && (*reinterpret_cast<volatile unsigned*>(err) & kErrBarrierTimeout)) return false;
    if (global_ns() - t0 > limit_ns || i >= kSpinLimit) {
        if (err) atomicOr(err, kErrBarrierTimeout);
        return false;
    }
    return true;
}

// Bounded mbarrier wait; false (and the error bit set) if it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (kWaitSleepHintNs ? mbar_try_wait_sleep(bar, parity, kWaitSleepHintNs) : mbar_try_wait(bar, parity))
            return true;
        if (!wait_budget_left(t0, i, err, limit_ns)) return false;
    }
}

// Wait for copies this block issued before it exits (after an error as well): bounded by
// its own deadline, independent of the error bit.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > kWaitLimitNs) return;
}

// d += A B on the integer tensor cores: mma.sync m16n8k32, A unsigned 8-bit (row-major
// fragment a0..a3), B signed 8-bit (column-major fragment b0, b1), exact s32 accumulation. Not
// volatile: the compiler may interleave independent accumulator chains.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint4 ld_shared_v4(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

// ------------------------------------------------------------------------------------
// Reductions
// ------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Scalar activations with the reference's formulas (custom_model.cpp:271-292).
__device__ __forceinline__ float dsilu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float dsigmoid(float x) {
    if (x >= 0.0f) {
        const float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    const float z = expf(x);
    return z / (1.0f + z);
}
__device__ __forceinline__ float dsoftplus(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return expf(x);
    return log1pf(expf(x));
}

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

}  // namespace xqb
