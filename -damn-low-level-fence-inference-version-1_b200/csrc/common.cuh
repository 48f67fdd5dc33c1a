// common.cuh — device helpers shared by every kernel of the engine (sm_100a only).
//
//  * bounded mbarrier waits: every spin on an mbarrier gives up after a fixed number of
//    try_wait rounds, records FENCE_E_DEVICE_WAIT in the device error word and lets the kernel
//    return instead of hanging the GPU;
//  * 1-D bulk copies global -> shared (cp.async.bulk, TMA engine) completing on an mbarrier,
//    without cluster multicast;
//  * programmatic-dependent-launch controls (griddepcontrol.*);
//  * Ampere-style 16-byte async copies (cp.async) for swizzled staging.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#ifndef FENCE_WAIT_ROUNDS
// try_wait suspends the thread for a hardware-defined interval per round; 2^24 rounds is
// seconds of waiting, far beyond any legitimate copy latency.
#define FENCE_WAIT_ROUNDS (1u << 24)
#endif

namespace fence {

// Device error word: 0 = ok; kernels store a FENCE_E_* code when they give up on a wait.
// Every kernel of the library is compiled in one translation unit, so this is its only definition.
__device__ int g_device_error = 0;

__device__ __forceinline__ void set_device_error(int code) { atomicExch(&g_device_error, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}
// Arrive and add `bytes` to the transaction count the phase waits for.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], "
        "%1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity. Returns false (and sets the device error
// word) when the bound is exhausted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < FENCE_WAIT_ROUNDS; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    set_device_error(-5 /* FENCE_E_DEVICE_WAIT */);
    return false;
}

// ---------------------------------------------------------------- bulk copy (TMA, 1-D)
// dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- cp.async (16 B)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// waits until at most N of this thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---------------------------------------------------------------- programmatic dependent launch
// Wait until the preceding kernel in the stream has completed and its writes are visible.
// A no-op when the kernel was not launched with programmatic stream serialization.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to begin launching.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- misc math
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
// ---------------------------------------------------------------- shared-memory loads by 32-bit
// shared-window address (keeps them LDS instructions; volatile so they stay behind the mbarrier
// wait that made the data visible)
__device__ __forceinline__ uint32_t lds32(uint32_t sa) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(sa));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t sa) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(sa));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t sa) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(sa));
    return v;
}
// 32-bit word at a 2-byte aligned shared address: two aligned loads and a funnel shift.
__device__ __forceinline__ uint32_t lds_u32_a2(uint32_t sa) {
    const uint32_t w = sa & ~3u;
    return __funnelshift_r(lds32(w), lds32(w + 4), (sa & 2u) * 8u);
}
// Four consecutive words starting at a 2-byte aligned shared address (reads 20 bytes).
__device__ __forceinline__ void lds_16B_a2(uint32_t sa, uint32_t out[4]) {
    const uint32_t w = sa & ~3u;
    const uint32_t sh = (sa & 2u) * 8u;
    const uint32_t w0 = lds32(w), w1 = lds32(w + 4), w2 = lds32(w + 8), w3 = lds32(w + 12), w4 = lds32(w + 16);
    out[0] = __funnelshift_r(w0, w1, sh);
    out[1] = __funnelshift_r(w1, w2, sh);
    out[2] = __funnelshift_r(w2, w3, sh);
    out[3] = __funnelshift_r(w3, w4, sh);
}

__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xffffu)));
}

}  // namespace fence
