// common.cuh -- device helpers shared by the momij MoE kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "momij_moe.h"

namespace momij {

constexpr int kWarp = 32;
constexpr int kChunk = 256;          // codes of one row a warp handles per tile (64 B)
constexpr int kDigitGroup = 64;      // x elements sharing one digit exponent
constexpr int kDgStride = 200;       // bytes per digit group: three 64-B int8 planes + 8 B pad (bank spread)
constexpr int kMaxTmax = 8;          // max pairs (token columns) per unit
constexpr int kPlanHeader = 8;       // [0]=units, [1]=status, then the fused kernels' control words (decode.cuh)

// ---- 16-bit float formats --------------------------------------------------
template <int DT>
struct Half;
template <>
struct Half<MOMIJ_DTYPE_BF16> {
    static __device__ __forceinline__ float to_f(uint16_t h) {
        return __uint_as_float(static_cast<uint32_t>(h) << 16);
    }
    static __device__ __forceinline__ uint16_t from_f(float f) {
        // round to nearest even; NaN kept quiet
        uint32_t u = __float_as_uint(f);
        if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
        u += 0x7fffu + ((u >> 16) & 1u);
        return static_cast<uint16_t>(u >> 16);
    }
};
template <>
struct Half<MOMIJ_DTYPE_F16> {
    static __device__ __forceinline__ float to_f(uint16_t h) {
        float f;
        asm("{ cvt.f32.f16 %0, %1; }" : "=f"(f) : "h"(h));
        return f;
    }
    static __device__ __forceinline__ uint16_t from_f(float f) {
        uint16_t h;
        asm("{ cvt.rn.f16.f32 %0, %1; }" : "=h"(h) : "f"(f));
        return h;
    }
};

// Clamped SwiGLU with the reference's rounding staging: the up and gate
// gather outputs are activation-dtype values first (MLX gather_qmm outputs,
// MapleMoE.swift:65-70), the SwiGLU runs in fp32 on them and is rounded once
// (maple_clamped_swiglu, SeedlessMetal.swift:2435-2450).
template <int DT>
__device__ __forceinline__ uint16_t swiglu_staged(float up, float gate, float clamp) {
    float u = Half<DT>::to_f(Half<DT>::from_f(up));
    float g = Half<DT>::to_f(Half<DT>::from_f(gate));
    g = fminf(g, clamp);
    u = fminf(fmaxf(u, -clamp), clamp);
    return Half<DT>::from_f(g / (1.f + expf(-g)) * u);
}

// ---- tensor core: D(16x8 s32) += A(16x32 u8, row) * B(32x8 s8, col) --------
// Fragment ownership (lane = 4*g + t): a0 (row g, k 4t..4t+3), a1 (row g+8,
// same k), a2 (row g, k 16+4t..), a3 (row g+8, k 16+4t..); b0 (k 4t.., col g),
// b1 (k 16+4t.., col g); d0,d1 (row g, cols 2t, 2t+1), d2,d3 (row g+8, ...).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- asynchronous global->shared copies ------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    int n = valid ? 16 : 0;  // n == 0 zero-fills the destination, reads nothing
    asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(n));
}
// The same copies with an L2 eviction-priority policy (createpolicy).
__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void* src, bool valid,
                                                uint64_t policy) {
    int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(dst),
                 "l"(src), "r"(n), "l"(policy));
}
__device__ __forceinline__ void cp_async8_hint(uint32_t dst, const void* src, bool valid,
                                               uint64_t policy) {
    int n = valid ? 8 : 0;
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, %2, %3;\n" ::"r"(dst),
                 "l"(src), "r"(n), "l"(policy));
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, bool valid) {
    int n = valid ? 8 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool valid) {
    int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ---- mbarriers and TMA bulk copies (each into this CTA only) ----------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Arrives on `bar` once every cp.async this thread issued so far has landed
// (the barrier's expected count includes this arrival).
__device__ __forceinline__ void mbar_arrive_cp_async(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking test of the same condition (no hardware suspend: cheaper to
// poll when the phase has usually completed already).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
    return p;
}
// Global -> shared bulk copy completing on `bar` (16-B aligned, 16-B multiple).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;\n" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// Named barrier over `count` threads (a subset of the block).
__device__ __forceinline__ void bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// ---- programmatic dependent launch -----------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::);
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier over gridDim.x co-resident CTAs by one thread (after a
// block barrier of the CTA's threads whose writes it publishes): an arrival
// counter that the last arriver resets, and a generation word it then
// increments with release semantics; the others wait for the generation to
// differ from g0, its value read when the kernel started (it cannot change
// before this CTA arrives).  The counter never exceeds the grid size and the
// generation is compared for change only, so neither wraps into a wrong
// state.  Every CTA arrives even when it later gives up waiting, so the
// counter is back at zero after every call.
__device__ inline bool grid_barrier_thread(unsigned* arrive, unsigned* gen, unsigned g0, int limit, bool wait) {
    __threadfence();  // the CTA's writes (ordered before this thread by the block barrier)
    const unsigned old = atomicAdd(arrive, 1u);
    if (old == gridDim.x - 1) {
        *reinterpret_cast<volatile unsigned*>(arrive) = 0u;  // no other CTA touches it before the generation moves
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(gen) : "memory");
        return true;
    }
    if (!wait) return false;
    for (int it = 0; it < limit; ++it) {
        if (ld_acquire_u32(gen) != g0) return true;
        __nanosleep(32);
    }
    return ld_acquire_u32(gen) != g0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace momij
