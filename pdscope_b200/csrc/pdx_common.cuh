// Shared device helpers for the pdx_moe kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pdx_moe.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "pdx_moe targets sm_100a (B200) only"
#endif

namespace pdx {

typedef __nv_bfloat16 bf16;

// Device error word: first nonzero PDX_DEVERR_* code raised by any kernel of
// this library on this device.  Read and cleared by pdx_device_error().
// (The library is one translation unit, so this is its only definition.)
__device__ unsigned int g_device_error = 0;

__device__ __forceinline__ void raise_error(unsigned int code) {
    atomicCAS(&g_device_error, 0u, code);
}

__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float bits2f(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t f2bits(float v) {  // RNE
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float round_bf16(float v) { return bits2f(f2bits(v)); }

// float64 -> BF16 with one round-to-nearest-even step at BF16's 8-bit
// significand (IEEE-754 definition; no intermediate float32 rounding).
__device__ __forceinline__ uint16_t f64_to_bf16_bits(double x) {
    const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(x));
    const uint32_t sign = static_cast<uint32_t>(b >> 63) << 15;
    const int exp = static_cast<int>((b >> 52) & 0x7FF);
    const unsigned long long mant = b & 0xFFFFFFFFFFFFFull;
    if (exp == 0x7FF) return static_cast<uint16_t>(sign | (mant ? 0x7FC0u : 0x7F80u));
    if (exp == 0) return static_cast<uint16_t>(sign);  // |x| < 2^-1022: rounds to zero
    const int e = exp - 1023;
    if (e >= -126) {
        unsigned long long m7 = mant >> 45;
        const unsigned long long rem = mant & ((1ull << 45) - 1);
        const unsigned long long half = 1ull << 44;
        if (rem > half || (rem == half && (m7 & 1ull))) ++m7;
        int be = e + 127;
        if (m7 == 128) { m7 = 0; ++be; }
        if (be >= 255) return static_cast<uint16_t>(sign | 0x7F80u);
        return static_cast<uint16_t>(sign | (static_cast<uint32_t>(be) << 7) | static_cast<uint32_t>(m7));
    }
    // BF16 subnormal: value / 2^-133 = (2^52 + mant) / 2^(52 - 133 - e)
    const int shift = -81 - e;  // >= 46
    if (shift > 62) return static_cast<uint16_t>(sign);
    const unsigned long long full = (1ull << 52) | mant;
    unsigned long long m = full >> shift;
    const unsigned long long rem = full & ((1ull << shift) - 1);
    const unsigned long long half = 1ull << (shift - 1);
    if (rem > half || (rem == half && (m & 1ull))) ++m;
    return static_cast<uint16_t>(sign | static_cast<uint32_t>(m));
}

// ---------------------------------------------------------------------------
// Bounded mbarrier / TMA / tcgen05 helpers.  Every wait gives up after
// kWaitLimitNs of wall time (globaltimer), raises PDX_DEVERR_WAIT_TIMEOUT and
// reports failure so the caller can unwind instead of hanging the GPU.
// ---------------------------------------------------------------------------
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  `abort_flag` (shared
// memory) lets one timed-out role release every other waiter of the CTA.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const unsigned long long start = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(addr, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - start > kWaitLimitNs) {
                *abort_flag = 1;
                raise_error(PDX_DEVERR_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 2-D tiled TMA load of one box into this CTA's shared memory: (x = inner, y = outer).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x,
                                            int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start before its predecessor in the stream finishes;
// griddep_wait() blocks until the predecessor has completed and its memory is
// visible (every kernel of the chain calls it, so the guarantee is
// transitive).  griddep_launch() lets the next kernel of the chain start its
// prologue early.  Both are no-ops for a normal launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

}  // namespace pdx
