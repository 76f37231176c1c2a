// common.cuh -- shared device helpers for the sm_100a paged-KV kernels:
// element decoding, mbarrier / TMA / cp.async wrappers, bounded waits and the
// per-device status word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "gollek_kernels.h"

namespace gk {

// Sticky per-device status word (GOLLEK_STATUS_* bits).  Kernels OR bits into it;
// the host reads and clears it with gollek_device_status().
__device__ unsigned int g_status;

__device__ __forceinline__ void raise_status(unsigned bits) { atomicOr(&g_status, bits); }

// Iterations of a try_wait loop before a wait gives up and reports
// GOLLEK_STATUS_TIMEOUT.  Each try_wait blocks for a hardware-defined slice, so
// this bounds a wait at well over a second: far beyond any real TMA latency.
constexpr unsigned kWaitLimit = 1u << 24;
// Polling rounds (each with a short sleep) before a poll loop gives up.
constexpr unsigned kPollLimit = 1u << 24;

// ----------------------------------------------------------------- elements

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Two floats -> one 32-bit register of the 16-bit MMA type (x0 in the low half).
template <typename KV>
__device__ __forceinline__ uint32_t pack2(float x0, float x1) {
    if constexpr (std::is_same<KV, __half>::value) {
        __half2 h = __floats2half2_rn(x0, x1);
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

template <typename KV>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
    if constexpr (std::is_same<KV, __half>::value)
        return __half22float2(*reinterpret_cast<__half2 *>(&w));
    else
        return make_float2(bf16_lo(w), bf16_hi(w));
}

// ----------------------------------------------------------------- mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase of `bar` with the given parity (at most `limit` try_waits).
// Returns false (and raises GOLLEK_STATUS_TIMEOUT) if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned limit = kWaitLimit) {
    for (unsigned i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    raise_status(GOLLEK_STATUS_TIMEOUT);
    return false;
}

// mbarrier test that may suspend the thread until the phase completes, for at most ns
// nanoseconds (the suspend-time hint of mbarrier.try_wait).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Tests allowed to a wait whose tests suspend for up to 20 us each (kSuspendNs): at most
// about 5 s if every test suspends the whole hint, and still well above any wait of a
// working kernel if tests return early.
constexpr uint32_t kSuspendNs = 20000;
constexpr unsigned kSuspendTries = kWaitLimit >> 6;

// Bounded wait of one thread that also gives up (returning false, raising nothing) once
// `abort` is set by a thread that gave up first.
// suspend_ns > 0: each test may suspend the thread until the phase completes, for up to
// that long (the waiting thread then leaves the SM's issue slots and shared-memory pipe to
// the warps that do the work; give a limit of tries to match, e.g. kSuspendTries).
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort,
                                                   unsigned limit = kWaitLimit, uint32_t suspend_ns = 0) {
    for (unsigned i = 0; i < limit; ++i) {
        if (*abort) return false;
        if (suspend_ns ? mbar_try_wait_suspend(bar, parity, suspend_ns) : mbar_try_wait(bar, parity)) return true;
    }
    raise_status(GOLLEK_STATUS_TIMEOUT);
    return false;
}

// The same for a whole warp (every lane calls it; the result is warp-uniform).
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, unsigned limit,
                                          volatile int *abort, uint32_t suspend_ns = 0) {
    for (unsigned i = 0; i < limit; ++i) {
        if (__any_sync(0xffffffffu, *abort != 0)) return false;
        if (__all_sync(0xffffffffu, suspend_ns ? mbar_try_wait_suspend(bar, parity, suspend_ns)
                                               : mbar_try_wait(bar, parity)))
            return true;
    }
    raise_status(GOLLEK_STATUS_TIMEOUT);
    return false;
}

// Non-blocking test of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Shared-memory loads/stores by 32-bit shared address.  volatile keeps them ordered
// after the mbarrier waits that publish the data they read.
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void sts_u4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Four 8x8 matrices of 16-bit elements; lane l gives the row address of row l%8 of
// matrix l/8.  .trans delivers them transposed.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t *r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t *r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// --------------------------------------------------------------- TMA / async

// 2-D tiled TMA load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled TMA load (coordinates innermost first), completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// 4-D tiled TMA load (coordinates innermost first), completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            int c3, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`; both addresses
// 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 4-byte cp.async (Ampere-style) global -> shared.
__device__ __forceinline__ void cp_async_4(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}

// Arrive on `bar` once this thread's earlier cp.async copies have landed; the
// arrival counts against the barrier's expected count.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// --------------------------------------------------------------------- math

// 2^x with the hardware's approximate exponent (ex2.approx, flush-to-zero).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Named barrier over `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Math.round(float): closest integer, ties toward +infinity; NaN -> 0.
// (double)x + 0.5 is exact for every float below 2^29, so floor gives the
// correctly rounded result.
__device__ __forceinline__ int java_round(float x) {
    if (x != x) return 0;
    double r = floor(static_cast<double>(x) + 0.5);
    r = fmin(fmax(r, -2147483648.0), 2147483647.0);
    return static_cast<int>(r);
}

}  // namespace gk
