// tcgen05.cuh -- thin wrappers over the sm_100a 5th-generation tensor-core instructions
// (tcgen05.mma with operands in shared memory and the accumulator in tensor memory),
// tensor-memory allocation and loads, and the fences that order them with threads.
#pragma once

#include "common.cuh"

namespace gk {

// Shared-memory matrix descriptor for a 128-byte-swizzled operand (the layout TMA's
// SWIZZLE_128B writes from a 1024-byte-aligned base): start address, leading and
// stride byte offsets (encoded >> 4), the sm_100 descriptor version (1) and the
// swizzle mode (2 = 128B).
//   K-major:  rows of 64 elements (128 bytes); 8-row core groups `sbo` bytes apart;
//             lbo unused (one MMA's K of 16 elements lies inside the 128-byte row).
//   MN-major: 64 MN-elements per 128-byte row, the next 64 at `lbo`; K rows 128 bytes
//             apart, 8-row K groups `sbo` bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor of kind::f16 with an fp32 accumulator: A and B both bf16
// (bf16 = 1) or both f16 (bf16 = 0); a_mn / b_mn select the MN-major operand layout.
__host__ __device__ constexpr uint32_t umma_idesc_16bit(int M, int N, int bf16, int a_mn, int b_mn) {
    return (1u << 4) | (static_cast<uint32_t>(bf16) << 7) | (static_cast<uint32_t>(bf16) << 10) |
           (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A * B, issued by one thread; acc = 0 overwrites D.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// Arrive once on `bar` when every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Tensor-memory allocation (whole warp): the base address is written to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// N consecutive fp32 columns of this thread's tensor-memory lane (shape 32x32b: lane
// i of the warp reads lane base + i).  Complete after tmem_wait_ld().
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float *v);
template <>
__device__ __forceinline__ void tmem_ld<1>(uint32_t taddr, float *v) {
    uint32_t r0;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r0) : "r"(taddr) : "memory");
    v[0] = __uint_as_float(r0);
}
template <>
__device__ __forceinline__ void tmem_ld<2>(uint32_t taddr, float *v) {
    uint32_t r0, r1;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(taddr)
                 : "memory");
    v[0] = __uint_as_float(r0);
    v[1] = __uint_as_float(r1);
}
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, float *v) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float *v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's tensor-memory lane (shape 32x32b), written;
// complete after tmem_wait_st().
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])),
        "r"(__float_as_uint(v[1])),
        "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])),
        "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])),
        "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])),
        "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])),
        "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])),
        "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])),
        "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])),
        "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])),
        "r"(__float_as_uint(v[25])),
        "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])),
        "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])),
        "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Named barrier that also ORs a predicate over its `count` threads.
__device__ __forceinline__ bool bar_red_or(int id, int count, bool pred) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
        : "memory");
    return out != 0;
}

}  // namespace gk
