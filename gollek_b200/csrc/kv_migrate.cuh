// kv_migrate.cuh -- block-remapped KV copy (prefill -> decode migration, also the
// copy-on-write block copy) and per-block checksums for verifying a copy in place.
//
// Work is cut into 64 KiB segments of (block, K|V) so that a few long requests
// still spread over every SM.  A thread moves 4 x 16 bytes per step: four
// independent loads from local HBM in flight, then four 16-byte stores, which go
// over NVLink when the destination is a peer's memory.  Plain loads and stores only.
// Block ids outside a pool's [0, num_blocks) (when the caller gives num_blocks) are
// skipped and raise GOLLEK_STATUS_BAD_BLOCK_ID, so a stale or sentinel id never turns
// into a store outside the destination pool, a peer's included.
#pragma once

#include "common.cuh"

namespace gk {

constexpr long long kSegBytes = 64 * 1024;

struct MigrateArgs {
    const uint8_t *src[2];
    uint8_t *dst[2];
    const int *src_blocks;
    const int *dst_blocks;
    long long src_stride, dst_stride, bytes;
    long long segs_per_block;
    long long num_units;  // num_copies * tensors * segs_per_block
    int tensors;
    int src_num_blocks, dst_num_blocks;  // 0: unchecked
};

// True when both ids of copy i lie inside their pools (every thread of the CTA reads
// the same ids, so the test is uniform across the CTA).
__device__ __forceinline__ bool migrate_ids_ok(const MigrateArgs &a, long long i, int &s, int &d) {
    s = a.src_blocks[i];
    d = a.dst_blocks[i];
    const bool ok = s >= 0 && d >= 0 && (a.src_num_blocks <= 0 || s < a.src_num_blocks) &&
                    (a.dst_num_blocks <= 0 || d < a.dst_num_blocks);
    if (!ok && threadIdx.x == 0) raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
    return ok;
}

__global__ void __launch_bounds__(512) kv_migrate_kernel_v16(const MigrateArgs a) {
    for (long long u = blockIdx.x; u < a.num_units; u += gridDim.x) {
        const long long seg = u % a.segs_per_block;
        const long long bt = u / a.segs_per_block;
        const int tensor = static_cast<int>(bt % a.tensors);
        const long long i = bt / a.tensors;
        int sb, db;
        if (!migrate_ids_ok(a, i, sb, db)) continue;
        const uint4 *src = reinterpret_cast<const uint4 *>(
            a.src[tensor] + static_cast<long long>(sb) * a.src_stride + seg * kSegBytes);
        uint4 *dst = reinterpret_cast<uint4 *>(
            a.dst[tensor] + static_cast<long long>(db) * a.dst_stride + seg * kSegBytes);
        const long long rem = a.bytes - seg * kSegBytes;
        const int n16 = static_cast<int>((rem < kSegBytes ? rem : kSegBytes) >> 4);
        int k = threadIdx.x;
        for (; k + 3 * 512 < n16; k += 4 * 512) {
            const uint4 x0 = __ldcs(src + k);
            const uint4 x1 = __ldcs(src + k + 512);
            const uint4 x2 = __ldcs(src + k + 1024);
            const uint4 x3 = __ldcs(src + k + 1536);
            __stcs(dst + k, x0);
            __stcs(dst + k + 512, x1);
            __stcs(dst + k + 1024, x2);
            __stcs(dst + k + 1536, x3);
        }
        for (; k < n16; k += 512) __stcs(dst + k, __ldcs(src + k));
    }
}

// Byte-granular fallback for unaligned pools or sizes.
__global__ void __launch_bounds__(256) kv_migrate_kernel_bytes(const MigrateArgs a) {
    for (long long u = blockIdx.x; u < a.num_units; u += gridDim.x) {
        const long long seg = u % a.segs_per_block;
        const long long bt = u / a.segs_per_block;
        const int tensor = static_cast<int>(bt % a.tensors);
        const long long i = bt / a.tensors;
        int sb, db;
        if (!migrate_ids_ok(a, i, sb, db)) continue;
        const uint8_t *src = a.src[tensor] + static_cast<long long>(sb) * a.src_stride + seg * kSegBytes;
        uint8_t *dst = a.dst[tensor] + static_cast<long long>(db) * a.dst_stride + seg * kSegBytes;
        const long long rem = a.bytes - seg * kSegBytes;
        const long long n = rem < kSegBytes ? rem : kSegBytes;
        for (long long k = threadIdx.x; k < n; k += blockDim.x) dst[k] = src[k];
    }
}

// One CTA per block: sum over 8-byte words w_j of (w_j ^ (j * golden)) mod 2^64.  An id
// outside [0, num_blocks) (num_blocks > 0) reads nothing, gets checksum 0 and raises
// GOLLEK_STATUS_BAD_BLOCK_ID.
__global__ void __launch_bounds__(256) block_checksum_kernel(const uint8_t *pool, const int *blocks,
                                                             int num_blocks, long long stride,
                                                             long long bytes, unsigned long long *out) {
    __shared__ unsigned long long part[8];
    const int b = blocks[blockIdx.x];
    if (b < 0 || (num_blocks > 0 && b >= num_blocks)) {
        if (threadIdx.x == 0) {
            raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
            out[blockIdx.x] = 0;
        }
        return;
    }
    const uint64_t *w = reinterpret_cast<const uint64_t *>(pool + static_cast<long long>(b) * stride);
    const long long n = bytes >> 3;
    unsigned long long acc = 0;
    for (long long j = threadIdx.x; j < n; j += blockDim.x)
        acc += w[j] ^ (static_cast<unsigned long long>(j) * 0x9E3779B97F4A7C15ull);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long t = 0;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += part[i];
        out[blockIdx.x] = t;
    }
}

}  // namespace gk
