// kv_append.cuh -- scatter new key/value rows into their KV pages, with int8/int4
// quantisation that reproduces the reference's Java arithmetic bit for bit.
//
// One warp per (token, kv-head) row: the warp max gives the row's absmax (exact,
// order-free), the scale is absmax/127 (absmax/7) by IEEE division, each element is
// clamp(Math.round(x / scale)) with Java's ties-toward-+infinity rounding.
#pragma once

#include "common.cuh"

namespace gk {

struct AppendArgs {
    const void *key;
    const void *value;
    const int *token_seq;
    const int *token_pos;
    const int *block_tables;
    void *k;
    void *v;
    float *k_scales;
    float *v_scales;
    long long page_stride, scale_page_stride, scale_head_stride, scale_token_stride;
    int src_bf16, kv_dtype, num_tokens, num_kv_heads, head_dim, block_size, max_blocks, num_blocks;
};

__device__ __forceinline__ float load_src(const void *p, int bf16, long long i) {
    return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i])
                : reinterpret_cast<const float *>(p)[i];
}

// Writes one row (head_dim values) into the pool; the warp works together.
__device__ __forceinline__ void append_row(const AppendArgs &a, const void *src, long long src0,
                                           void *pool, float *scales, long long e0, long long so,
                                           int lane) {
    const int D = a.head_dim;
    switch (a.kv_dtype) {
        case GOLLEK_DTYPE_F32:
            for (int d = lane; d < D; d += 32)
                reinterpret_cast<float *>(pool)[e0 + d] = load_src(src, a.src_bf16, src0 + d);
            return;
        case GOLLEK_DTYPE_BF16:
            for (int d = lane; d < D; d += 32)
                reinterpret_cast<__nv_bfloat16 *>(pool)[e0 + d] =
                    __float2bfloat16_rn(load_src(src, a.src_bf16, src0 + d));
            return;
        case GOLLEK_DTYPE_F16:
            for (int d = lane; d < D; d += 32)
                reinterpret_cast<__half *>(pool)[e0 + d] =
                    __float2half_rn(load_src(src, a.src_bf16, src0 + d));
            return;
        default:
            break;
    }
    const bool i8 = a.kv_dtype == GOLLEK_DTYPE_I8;
    float absmax = 0.f;
    for (int d = lane; d < D; d += 32) absmax = fmaxf(absmax, fabsf(load_src(src, a.src_bf16, src0 + d)));
    absmax = warp_max(absmax);
    const float scale = absmax == 0.f ? 1.0f : __fdiv_rn(absmax, i8 ? 127.0f : 7.0f);
    if (lane == 0 && scales) scales[so] = scale;
    if (i8) {
        for (int d = lane; d < D; d += 32) {
            int q = java_round(__fdiv_rn(load_src(src, a.src_bf16, src0 + d), scale));
            q = max(-127, min(127, q));
            reinterpret_cast<int8_t *>(pool)[e0 + d] = static_cast<int8_t>(q);
        }
    } else {
        // Packed nibbles: lane writes whole bytes (element pairs); e0 and D are even.
        for (int d = 2 * lane; d < D; d += 64) {
            int q0 = java_round(__fdiv_rn(load_src(src, a.src_bf16, src0 + d), scale));
            int q1 = java_round(__fdiv_rn(load_src(src, a.src_bf16, src0 + d + 1), scale));
            q0 = max(-8, min(7, q0)) + 8;
            q1 = max(-8, min(7, q1)) + 8;
            reinterpret_cast<uint8_t *>(pool)[(e0 + d) >> 1] =
                static_cast<uint8_t>((q0 & 0xF) | ((q1 & 0xF) << 4));
        }
    }
}

__global__ void __launch_bounds__(128) kv_append_kernel(const AppendArgs a) {
    const long long row = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= static_cast<long long>(a.num_tokens) * a.num_kv_heads) return;
    const int t = static_cast<int>(row / a.num_kv_heads);
    const int h = static_cast<int>(row - static_cast<long long>(t) * a.num_kv_heads);
    const int seq = a.token_seq ? a.token_seq[t] : t;
    const int pos = a.token_pos[t];
    if (pos < 0 || pos >= a.max_blocks * a.block_size || seq < 0) {
        if (lane == 0) raise_status(GOLLEK_STATUS_BAD_POSITION);
        return;
    }
    const int page = a.block_tables[static_cast<long long>(seq) * a.max_blocks + pos / a.block_size];
    if (page < 0 || (a.num_blocks > 0 && page >= a.num_blocks)) {
        if (lane == 0) raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
        return;
    }
    const int slot = pos % a.block_size;
    const long long e0 = static_cast<long long>(page) * a.page_stride +
                         (static_cast<long long>(h) * a.block_size + slot) * a.head_dim;
    const long long so = static_cast<long long>(page) * a.scale_page_stride +
                         static_cast<long long>(h) * a.scale_head_stride +
                         static_cast<long long>(slot) * a.scale_token_stride;
    const long long src0 = row * a.head_dim;
    append_row(a, a.key, src0, a.k, a.k_scales, e0, so, lane);
    append_row(a, a.value, src0, a.v, a.v_scales, e0, so, lane);
}

}  // namespace gk
