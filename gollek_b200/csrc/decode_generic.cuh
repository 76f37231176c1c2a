// decode_generic.cuh -- paged decode attention for shapes outside the TMA path
// (any head_dim <= 256, any block size, int4 storage, unaligned pools).
//
// One CTA (4 warps) per (sequence, kv-head).  Warp w takes tokens w, w+4, ... of
// the window; lane j owns head-dim columns j, j+32, ...; each token's score is a
// warp reduction per query head; online softmax per warp; the 4 warp states merge
// through shared memory.  Correct for every shape the ABI accepts; the hot shapes
// go through decode_tma_kernel instead.
#pragma once

#include "common.cuh"

namespace gk {

constexpr int kGenMaxG = 8;
constexpr int kGenMaxJ = 8;  // head_dim <= 256
constexpr int kGenWarps = 4;

struct GenericArgs {
    void *out;
    const void *q;
    const void *k;
    const void *v;
    const float *k_scales;
    const float *v_scales;
    const int *block_tables;
    const int *context_lens;
    long long page_stride;  // elements (nibbles for int4)
    long long scale_page_stride, scale_head_stride, scale_token_stride;
    int num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, num_blocks;
    int window, q_bf16, kv_dtype;
    int seq_div;  // block-table row of sequence s is s / seq_div
    float q_scale, soft_cap, post_scale, norm_eps;
};

__device__ __forceinline__ float load_kv(const void *base, int dtype, long long e) {
    switch (dtype) {
        case GOLLEK_DTYPE_F32:
            return reinterpret_cast<const float *>(base)[e];
        case GOLLEK_DTYPE_BF16:
            return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(base)[e]);
        case GOLLEK_DTYPE_F16:
            return __half2float(reinterpret_cast<const __half *>(base)[e]);
        case GOLLEK_DTYPE_I8:
            return static_cast<float>(reinterpret_cast<const int8_t *>(base)[e]);
        default: {  // I4: nibble e of the byte stream, stored as value + 8
            const int b = reinterpret_cast<const uint8_t *>(base)[e >> 1];
            const int nib = (e & 1) ? ((b >> 4) & 0xF) : (b & 0xF);
            return static_cast<float>(nib - 8);
        }
    }
}

__global__ void __launch_bounds__(kGenWarps * 32) decode_generic_kernel(const GenericArgs a) {
    const int s = blockIdx.x;
    const int h = blockIdx.y;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = a.num_q_heads / a.num_kv_heads;
    const int D = a.head_dim;
    const int BS = a.block_size;

    __shared__ float sm_m[kGenWarps][kGenMaxG];
    __shared__ float sm_l[kGenWarps][kGenMaxG];
    __shared__ float sm_acc[kGenWarps][kGenMaxG][kGenMaxJ * 32];

    int len = a.context_lens[s];
    if (len < 0 || len > a.max_blocks * BS) {
        if (threadIdx.x == 0) raise_status(GOLLEK_STATUS_BAD_POSITION);
        len = len < 0 ? 0 : a.max_blocks * BS;
    }
    const int win_start = (a.window > 0 && len > a.window) ? len - a.window : 0;

    float qr[kGenMaxG][kGenMaxJ];
    const long long qrow = (static_cast<long long>(s) * a.num_kv_heads + h) * G * D;
#pragma unroll
    for (int hh = 0; hh < kGenMaxG; ++hh)
#pragma unroll
        for (int j = 0; j < kGenMaxJ; ++j) {
            const int d = lane + 32 * j;
            float v = 0.f;
            if (hh < G && d < D) {
                const long long i = qrow + static_cast<long long>(hh) * D + d;
                v = a.q_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.q)[i])
                             : reinterpret_cast<const float *>(a.q)[i];
            }
            qr[hh][j] = v * a.q_scale;
        }

    float m[kGenMaxG], l[kGenMaxG], acc[kGenMaxG][kGenMaxJ];
#pragma unroll
    for (int hh = 0; hh < kGenMaxG; ++hh) {
        m[hh] = -INFINITY;
        l[hh] = 0.f;
#pragma unroll
        for (int j = 0; j < kGenMaxJ; ++j) acc[hh][j] = 0.f;
    }

    const bool quant = a.kv_dtype == GOLLEK_DTYPE_I8 || a.kv_dtype == GOLLEK_DTYPE_I4;
    for (int t = win_start + warp; t < len; t += kGenWarps) {
        int page = a.block_tables[static_cast<long long>(s / a.seq_div) * a.max_blocks + t / BS];
        if (page < 0 || (a.num_blocks > 0 && page >= a.num_blocks)) {
            if (lane == 0) raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
            continue;
        }
        const int slot = t % BS;
        const long long e0 = static_cast<long long>(page) * a.page_stride +
                             (static_cast<long long>(h) * BS + slot) * D;
        float ks = 1.f, vs = 1.f;
        if (quant) {
            const long long so = static_cast<long long>(page) * a.scale_page_stride +
                                 static_cast<long long>(h) * a.scale_head_stride +
                                 static_cast<long long>(slot) * a.scale_token_stride;
            ks = a.k_scales ? a.k_scales[so] : 1.f;
            vs = a.v_scales ? a.v_scales[so] : 1.f;
        }
        float kv[kGenMaxJ], vv[kGenMaxJ];
#pragma unroll
        for (int j = 0; j < kGenMaxJ; ++j) {
            const int d = lane + 32 * j;
            kv[j] = d < D ? load_kv(a.k, a.kv_dtype, e0 + d) : 0.f;
            vv[j] = d < D ? load_kv(a.v, a.kv_dtype, e0 + d) * vs : 0.f;
        }
#pragma unroll
        for (int hh = 0; hh < kGenMaxG; ++hh) {
            if (hh >= G) break;
            float part = 0.f;
#pragma unroll
            for (int j = 0; j < kGenMaxJ; ++j) part += qr[hh][j] * kv[j];
            float sc = warp_sum(part) * ks;
            if (a.soft_cap > 0.f) sc = a.soft_cap * tanhf(sc / a.soft_cap) * a.post_scale;
            const float mn = fmaxf(m[hh], sc);
            const float alpha = (mn == m[hh]) ? 1.f : fast_exp2(m[hh] - mn);
            const float p = fast_exp2(sc - mn);
            l[hh] = l[hh] * alpha + p;
            m[hh] = mn;
#pragma unroll
            for (int j = 0; j < kGenMaxJ; ++j) acc[hh][j] = acc[hh][j] * alpha + p * vv[j];
        }
    }

#pragma unroll
    for (int hh = 0; hh < kGenMaxG; ++hh) {
        if (lane == 0) {
            sm_m[warp][hh] = m[hh];
            sm_l[warp][hh] = l[hh];
        }
#pragma unroll
        for (int j = 0; j < kGenMaxJ; ++j) sm_acc[warp][hh][lane + 32 * j] = acc[hh][j];
    }
    __syncthreads();
    for (int o = threadIdx.x; o < G * D; o += kGenWarps * 32) {
        const int hh = o / D;
        const int d = o - hh * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kGenWarps; ++w) M = fmaxf(M, sm_m[w][hh]);
        float Ls = 0.f, As = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kGenWarps; ++w) {
                const float f = (sm_m[w][hh] == -INFINITY) ? 0.f : fast_exp2(sm_m[w][hh] - M);
                Ls += sm_l[w][hh] * f;
                As += sm_acc[w][hh][d] * f;
            }
        }
        const float v = Ls > 0.f ? As * (1.0f / (Ls + a.norm_eps)) : 0.f;
        const long long oi = qrow + o;
        if (a.q_bf16)
            reinterpret_cast<__nv_bfloat16 *>(a.out)[oi] = __float2bfloat16_rn(v);
        else
            reinterpret_cast<float *>(a.out)[oi] = v;
    }
}

}  // namespace gk
