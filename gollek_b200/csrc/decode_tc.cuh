// decode_tc.cuh -- paged decode attention with the dot products on the 5th-generation
// tensor cores: tcgen05.mma from shared memory into tensor memory, for bf16 KV with
// head_dim 128.
//
// Work: the same 16-token groups and stream-K CTA ranges as decode_tma_kernel
// (decode_common.cuh), cut into tiles of up to 128 tokens (tc_tiles.cuh, which also
// gives the tiles' shared-memory layout).  K and V tiles (32 KB each) live in two
// separate rings, so a K tile is free again as soon as the score MMAs have read it,
// while a V tile waits for the probabilities.  K is the score MMA's K-major A operand
// (2 KB between 8-token core groups), V the value MMA's MN-major A operand (slabs 1 KB
// apart along head_dim, core groups 2 KB apart along tokens).
//
// One CTA per SM, 8 warps:
//   warp 0  K producer, warp 7 V producer: per tile, lane i looks up group i's page
//           (two tiles ahead) and, once its ring slot is free, issues the group's TMA box.
//   warp 1  allocates 64 tensor-memory columns; lane 0 issues the score MMAs
//             S[128 tok x 16] = K[128 tok x 128 d] . Qt
//           and releases the K tile by a commit once they have read it.
//   warp 6  lane 0 issues the value MMAs
//             O[128 d x 16]   = Vt[128 d x 128 tok] . Pt
//           and releases the V tile the same way.
//           The q heads of the GQA group are the 16 MMA columns (zero-padded).  S and O
//           are double-buffered in tensor memory.
//   warps 2-5 (128 threads) softmax: thread i owns token i of the tile for the scores
//           and head-dim row i for the values.  Per tile: scores from tensor memory,
//           window / length mask, running max per head across the 4 warps, exp2,
//           probabilities as bf16 into shared memory (the B operand of the value MMA),
//           out-of-window V rows cleared, then the previous tile's O added into
//           registers (O = O * alpha + O_tile).  At a run's end: normaliser, output or
//           split-K partial, and the last-arriver merge of the partials.
// q of the next two runs is staged ahead (two buffers), so run boundaries do not stall
// the score issuer.  Every wait is bounded; a wait that gives up raises TIMEOUT and the
// CTA drains in-flight copies and MMAs before releasing tensor memory.
#pragma once

#include "tc_tiles.cuh"

namespace gk {

constexpr int kTcN = 16;                                // MMA N: q heads, zero-padded
constexpr uint32_t kTcOpBuf = kTcN * 256;               // 4 KB: 16 rows x 128 16-bit values
constexpr int kTcThreads = 256;
constexpr uint32_t kTcCols = 64;                        // S x2, O x2 (16 columns each)

struct TcSmem {
    uint32_t kring, vring, q, p, red, prefix, cprefix, lens, rstart, misc, bars, total;
};

__host__ __device__ inline TcSmem tc_smem_layout(int kst, int vst, bool split, int num_seqs, int num_ctas) {
    TcSmem L;
    uint32_t o = 0;
    L.kring = o;
    o += kst * kTcTile;
    L.vring = o;
    o += vst * kTcTile;
    L.q = o;  // q hi [2], then (split) q lo [2]
    o += (split ? 4 : 2) * kTcOpBuf;
    L.p = o;  // probabilities [2]
    o += 2 * kTcOpBuf;
    L.red = o;  // tile max [2][4][16], normaliser sums [4][16]
    o += (2 * 4 * kTcN + 4 * kTcN) * 4;
    L.prefix = o;
    o += (num_seqs + 1) * 4;
    L.cprefix = o;
    o += (num_seqs + 1) * 4;
    L.lens = o;
    o += num_seqs * 4;
    o = align_up(o, 16);
    L.rstart = o;
    o += (num_ctas + 1) * 8;
    L.misc = o;
    o += 64;
    L.bars = o;
    o += (2 * kst + 2 * vst + 14) * 8;
    L.total = o + 1024;  // slack to align the base to 1024 bytes
    return L;
}

// Byte offset of 16-bit element (row r, column c) of a [rows][128] operand stored as two
// 128-byte-swizzled 64-column slabs (q and the probabilities).
__device__ __forceinline__ uint32_t sw128_off(int rows, int r, int c) {
    const int b = (c & 63) * 2;
    return static_cast<uint32_t>((c >> 6) * rows * 128 + r * 128 + ((((b >> 4) ^ (r & 7))) << 4) +
                                 (b & 15));
}

// SPLIT: fp32 q enters the score MMAs as bf16 hi + lo halves.
template <int G, bool SPLIT>
__global__ void __launch_bounds__(kTcThreads, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const DecodeArgs a) {
    constexpr int D = 128;
    static_assert(G == 1 || G == 2 || G == 4 || G == 8 || G == 16, "GQA group size");
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int NK = a.num_stages;
    const int NV = a.num_vstages;
    const TcSmem L = tc_smem_layout(NK, NV, SPLIT, a.num_seqs, gridDim.x);
    uint8_t *sm_kring = smem + L.kring;
    uint8_t *sm_vring = smem + L.vring;
    uint8_t *sm_q = smem + L.q;
    uint8_t *sm_p = smem + L.p;
    float *sm_red = reinterpret_cast<float *>(smem + L.red);
    int *sm_prefix = reinterpret_cast<int *>(smem + L.prefix);
    int *sm_cprefix = reinterpret_cast<int *>(smem + L.cprefix);
    int *sm_len = reinterpret_cast<int *>(smem + L.lens);
    long long *sm_rstart = reinterpret_cast<long long *>(smem + L.rstart);
    // [0] merge flag, [1] max groups of a sequence, [2] tensor-memory base, [3] abort
    volatile int *sm_misc = reinterpret_cast<volatile int *>(smem + L.misc);
    uint64_t *k_full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *k_empty = k_full + NK;
    uint64_t *v_full = k_empty + NK;
    uint64_t *v_empty = v_full + NV;
    uint64_t *s_full = v_empty + NV;  // scores in tensor memory [2]
    uint64_t *s_free = s_full + 2;    // scores read by the softmax warps [2]
    uint64_t *p_full = s_free + 2;    // probabilities written [2]
    uint64_t *o_full = p_full + 2;    // value tile in tensor memory [2]
    uint64_t *o_free = o_full + 2;    // value tile read [2]
    uint64_t *q_full = o_free + 2;    // q staged [2]
    uint64_t *mma_done = q_full + 2;  // [2]: score and value issuers drained

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int S = a.num_seqs;
    const int Hkv = a.num_kv_heads;

    if (tid == 0) {
        for (int i = 0; i < NK; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < NV; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
            mbar_init(&p_full[i], 4);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 4);
            mbar_init(&q_full[i], 1);
            mbar_init(&mma_done[i], 1);
        }
        fence_barrier_init();
        sm_misc[0] = 0;
        sm_misc[1] = 0;
        sm_misc[3] = 0;
    }
    if ((warp == 0 || warp == 7) && lane == 0) prefetch_tensormap(warp == 0 ? &tm_k : &tm_v);
    if (warp == 1) {
        tmem_alloc(smem_u32(const_cast<int *>(&sm_misc[2])), kTcCols);
        tmem_relinquish();
    }
    // q and probability buffers start zeroed: the padding rows (heads >= G) stay zero
    for (uint32_t o = tid * 16; o < L.red - L.q; o += kTcThreads * 16)
        sts_u4(smem_u32(sm_q) + o, make_uint4(0, 0, 0, 0));
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = static_cast<uint32_t>(sm_misc[2]);

    const Schedule sch = schedule_prologue(a, sm_prefix, sm_cprefix, sm_len, sm_rstart, &sm_misc[1],
                                           reinterpret_cast<int *>(sm_red));

    if (warp == 0 || warp == 7) {
        // ========================================================= producers (K: warp 0, V: warp 7)
        const bool is_k = warp == 0;
        tc_producer(a, sch, sm_len, &sm_misc[3], is_k ? &tm_k : &tm_v, is_k ? sm_kring : sm_vring,
                    is_k ? k_full : v_full, is_k ? k_empty : v_empty, is_k ? NK : NV, lane);
    } else if (warp == 1) {
        // ========================================================= score MMAs
        if (lane == 0) {
            constexpr uint32_t id_s = umma_idesc_16bit(kTcTokens, kTcN, 1, 0, 0);
            const uint32_t k_base = smem_u32(sm_kring);
            const uint32_t q_base = smem_u32(sm_q);
            for (TileIt is = tile_begin(sch); is.live; tile_next(sch, is)) {
                const int slot = is.ti % NK;
                const int sb = is.ti & 1;
                bool ok = mbar_wait(&k_full[slot], (is.ti / NK) & 1);
                if (ok && is.ti >= 2) ok = mbar_wait(&s_free[sb], ((is.ti >> 1) + 1) & 1);
                if (ok && is.tg0 == 0) ok = mbar_wait(&q_full[is.ri & 1], (is.ri >> 1) & 1);
                if (!ok || sm_misc[3]) {
                    sm_misc[3] = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t kb = k_base + static_cast<uint32_t>(slot) * kTcTile;
                const uint32_t qb = q_base + (is.ri & 1) * kTcOpBuf;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem + 16 * sb, umma_desc_sw128(kb + (kk >> 2) * 1024 + (kk & 3) * 32, 16, 2048),
                             umma_desc_sw128(qb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
                if constexpr (SPLIT) {
                    const uint32_t qlb = q_base + (2 + (is.ri & 1)) * kTcOpBuf;
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        umma_f16(tmem + 16 * sb,
                                 umma_desc_sw128(kb + (kk >> 2) * 1024 + (kk & 3) * 32, 16, 2048),
                                 umma_desc_sw128(qlb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), id_s, 1);
                }
                umma_commit(&s_full[sb]);
                umma_commit(&k_empty[slot]);
            }
            // every MMA issued has completed before tensor memory is released
            umma_commit(&mma_done[0]);
            mbar_wait(&mma_done[0], 0);
        }
        __syncwarp();
    } else if (warp == 6) {
        // ========================================================= value MMAs
        if (lane == 0) {
            constexpr uint32_t id_o = umma_idesc_16bit(D, kTcN, 1, 1, 0);
            const uint32_t v_base = smem_u32(sm_vring);
            const uint32_t p_base = smem_u32(sm_p);
            for (TileIt ip = tile_begin(sch); ip.live; tile_next(sch, ip)) {
                const int slot = ip.ti % NV;
                const int sb = ip.ti & 1;
                bool ok = mbar_wait(&p_full[sb], (ip.ti >> 1) & 1);
                if (ok) ok = mbar_wait(&v_full[slot], (ip.ti / NV) & 1);
                if (ok && ip.ti >= 2) ok = mbar_wait(&o_free[sb], ((ip.ti >> 1) + 1) & 1);
                if (!ok || sm_misc[3]) {
                    sm_misc[3] = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t vb = v_base + static_cast<uint32_t>(slot) * kTcTile;
                const uint32_t pb = p_base + sb * kTcOpBuf;
#pragma unroll
                for (int kk = 0; kk < kTcTokens / 16; ++kk)
                    umma_f16(tmem + 32 + 16 * sb, umma_desc_sw128(vb + kk * 4096, 1024, 2048),
                             umma_desc_sw128(pb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), id_o, kk > 0);
                umma_commit(&o_full[sb]);
                umma_commit(&v_empty[slot]);
            }
            umma_commit(&mma_done[1]);
            mbar_wait(&mma_done[1], 0);
        }
        __syncwarp();
    } else {
        // ========================================================= softmax warps
        const int wq = warp & 3;           // tensor-memory lane quarter of this warp
        const int row = 32 * wq + lane;    // token of the tile (scores), head-dim row (values)
        const int ctid = tid - 64;         // 0..127 (warps 2-5)
        const uint32_t t_lane = static_cast<uint32_t>(32 * wq) << 16;
        const int slot_floats = 2 * G + G * D;

        // Sequences with nothing to attend to: zeros, written by CTA s % grid.
        for (int s = blockIdx.x; s < S; s += gridDim.x) {
            if (sm_prefix[s + 1] != sm_prefix[s]) continue;
            for (int o = ctid; o < Hkv * G * D; o += 128)
                store_out(a.out, static_cast<long long>(s) * Hkv * G * D + o, 0.f, a.q_bf16);
        }

        // q of a run -> buffer `buf` as the score MMA's B operand (rows = heads).
        long long qx = sch.x_beg;
        int qri = 0;
        auto stage_next_q = [&]() {
            if (qx >= sch.x_end) return;
            const Run rq = sch.run_at(qx);
            const int buf = qri & 1;
            for (int c = ctid; c < G * 16; c += 128) {
                const int hh = c >> 4, ch = c & 15;  // head, 8-element chunk
                const long long qo = ((static_cast<long long>(rq.s) * Hkv + rq.h) * G + hh) * D + ch * 8;
                float x[8];
                if (a.q_bf16) {
                    const uint4 w = __ldg(reinterpret_cast<const uint4 *>(
                        reinterpret_cast<const __nv_bfloat16 *>(a.q) + qo));
                    x[0] = bf16_lo(w.x), x[1] = bf16_hi(w.x), x[2] = bf16_lo(w.y), x[3] = bf16_hi(w.y);
                    x[4] = bf16_lo(w.z), x[5] = bf16_hi(w.z), x[6] = bf16_lo(w.w), x[7] = bf16_hi(w.w);
                } else {
                    const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.q) + qo);
                    const float4 u = __ldg(src), v = __ldg(src + 1);
                    x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = v.x, x[5] = v.y, x[6] = v.z, x[7] = v.w;
                }
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
                    hi[i] = *reinterpret_cast<uint32_t *>(&h2);
                    if constexpr (SPLIT) {
                        __nv_bfloat162 l2 = __floats2bfloat162_rn(x[2 * i] - bf16_lo(hi[i]),
                                                                  x[2 * i + 1] - bf16_hi(hi[i]));
                        lo[i] = *reinterpret_cast<uint32_t *>(&l2);
                    }
                }
                const uint32_t off = (ch >> 3) * 2048 + hh * 128 + ((((ch & 7) ^ (hh & 7))) << 4);
                sts_u4(smem_u32(sm_q) + buf * kTcOpBuf + off, make_uint4(hi[0], hi[1], hi[2], hi[3]));
                if constexpr (SPLIT)
                    sts_u4(smem_u32(sm_q) + (2 + buf) * kTcOpBuf + off, make_uint4(lo[0], lo[1], lo[2], lo[3]));
            }
            fence_proxy_async_smem();
            named_barrier(1, 128);
            if (ctid == 0) mbar_arrive(&q_full[buf]);
            qx += rq.len;
            ++qri;
        };
        stage_next_q();
        stage_next_q();

        float m_run[G], l_part[G], o_acc[G], alpha_prev[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
            m_run[h] = -INFINITY;
            l_part[h] = 0.f;
            o_acc[h] = 0.f;
            alpha_prev[h] = 1.f;
        }
        bool bad = false;  // a wait of this warp gave up
        // O of tile u into the registers: o_acc = o_acc * alpha + O_tile(u)
        auto accumulate = [&](int u, const float *alpha) {
            const int ub = u & 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&o_full[ub], (u >> 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            bad |= !ok;
            tc_fence_after();
            float ov[G];
            tmem_ld<G>(tmem + 32 + 16 * ub + t_lane, ov);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[ub]);
#pragma unroll
            for (int h = 0; h < G; ++h) o_acc[h] = o_acc[h] * alpha[h] + ov[h];
        };

        int prev_ti = -1;
        for (TileIt it = tile_begin(sch); it.live;) {
            const int ti = it.ti;
            const int sb = ti & 1;
            const Run r = it.r;
            const int ng = min(kTcGroups, r.len - it.tg0);
            const bool run_end = it.tg0 + kTcGroups >= r.len;
            // ---------------- scores of this tile
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&s_full[sb], (ti >> 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            bad |= !ok;
            tc_fence_after();
            float sv[G];
            tmem_ld<G>(tmem + 16 * sb + t_lane, sv);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[sb]);
            const int len = sm_len[r.s];
            const int ws = tc_win_start(a, len);
            const int gi = row >> 4;
            const int tok = (ws / kRows + r.g + it.tg0 + gi) * kRows + (row & 15);
            const bool valid = gi < ng && tok >= ws && tok < len;
            float x[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float v = sv[h] * a.q_scale;
                if (a.soft_cap > 0.f) v = a.soft_cap * tanhf(v / a.soft_cap) * a.post_scale;
                x[h] = valid ? v : -INFINITY;
            }
            // ---------------- running max per head over the 128 tokens (4 warps)
            float *red = sm_red + sb * 4 * kTcN;
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float mx = warp_max(x[h]);
                if (lane == 0) red[wq * kTcN + h] = mx;
            }
            if (bar_red_or(1, 128, bad)) {
                if (ctid == 0) sm_misc[3] = 1;
                break;
            }
            float alpha[G], mref[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float tmax = fmaxf(fmaxf(red[h], red[kTcN + h]), fmaxf(red[2 * kTcN + h], red[3 * kTcN + h]));
                const float mn = fmaxf(m_run[h], tmax);
                alpha[h] = (mn == m_run[h]) ? 1.f : fast_exp2(m_run[h] - mn);
                m_run[h] = mn;
                mref[h] = (mn == -INFINITY) ? 0.f : mn;
            }
            // ---------------- probabilities -> bf16 B operand of the value MMA
            const uint32_t pb = smem_u32(sm_p) + sb * kTcOpBuf;
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float p = fast_exp2(x[h] - mref[h]);
                l_part[h] = l_part[h] * alpha[h] + p;
                const __nv_bfloat16 pbf = __float2bfloat16_rn(p);
                asm volatile("st.shared.b16 [%0], %1;" ::"r"(pb + sw128_off(kTcN, h, row)),
                             "h"(*reinterpret_cast<const unsigned short *>(&pbf))
                             : "memory");
            }
            if (!valid) {
                // Rows outside the window may hold anything (NaN included) and a zero
                // probability does not cancel a NaN on the tensor pipe: clear them, once
                // the tile's V copies have landed.
                const int vslot = ti % NV;
                if (!mbar_wait(&v_full[vslot], (ti / NV) & 1)) bad = true;
                const uint32_t vt = smem_u32(sm_vring) + static_cast<uint32_t>(vslot) * kTcTile;
#pragma unroll
                for (int c = 0; c < 16; ++c) sts_u4(vt + tile_chunk_off(row, c), make_uint4(0, 0, 0, 0));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[sb]);
            // ---------------- the previous tile's values (same run)
            if (prev_ti >= 0) accumulate(prev_ti, alpha_prev);
#pragma unroll
            for (int h = 0; h < G; ++h) alpha_prev[h] = alpha[h];
            prev_ti = ti;
            tile_next(sch, it);
            if (!run_end) continue;

            // ---------------- end of the run
            accumulate(ti, alpha_prev);
            prev_ti = -1;
            float *lsum = sm_red + 2 * 4 * kTcN;
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float lw = warp_sum(l_part[h]);
                if (lane == 0) lsum[wq * kTcN + h] = lw;
            }
            if (bar_red_or(1, 128, bad)) {
                if (ctid == 0) sm_misc[3] = 1;
                break;
            }
            float lt[G];
#pragma unroll
            for (int h = 0; h < G; ++h)
                lt[h] = (lsum[h] + lsum[kTcN + h]) + (lsum[2 * kTcN + h] + lsum[3 * kTcN + h]);
            const long long out_row = (static_cast<long long>(r.s) * Hkv + r.h) * G * D;
            if (r.pieces == 1) {
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float v = lt[h] > 0.f ? o_acc[h] * (1.0f / (lt[h] + a.norm_eps)) : 0.f;
                    store_out(a.out, out_row + h * D + row, v, a.q_bf16);
                }
            } else {
                float *part = a.partials +
                              (static_cast<long long>(r.s * Hkv + r.h) * kMaxSplits + r.piece) * slot_floats;
#pragma unroll
                for (int h = 0; h < G; ++h) part[2 * G + h * D + row] = o_acc[h];
                if (ctid == 0) {
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        part[h] = m_run[h];
                        part[G + h] = lt[h];
                    }
                }
                __threadfence();
                named_barrier(1, 128);
                if (ctid == 0) {
                    const int old = atomicAdd(&a.counters[r.s * Hkv + r.h], 1);
                    sm_misc[0] = (old == r.pieces - 1) ? 1 : 0;
                }
                named_barrier(1, 128);
                if (sm_misc[0]) {
                    __threadfence();
                    const float *base =
                        a.partials + static_cast<long long>(r.s * Hkv + r.h) * kMaxSplits * slot_floats;
                    for (int o = ctid; o < G * D; o += 128) {
                        const int hh = o / D;
                        float M = -INFINITY;
                        for (int c = 0; c < r.pieces; ++c) M = fmaxf(M, __ldcg(base + c * slot_floats + hh));
                        float Ls = 0.f, As = 0.f;
                        if (M != -INFINITY) {
                            for (int c = 0; c < r.pieces; ++c) {
                                const float *pc = base + c * slot_floats;
                                const float mc = __ldcg(pc + hh);
                                const float f = (mc == -INFINITY) ? 0.f : fast_exp2(mc - M);
                                Ls += __ldcg(pc + G + hh) * f;
                                As += __ldcg(pc + 2 * G + o) * f;
                            }
                        }
                        const float v = Ls > 0.f ? As * (1.0f / (Ls + a.norm_eps)) : 0.f;
                        store_out(a.out, out_row + o, v, a.q_bf16);
                    }
                    if (ctid == 0) atomicExch(&a.counters[r.s * Hkv + r.h], 0);
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h) {
                m_run[h] = -INFINITY;
                l_part[h] = 0.f;
                o_acc[h] = 0.f;
            }
            stage_next_q();
        }
    }

    // ------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTcCols);
}

}  // namespace gk
