// prefill_tc.cuh -- multi-query paged attention (the queries of a prefill chunk, or
// speculative tokens, over the paged cache) on the 5th-generation tensor cores, for bf16
// KV and bf16 q with head_dim 128.
//
// The folded rows of a (chunk, kv-head) unit -- F queries x G heads, NQ = 64 of them
// (qo_row, decode_common.cuh; 32 works too, padded, but the library forms no 32-row
// folds) -- are the N columns of both MMAs, the tile's 128 tokens and the 128 head-dim
// rows their M rows:
//
//   S^T[128 tok x 64] = K[128 tok x 128 d] . Q^T                 (S[tile & 1], per tile)
//   O^T[128 d x 64]  += V^T[128 d x 128 tok] . P^T[128 tok x 64]  (one O per run)
//
// so the 128 softmax threads (4 warps, all four SM sub-partitions) each own one token of
// a tile (its NQ scores) and one head-dim row of O.  Every row's exponent reference is
// lazy: the NQ references sit in shared memory and the warps agree once per tile
// (barrier.cta.red.or) whether any score passed its row's reference by more than
// 2^kPtLazyMax; only then do they reduce the tile's column maxima, rescale O in tensor
// memory and redo the tile.  Row sums stay per thread until a run ends.
//
// Operands: K is the score MMA's K-major A operand and V the value MMA's MN-major A
// operand (tc_tiles.cuh); Q (64 rows x 128 d, two 64-column slabs) the K-major B operand;
// P^T the MN-major B operand: one 128-byte row (64 bf16 columns) per token, 8-token core
// groups 1 KB apart, so a thread writes its token's probabilities as 16-byte stores.
// Columns NQ..63 are padding whose scores and values nobody reads.
//
// Work: the stream-K ranges and 128-token tiles of tc_tiles.cuh.  One CTA per SM, 8 warps:
//   warp 0 K producer, warp 7 V producer (tc_producer);
//   warp 1 allocates tensor memory; lane 0 issues the score MMAs;
//   warp 6 lane 0 issues the value MMAs (overwriting O at a run's first tile);
//   warps 2-5 softmax (thread = token of the tile, and head-dim row of O).
// Every wait is bounded and gives up once another warp has given up; the softmax warps
// meet at one reducing barrier per tile, so they always leave together; tensor memory
// is released only after both MMA issuers have drained.
#pragma once

#include <type_traits>

#include "tc_tiles.cuh"

namespace gk {

constexpr int kPtThreads = 256;
constexpr int kPtN = 64;                       // MMA N: the folded rows, padded
constexpr uint32_t kPtCols = 256;              // S x2 (64 columns each), O (64)
constexpr uint32_t kPtQBuf = kPtN * 256;       // 16 KB: 64 rows x 128 bf16
constexpr uint32_t kPtPBuf = kTcTokens * 128;  // 16 KB: 128 tokens x 64 bf16

// Polling waits sleep this long between tests, which keeps the shared-memory pipe free for
// the MMA issue, tensor-memory loads and stores of the working warps.
constexpr unsigned kPtPollNs = 128;

// Scores may exceed their row's exponent reference by this much (log2 units) before the
// reference moves: probabilities stay below 2^8, far inside bf16 and fp32.
constexpr float kPtLazyMax = 8.f;

struct PtSmem {
    uint32_t kring, vring, q, p, red, prefix, cprefix, lens, rstart, misc, bars, total;
};

__host__ __device__ inline PtSmem pt_smem_layout(int kst, int vst, int num_seqs, int num_ctas) {
    PtSmem L;
    uint32_t o = 0;
    L.kring = o;
    o += kst * kTcTile;
    L.vring = o;
    o += vst * kTcTile;
    L.q = o;  // q of the current run (staged again when a run ends)
    o += kPtQBuf;
    L.p = o;  // P^T [2]
    o += 2 * kPtPBuf;
    L.red = o;  // per-warp column values [4][64], the combined [64], row references, factors
    o += 7 * kPtN * 4;
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
    o += (2 * kst + 2 * vst + 12) * 8;
    L.total = o + 1024;  // slack to align the base to 1024 bytes
    return L;
}

// Max (MAX) or sum over the 128 softmax threads (4 warps, named barrier 1) of one value
// per column j < NC; the result lands in red[4 * kPtN + j].
template <int NC, bool MAX>
__device__ __forceinline__ void pt_reduce_cols(const float *v, float *red, int wq, int lane, int ctid) {
#pragma unroll
    for (int j = 0; j < NC; ++j) {
        const float x = MAX ? warp_max(v[j]) : warp_sum(v[j]);
        if (lane == 0) red[wq * kPtN + j] = x;
    }
    named_barrier(1, 128);
    if (ctid < NC) {
        const float a0 = red[ctid], a1 = red[kPtN + ctid], a2 = red[2 * kPtN + ctid], a3 = red[3 * kPtN + ctid];
        red[4 * kPtN + ctid] = MAX ? fmaxf(fmaxf(a0, a1), fmaxf(a2, a3)) : (a0 + a1) + (a2 + a3);
    }
    named_barrier(1, 128);
}

template <int NQ>
__global__ void __launch_bounds__(kPtThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const DecodeArgs a) {
    constexpr int D = 128;
    static_assert(NQ == 32 || NQ == 64, "rows per unit");
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int NK = a.num_stages;
    const int NV = a.num_vstages;
    const PtSmem L = pt_smem_layout(NK, NV, a.num_seqs, gridDim.x);
    uint8_t *sm_kring = smem + L.kring;
    uint8_t *sm_vring = smem + L.vring;
    const uint32_t q_s = smem_u32(smem + L.q);
    const uint32_t p_s = smem_u32(smem + L.p);
    float *sm_red = reinterpret_cast<float *>(smem + L.red);
    int *sm_prefix = reinterpret_cast<int *>(smem + L.prefix);
    int *sm_cprefix = reinterpret_cast<int *>(smem + L.cprefix);
    int *sm_len = reinterpret_cast<int *>(smem + L.lens);
    long long *sm_rstart = reinterpret_cast<long long *>(smem + L.rstart);
    // [0] merge flag, [1] max groups of a sequence, [2] tensor-memory base, [3] abort
    volatile int *sm_misc = reinterpret_cast<volatile int *>(smem + L.misc);
    volatile int *abort = &sm_misc[3];
    uint64_t *k_full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *k_empty = k_full + NK;
    uint64_t *v_full = k_empty + NK;
    uint64_t *v_empty = v_full + NV;
    uint64_t *s_full = v_empty + NV;  // [2] scores in tensor memory
    uint64_t *s_free = s_full + 2;    // [2] scores read by the softmax warps
    uint64_t *p_full = s_free + 2;    // [2] probabilities written (and O rescaled)
    uint64_t *o_done = p_full + 2;    // [2] a tile's value MMAs complete
    uint64_t *o_free = o_done + 2;    // [1] O read at a run's end
    uint64_t *q_full = o_free + 1;    // [1] q staged
    uint64_t *mma_done = q_full + 2;  // [2] score and value issuers drained

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
            mbar_init(&o_done[i], 1);
            mbar_init(&mma_done[i], 1);
        }
        mbar_init(o_free, 4);
        mbar_init(q_full, 1);
        fence_barrier_init();
        sm_misc[0] = 0;
        sm_misc[1] = 0;
        sm_misc[3] = 0;
    }
    if ((warp == 0 || warp == 7) && lane == 0) prefetch_tensormap(warp == 0 ? &tm_k : &tm_v);
    if (warp == 1) {
        tmem_alloc(smem_u32(const_cast<int *>(&sm_misc[2])), kPtCols);
        tmem_relinquish();
    }
    // q rows NQ..63 (padding) stay zero
    for (uint32_t o = tid * 16; o < kPtQBuf; o += kPtThreads * 16) sts_u4(q_s + o, make_uint4(0, 0, 0, 0));
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = static_cast<uint32_t>(sm_misc[2]);
    const uint32_t t_o = tmem + 2 * kPtN;  // O^T columns

    const Schedule sch = schedule_prologue(a, sm_prefix, sm_cprefix, sm_len, sm_rstart, &sm_misc[1],
                                           reinterpret_cast<int *>(sm_red));

    if (warp == 0 || warp == 7) {
        // ========================================================= producers (K: warp 0, V: warp 7)
        const bool is_k = warp == 0;
        tc_producer(a, sch, sm_len, abort, is_k ? &tm_k : &tm_v, is_k ? sm_kring : sm_vring,
                    is_k ? k_full : v_full, is_k ? k_empty : v_empty, is_k ? NK : NV, lane, kPtPollNs);
    } else if (warp == 1) {
        // ========================================================= score MMAs
        if (lane == 0) {
            constexpr uint32_t id_s = umma_idesc_16bit(kTcTokens, kPtN, 1, 0, 0);
            const uint32_t k_base = smem_u32(sm_kring);
            for (TileIt is = tile_begin(sch); is.live; tile_next(sch, is)) {
                const int slot = is.ti % NK;
                const int sb = is.ti & 1;
                bool ok = mbar_wait_or_abort(&k_full[slot], (is.ti / NK) & 1, abort, kWaitLimit, kPtPollNs);
                if (ok && is.ti >= 2) ok = mbar_wait_or_abort(&s_free[sb], ((is.ti >> 1) + 1) & 1, abort, kWaitLimit, kPtPollNs);
                if (ok && is.tg0 == 0) ok = mbar_wait_or_abort(q_full, is.ri & 1, abort, kWaitLimit, kPtPollNs);
                if (!ok) {
                    *abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t kb = k_base + static_cast<uint32_t>(slot) * kTcTile;
                const uint32_t qb = q_s;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem + kPtN * sb, umma_desc_sw128(kb + (kk >> 2) * 1024 + (kk & 3) * 32, 16, 2048),
                             umma_desc_sw128(qb + (kk >> 2) * (kPtN * 128) + (kk & 3) * 32, 16, 1024), id_s,
                             kk > 0);
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
            constexpr uint32_t id_o = umma_idesc_16bit(D, kPtN, 1, 1, 1);
            const uint32_t v_base = smem_u32(sm_vring);
            for (TileIt ip = tile_begin(sch); ip.live; tile_next(sch, ip)) {
                const int slot = ip.ti % NV;
                const int sb = ip.ti & 1;
                bool ok = mbar_wait_or_abort(&p_full[sb], (ip.ti >> 1) & 1, abort, kWaitLimit, kPtPollNs);
                if (ok) ok = mbar_wait_or_abort(&v_full[slot], (ip.ti / NV) & 1, abort, kWaitLimit, kPtPollNs);
                if (ok && ip.tg0 == 0 && ip.ri > 0) ok = mbar_wait_or_abort(o_free, (ip.ri - 1) & 1, abort, kWaitLimit, kPtPollNs);
                if (!ok) {
                    *abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t vb = v_base + static_cast<uint32_t>(slot) * kTcTile;
                const uint32_t pb = p_s + static_cast<uint32_t>(sb) * kPtPBuf;
#pragma unroll
                for (int kk = 0; kk < kTcTokens / 16; ++kk)
                    umma_f16(t_o, umma_desc_sw128(vb + kk * 4096, 1024, 2048),
                             umma_desc_sw128(pb + kk * 2048, kPtPBuf, 1024), id_o, (ip.tg0 > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&o_done[sb]);
                umma_commit(&v_empty[slot]);
            }
            umma_commit(&mma_done[1]);
            mbar_wait(&mma_done[1], 0);
        }
        __syncwarp();
    } else {
        // ========================================================= softmax warps (2-5)
        const int wq = warp & 3;                                   // tensor-memory lane quarter
        const int row = 32 * wq + lane;                            // token of the tile; head-dim row of O
        const int ctid = tid - 64;                                 // 0..127
        const uint32_t t_lane = static_cast<uint32_t>(32 * wq) << 16;
        const unsigned wl = a.wait_limit ? a.wait_limit : kWaitLimit;
        const int gm = NQ / a.qfold;                               // heads per query
        const int slot_floats = 2 * NQ + NQ * D;
        float *red_out = sm_red + 4 * kPtN;                        // combined column values
        float *sm_mref = sm_red + 5 * kPtN;                        // row references (-inf: none yet)
        float *sm_alpha = sm_red + 6 * kPtN;                       // their last moves' factors
        if (ctid < kPtN) sm_mref[ctid] = -INFINITY;                // (published by stage_next_q's barrier)

        // Sequences with nothing to attend to: zeros, written by CTA s % grid.
        for (int s = blockIdx.x; s < S; s += gridDim.x) {
            if (sm_prefix[s + 1] != sm_prefix[s]) continue;
            for (int o = ctid; o < Hkv * NQ * D; o += 128)
                store_out(a.out, static_cast<long long>(s) * Hkv * NQ * D + o, 0.f, 1);
        }

        // q of the next run -> the q buffer (rows = the unit's NQ folded rows); called when
        // the score MMAs of the previous run have completed
        long long qx = sch.x_beg;
        auto stage_next_q = [&]() {
            if (qx >= sch.x_end) return;
            const Run rq = sch.run_at(qx);
            for (int c = ctid; c < NQ * 16; c += 128) {
                const int rr = c >> 4, ch = c & 15;  // row, 8-element chunk
                const uint4 w = __ldg(reinterpret_cast<const uint4 *>(
                    reinterpret_cast<const __nv_bfloat16 *>(a.q) +
                    qo_row(rq.s, rq.h, rr, Hkv, NQ, a.qfold, a.seq_div) * D + ch * 8));
                sts_u4(q_s + (ch >> 3) * (kPtN * 128) + rr * 128 +
                           ((((ch & 7) ^ (rr & 7))) << 4),
                       w);
            }
            fence_proxy_async_smem();
            named_barrier(1, 128);
            if (ctid == 0) mbar_arrive(q_full);
            qx += rq.len;
        };
        stage_next_q();

        float lp[NQ];  // this thread's share of each row's normaliser
#pragma unroll
        for (int j = 0; j < NQ; ++j) lp[j] = 0.f;
        const float qs = a.q_scale;
        const bool cap = a.soft_cap > 0.f;
        // this thread's probabilities of the tile (row j of P^T: token `row`) against the
        // references, packed as bf16 pairs; rows j < jmin do not see the token; dmax: the
        // largest x - reference over the rows that do
        auto probs_t = [&](auto cap_t, int sb, int jmin, uint32_t *pk, float &dmax) {
            constexpr bool CAP = decltype(cap_t)::value;
            dmax = -INFINITY;
#pragma unroll
            for (int c32 = 0; c32 < NQ / 32; ++c32) {
                float v[32], mr[32];
                tmem_ld<32>(tmem + kPtN * sb + 32 * c32 + t_lane, v);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 m4 = lds_f4(smem_u32(sm_mref + 32 * c32 + 4 * i));
                    mr[4 * i] = m4.x;
                    mr[4 * i + 1] = m4.y;
                    mr[4 * i + 2] = m4.z;
                    mr[4 * i + 3] = m4.w;
                }
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    float pe[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int j = 32 * c32 + i + e;
                        float d;
                        if constexpr (CAP)
                            d = a.soft_cap * tanhf(v[i + e] * qs / a.soft_cap) * a.post_scale - mr[i + e];
                        else
                            d = fmaf(v[i + e], qs, -mr[i + e]);
                        d = (j >= jmin) ? d : -INFINITY;
                        dmax = fmaxf(dmax, d);
                        pe[e] = fast_exp2(d);
                    }
                    pk[(32 * c32 + i) >> 1] = pack2<__nv_bfloat16>(pe[0], pe[1]);
                }
            }
        };
        auto probs = [&](int sb, int jmin, uint32_t *pk, float &dmax) {
            if (cap)
                probs_t(std::true_type{}, sb, jmin, pk, dmax);
            else
                probs_t(std::false_type{}, sb, jmin, pk, dmax);
        };
        auto add_sums = [&](const uint32_t *pk) {
#pragma unroll
            for (int i = 0; i < NQ / 2; ++i) {
                lp[2 * i] += __uint_as_float(pk[i] << 16);
                lp[2 * i + 1] += __uint_as_float(pk[i] & 0xffff0000u);
            }
        };
        bool bad = false;  // a wait of this thread's warp gave up
        for (TileIt it = tile_begin(sch); it.live;) {
            const int ti = it.ti;
            const int sb = ti & 1;
            const Run r = it.r;
            const int ng = min(kTcGroups, r.len - it.tg0);
            const bool run_end = it.tg0 + kTcGroups >= r.len;
            const int len = sm_len[r.s];
            const int ws = tc_win_start(a, len);
            const int t0 = (ws / kRows + r.g + it.tg0) * kRows;  // position of the tile's token 0
            const int pos = t0 + row;
            // row j's query sees the positions before len - (qfold - 1 - j / gm): the token is
            // seen by rows jmin.. (none when it lies outside the run's tokens or the window)
            const bool tok_ok = row < ng * kRows && pos >= ws && pos < len;
            const int jmin = tok_ok ? max(0, gm * (a.qfold - 1 - (len - 1 - pos))) : NQ;
            bool ok = warp_wait(&s_full[sb], (ti >> 1) & 1, wl, abort, kPtPollNs);
            // the probability buffer is free once the value MMAs of tile ti - 2 completed
            if (ok && ti >= 2) ok = warp_wait(&o_done[sb], ((ti - 2) >> 1) & 1, wl, abort, kPtPollNs);
            bad |= !ok;
            tc_fence_after();
            uint32_t pk[NQ / 2];
            float dmax = -INFINITY;
            // a run's first tile sets the references; later ones keep them unless a score
            // passes its row's by more than 2^kPtLazyMax
            const bool first = it.tg0 == 0;
            if (!bad && !first) probs(sb, jmin, pk, dmax);
            if (bar_red_or(1, 128, bad || first || dmax > kPtLazyMax)) {
                if (bar_red_or(1, 128, bad)) {
                    if (ctid == 0) *abort = 1;
                    break;
                }
                // ---------------- move the references to the tile's column maxima
#pragma unroll 1
                for (int c32 = 0; c32 < NQ / 32; ++c32) {
                    float cm[32];
                    tmem_ld<32>(tmem + kPtN * sb + 32 * c32 + t_lane, cm);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float x = cap ? a.soft_cap * tanhf(cm[i] * qs / a.soft_cap) * a.post_scale : cm[i] * qs;
                        cm[i] = (32 * c32 + i >= jmin) ? x : -INFINITY;
                    }
                    pt_reduce_cols<32, true>(cm, sm_red, wq, lane, ctid);
                    if (ctid < 32) {
                        const int j = 32 * c32 + ctid;
                        const float old = sm_mref[j];
                        const float mn = fmaxf(old, red_out[ctid]);
                        sm_mref[j] = mn;
                        sm_alpha[j] = (mn == old) ? 1.f : fast_exp2(old - mn);
                    }
                    named_barrier(1, 128);
                }
                bool moved = false;
#pragma unroll
                for (int j = 0; j < NQ; ++j) {
                    const float alpha = sm_alpha[j];
                    moved |= alpha != 1.f;
                    lp[j] *= alpha;
                }
                if (moved && !first) {
                    // O holds this run's earlier tiles: once the previous tile's value MMAs
                    // are complete, scale column j of head-dim row `row` by alpha_j
                    if (warp_wait(&o_done[(ti - 1) & 1], ((ti - 1) >> 1) & 1, wl, abort, kPtPollNs)) {
                        tc_fence_after();
#pragma unroll 1
                        for (int c32 = 0; c32 < NQ / 32; ++c32) {
                            float o[32];
                            tmem_ld<32>(t_o + 32 * c32 + t_lane, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] *= sm_alpha[32 * c32 + i];
                            tmem_st32(t_o + 32 * c32 + t_lane, o);
                        }
                        tmem_wait_st();
                    } else {
                        bad = true;  // the next barrier takes every warp out
                    }
                }
                probs(sb, jmin, pk, dmax);
            }
            add_sums(pk);
            // ---------------- P^T row `row`: NQ bf16 columns, 16-byte chunks (128-byte swizzle)
            {
                const uint32_t prow = p_s + static_cast<uint32_t>(sb) * kPtPBuf + row * 128;
#pragma unroll
                for (int c8 = 0; c8 < NQ / 8; ++c8)
                    sts_u4(prow + ((c8 ^ (row & 7)) << 4),
                           make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]));
            }
            if (__any_sync(0xffffffffu, !tok_ok)) {
                // V rows of tokens no row may see are cleared once the tile's V copies have
                // landed (a zero probability does not cancel a NaN on the tensor pipe)
                const int vslot = ti % NV;
                if (warp_wait(&v_full[vslot], (ti / NV) & 1, wl, abort, kPtPollNs)) {
                    if (!tok_ok) {
                        const uint32_t vt = smem_u32(sm_vring) + static_cast<uint32_t>(vslot) * kTcTile;
#pragma unroll
                        for (int ch = 0; ch < 16; ++ch) sts_u4(vt + tile_chunk_off(row, ch), make_uint4(0, 0, 0, 0));
                    }
                } else {
                    bad = true;
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s_free[sb]);
                mbar_arrive(&p_full[sb]);
            }
            tile_next(sch, it);
            if (!run_end) continue;

            // ---------------- end of the run: normalisers, then O^T from tensor memory
            pt_reduce_cols<NQ, false>(lp, sm_red, wq, lane, ctid);
            if (bar_red_or(1, 128, bad || !warp_wait(&o_done[sb], (ti >> 1) & 1, wl, abort, kPtPollNs))) {
                if (ctid == 0) *abort = 1;
                break;
            }
            tc_fence_after();
            const long long unit = static_cast<long long>(r.s) * Hkv + r.h;
            float *part = a.partials + (unit * kMaxSplits + r.piece) * slot_floats;
#pragma unroll 1
            for (int c32 = 0; c32 < NQ / 32; ++c32) {
                float o[32];
                tmem_ld<32>(t_o + 32 * c32 + t_lane, o);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int j = 32 * c32 + i;
                    if (r.pieces == 1) {
                        const float l = red_out[j];
                        const float v = l > 0.f ? o[i] * (1.0f / (l + a.norm_eps)) : 0.f;
                        store_out(a.out, qo_row(r.s, r.h, j, Hkv, NQ, a.qfold, a.seq_div) * D + row, v, 1);
                    } else {
                        part[2 * NQ + j * D + row] = o[i];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            if (r.pieces > 1) {
                // this piece's (reference, normaliser, O) per row; the last piece of the unit
                // to arrive merges them (log-sum-exp)
                if (ctid < NQ) {
                    part[ctid] = sm_mref[ctid];
                    part[NQ + ctid] = red_out[ctid];
                }
                __threadfence();
                named_barrier(1, 128);
                if (ctid == 0) {
                    const int old = atomicAdd(&a.counters[unit], 1);
                    sm_misc[0] = (old == r.pieces - 1) ? 1 : 0;
                }
                named_barrier(1, 128);
                if (sm_misc[0]) {
                    __threadfence();
                    const float *base = a.partials + unit * kMaxSplits * slot_floats;
                    // thread t: head-dim columns 4 (f % 32) .. + 3 of row f / 32, f = t, t + 128, ...
                    for (int f = ctid; f < NQ * D / 4; f += 128) {
                        const int hh = f / (D / 4);
                        const int d4 = f - hh * (D / 4);
                        float M = -INFINITY;
                        for (int pc = 0; pc < r.pieces; ++pc) M = fmaxf(M, __ldcg(base + pc * slot_floats + hh));
                        float Ls = 0.f;
                        float4 As = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (M != -INFINITY) {
                            for (int pc = 0; pc < r.pieces; ++pc) {
                                const float *pp = base + pc * slot_floats;
                                const float mc = __ldcg(pp + hh);
                                const float w = (mc == -INFINITY) ? 0.f : fast_exp2(mc - M);
                                Ls += __ldcg(pp + NQ + hh) * w;
                                const float4 a4 = __ldcg(reinterpret_cast<const float4 *>(pp + 2 * NQ + hh * D) + d4);
                                As.x += a4.x * w;
                                As.y += a4.y * w;
                                As.z += a4.z * w;
                                As.w += a4.w * w;
                            }
                        }
                        const float inv = Ls > 0.f ? 1.0f / (Ls + a.norm_eps) : 0.f;
                        __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(a.out) +
                                             qo_row(r.s, r.h, hh, Hkv, NQ, a.qfold, a.seq_div) * D + 4 * d4;
                        *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2<__nv_bfloat16>(As.x * inv, As.y * inv),
                                                                     pack2<__nv_bfloat16>(As.z * inv, As.w * inv));
                    }
                    if (ctid == 0) atomicExch(&a.counters[unit], 0);
                }
            }
#pragma unroll
            for (int j = 0; j < NQ; ++j) lp[j] = 0.f;
            named_barrier(1, 128);  // every thread is done with this run's references
            if (ctid < kPtN) sm_mref[ctid] = -INFINITY;
            stage_next_q();  // (its barrier publishes the reset)
        }
    }

    // ------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kPtCols);
}

}  // namespace gk
