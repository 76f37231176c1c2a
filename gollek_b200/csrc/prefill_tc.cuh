// prefill_tc.cuh -- multi-query paged attention (the queries of a prefill chunk, or
// speculative tokens, over the paged cache), and decode with 32 or 64 q heads per kv head,
// on the 5th-generation tensor cores, for bf16 KV and bf16 q with head_dim 128.
//
// The rows of a (chunk or sequence, kv-head) unit -- F queries x G heads folded, or the G
// heads of one query; NQ = 32 or 64 of them (qo_row, decode_common.cuh) -- are the M rows
// of both MMAs, so one thread owns one row: its exponent reference and
// normaliser stay in its registers, with no cross-thread reduction, and the values
// accumulate in tensor memory over the whole run:
//
//   S[128 rows x 128 tok] = Q[128 rows x 128 d] . K[128 tok x 128 d]^T   (S[tile & 1])
//   O[128 rows x 128 d]  += P[128 rows x 128 tok] . V[128 tok x 128 d]   (one O per run)
//
// Q and P are K-major operands of NQ real rows; rows NQ..127 are padding that the MMAs
// read from whatever follows the real rows in shared memory and whose results nobody
// reads.  K is the score MMA's K-major B operand and V the value MMA's MN-major B
// operand, as tc_tiles.cuh lays them out.
//
// The exponent reference is lazy: a tile's probabilities are taken against the row's
// current reference in one pass, and only when a score passes it by more than
// 2^kPtLazyMax does the warp move it, rescale its rows of O in tensor memory (once the
// previous tile's value MMAs are complete) and do the tile again.
//
// Work: the stream-K ranges and 128-token tiles of tc_tiles.cuh.  One CTA per SM, 8 warps
// (warp w runs on SM sub-partition w % 4 and reads tensor-memory lanes 32 (w % 4) ..):
//   warp 2 K producer, warp 7 V producer (tc_producer);
//   warp 3 allocates tensor memory; lane 0 issues the score MMAs;
//   warp 6 lane 0 issues the value MMAs (overwriting O at a run's first tile);
//   warps 4 .. 4 + NQ/32 - 1 (tensor-memory lane quarters 0, 1): row threads, whose
//     sub-partitions hold no producer or issuer;
//   warps 0, 1: zero the outputs of empty sequences; then (HALVES) warps 0 .. NQ/32 - 1
//     take the second half of the rows' tokens, and the remaining warps idle.
// The row warps never wait for one another: each arrives on the barriers the MMA issuers
// wait for, and at a run's end each writes its own rows (a split run's last arriving warp
// merges all rows).  Every wait is bounded and gives up once another warp has given up;
// tensor memory is released only after both MMA issuers have drained.
//
// HALVES (the default; GOLLEK_PREFILL_TC_HALVES=0: off): two warps per 32 rows on the same SM
// sub-partition, warp 4 + i taking tokens 0-63 of every tile and warp i tokens 64-127,
// each with its own exponent reference, normaliser and O accumulator in tensor memory
// (columns 256-383 and 384-511), so a tile's softmax pass is split over two warps whose
// latencies overlap.  At a run's end warp i hands its (reference, normaliser) through
// shared memory and warp 4 + i merges the two halves of its rows.  Warps 0 and 1 zero the
// empty outputs before their rows.
#pragma once

#include <type_traits>

#include "tc_tiles.cuh"

namespace gk {

constexpr int kPtThreads = 256;
constexpr uint32_t kPtCols = 512;  // S x2 (128 columns each), O (128; HALVES: two of them)

// Waits suspend the waiting thread until the phase completes (up to this long per test),
// which leaves the issue slots and the shared-memory pipe to the MMA issue, tensor-memory
// loads and stores of the working warps (measured against polling with 256 / 512 ns
// sleeps: 0.503 against 0.527 / 0.514 ms at Tq = 16).
constexpr uint32_t kPtSuspendNs = kSuspendNs;

// Scores may exceed their row's exponent reference by this much (log2 units) before the
// reference moves: probabilities stay below 2^8, far inside bf16 and fp32.
constexpr float kPtLazyMax = 8.f;

struct PtSmem {
    uint32_t q, p, kring, vring, prefix, cprefix, lens, rstart, misc, ml, bars, total;
};

// q [slab] and P [buffer][slab]: NQ rows of 128 bytes each, 1 KB aligned; the padding rows
// of the last q slab read into P, those of the last P slab into the K ring.  halves: the
// second-half warps' (reference, normaliser) per row and their two hand-over barriers.
__host__ __device__ inline PtSmem pt_smem_layout(int nq, int kst, int vst, int num_seqs, int num_ctas,
                                                 bool halves = false) {
    PtSmem L;
    const uint32_t slab = static_cast<uint32_t>(nq) * 128;
    uint32_t o = 0;
    L.q = o;
    o += 2 * slab;
    L.p = o;
    o += 4 * slab;
    L.kring = o;
    o += kst * kTcTile;
    L.vring = o;
    o += vst * kTcTile;
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
    L.ml = o;
    o += halves ? 2 * nq * 4 : 0;
    L.bars = o;
    o += (2 * kst + 2 * vst + 12 + (halves ? 2 : 0)) * 8;
    L.total = o + 1024;  // slack to align the base to 1024 bytes
    return L;
}

template <int NQ, bool HALVES = false>
__global__ void __launch_bounds__(kPtThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const DecodeArgs a) {
    constexpr int D = 128;
    constexpr int NW = NQ / 32;           // row warps (per token half with HALVES)
    constexpr int NRW = HALVES ? 2 * NW : NW;
    constexpr uint32_t kSlab = NQ * 128;  // one operand slab: NQ rows x 64 columns
    static_assert(NQ == 32 || NQ == 64, "rows per unit");
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int NK = a.num_stages;
    const int NV = a.num_vstages;
    const PtSmem L = pt_smem_layout(NQ, NK, NV, a.num_seqs, gridDim.x, HALVES);
    const uint32_t q_s = smem_u32(smem + L.q);
    const uint32_t p_s = smem_u32(smem + L.p);
    uint8_t *sm_kring = smem + L.kring;
    uint8_t *sm_vring = smem + L.vring;
    int *sm_prefix = reinterpret_cast<int *>(smem + L.prefix);
    int *sm_cprefix = reinterpret_cast<int *>(smem + L.cprefix);
    int *sm_len = reinterpret_cast<int *>(smem + L.lens);
    long long *sm_rstart = reinterpret_cast<long long *>(smem + L.rstart);
    // [1] max groups of a sequence, [2] tensor-memory base, [3] abort
    volatile int *sm_misc = reinterpret_cast<volatile int *>(smem + L.misc);
    volatile int *abort = &sm_misc[3];
    uint64_t *k_full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *k_empty = k_full + NK;
    uint64_t *v_full = k_empty + NK;
    uint64_t *v_empty = v_full + NV;
    uint64_t *s_full = v_empty + NV;  // [2] scores in tensor memory
    uint64_t *s_free = s_full + 2;    // [2] scores read by the row warps
    uint64_t *p_full = s_free + 2;    // [2] probabilities written (and O rescaled)
    uint64_t *o_done = p_full + 2;    // [2] a tile's value MMAs complete
    uint64_t *o_free = o_done + 2;    // [1] O read at a run's end
    uint64_t *q_full = o_free + 1;    // [1] q staged
    uint64_t *mma_done = q_full + 1;  // [2] score and value issuers drained
    uint64_t *ml_full = mma_done + 2; // HALVES [NW]: second-half (reference, normaliser) written
    float *sm_ml = reinterpret_cast<float *>(smem + L.ml);  // HALVES: [2][NQ]

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
            mbar_init(&s_free[i], NRW);
            mbar_init(&p_full[i], NRW);
            mbar_init(&o_done[i], 1);
            mbar_init(&mma_done[i], 1);
        }
        mbar_init(o_free, NW);
        mbar_init(q_full, NW);
        if constexpr (HALVES)
            for (int i = 0; i < NW; ++i) mbar_init(&ml_full[i], 1);
        fence_barrier_init();
        sm_misc[1] = 0;
        sm_misc[3] = 0;
    }
    if ((warp == 2 || warp == 7) && lane == 0) prefetch_tensormap(warp == 2 ? &tm_k : &tm_v);
    if (warp == 3) {
        tmem_alloc(smem_u32(const_cast<int *>(&sm_misc[2])), kPtCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = static_cast<uint32_t>(sm_misc[2]);
    const uint32_t t_o = tmem + 256;  // O columns

    const Schedule sch = schedule_prologue(a, sm_prefix, sm_cprefix, sm_len, sm_rstart, &sm_misc[1],
                                           reinterpret_cast<int *>(smem + L.p));

    // tries of a suspending wait (GOLLEK_TEST_WAIT_LIMIT shortens them, as for every wait)
    const unsigned it_tries = a.wait_limit ? max(1u, a.wait_limit >> 6) : kSuspendTries;

    // Sequences with nothing to attend to: zeros, written by CTA s % grid (threads 0-63).
    auto zero_empty = [&]() {
        for (int s = blockIdx.x; s < S; s += gridDim.x) {
            if (sm_prefix[s + 1] != sm_prefix[s]) continue;
            for (int o = tid; o < Hkv * NQ * D; o += 64)
                store_out(a.out, static_cast<long long>(s) * Hkv * NQ * D + o, 0.f, 1);
        }
    };

    if (warp == 2 || warp == 7) {
        // ========================================================= producers (K: warp 2, V: warp 7)
        const bool is_k = warp == 2;
        tc_producer(a, sch, sm_len, abort, is_k ? &tm_k : &tm_v, is_k ? sm_kring : sm_vring,
                    is_k ? k_full : v_full, is_k ? k_empty : v_empty, is_k ? NK : NV, lane, kPtSuspendNs);
    } else if (warp == 3) {
        // ========================================================= score MMAs
        if (lane == 0) {
            constexpr uint32_t id_s = umma_idesc_16bit(128, kTcTokens, 1, 0, 0);
            const uint32_t k_base = smem_u32(sm_kring);
            for (TileIt is = tile_begin(sch); is.live; tile_next(sch, is)) {
                const int slot = is.ti % NK;
                const int sb = is.ti & 1;
                bool ok = mbar_wait_or_abort(&k_full[slot], (is.ti / NK) & 1, abort, it_tries, kPtSuspendNs);
                if (ok && is.ti >= 2)
                    ok = mbar_wait_or_abort(&s_free[sb], ((is.ti >> 1) + 1) & 1, abort, it_tries, kPtSuspendNs);
                if (ok && is.tg0 == 0) ok = mbar_wait_or_abort(q_full, is.ri & 1, abort, it_tries, kPtSuspendNs);
                if (!ok) {
                    *abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t kb = k_base + static_cast<uint32_t>(slot) * kTcTile;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_f16(tmem + 128 * sb, umma_desc_sw128(q_s + (kk >> 2) * kSlab + (kk & 3) * 32, 16, 1024),
                             umma_desc_sw128(kb + (kk >> 2) * 1024 + (kk & 3) * 32, 16, 2048), id_s, kk > 0);
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
            constexpr uint32_t id_o = umma_idesc_16bit(128, D, 1, 0, 1);
            const uint32_t v_base = smem_u32(sm_vring);
            for (TileIt ip = tile_begin(sch); ip.live; tile_next(sch, ip)) {
                const int slot = ip.ti % NV;
                const int sb = ip.ti & 1;
                bool ok = mbar_wait_or_abort(&p_full[sb], (ip.ti >> 1) & 1, abort, it_tries, kPtSuspendNs);
                if (ok) ok = mbar_wait_or_abort(&v_full[slot], (ip.ti / NV) & 1, abort, it_tries, kPtSuspendNs);
                if (ok && ip.tg0 == 0 && ip.ri > 0)
                    ok = mbar_wait_or_abort(o_free, (ip.ri - 1) & 1, abort, it_tries, kPtSuspendNs);
                if (!ok) {
                    *abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t vb = v_base + static_cast<uint32_t>(slot) * kTcTile;
                const uint32_t pb = p_s + static_cast<uint32_t>(2 * sb) * kSlab;
#pragma unroll
                for (int kk = 0; kk < kTcTokens / 16; ++kk) {
                    // HALVES: tokens 64-127 (kk >= 4) accumulate into the second O
                    const uint32_t t_d = HALVES ? t_o + 128u * static_cast<uint32_t>(kk >> 2) : t_o;
                    const bool acc = HALVES ? (ip.tg0 > 0 || (kk & 3) > 0) : (ip.tg0 > 0 || kk > 0);
                    umma_f16(t_d, umma_desc_sw128(pb + (kk >> 2) * kSlab + (kk & 3) * 32, 16, 1024),
                             umma_desc_sw128(vb + kk * 4096, 1024, 2048), id_o, acc ? 1u : 0u);
                }
                umma_commit(&o_done[sb]);
                umma_commit(&v_empty[slot]);
            }
            umma_commit(&mma_done[1]);
            mbar_wait(&mma_done[1], 0);
        }
        __syncwarp();
    } else if ((warp >= 4 && warp < 4 + NW) || (HALVES && warp < NW)) {
        // ========================================================= row threads
        // sec: a HALVES second-half warp (tokens 64-127 of every tile; warps 0 .. NW-1)
        const bool sec = HALVES && warp < 4;
        const int half = sec ? 1 : 0;
        if (sec) zero_empty();
        // rows 32 (warp & 3) .. + 31: warp 4 + i and (HALVES) warp i share lane quarter i
        const int c = 32 * (warp & 3) + lane;  // row = tensor-memory lane
        const uint32_t t_lane = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const uint32_t t_om = HALVES ? t_o + 128u * static_cast<uint32_t>(half) : t_o;  // this warp's O
        const int gm = NQ / a.qfold;                 // heads per query
        const int qshift = a.qfold - 1 - c / gm;     // row c's query sees the positions before len - qshift
        const unsigned wl = a.wait_limit ? max(1u, a.wait_limit >> 6) : kSuspendTries;
        const int slot_floats = 2 * NQ + NQ * D;
        const float qs = a.q_scale;
        const bool cap = a.soft_cap > 0.f;

        // q row c of the next run -> the q buffer (both 64-column slabs); called when the
        // score MMAs of the previous run have completed
        long long qx = sch.x_beg;
        auto stage_next_q = [&]() {
            if (qx >= sch.x_end) return;
            const Run rq = sch.run_at(qx);
            const uint4 *src = reinterpret_cast<const uint4 *>(
                reinterpret_cast<const __nv_bfloat16 *>(a.q) +
                qo_row(rq.s, rq.h, c, Hkv, NQ, a.qfold, a.seq_div) * D);
#pragma unroll
            for (int ch = 0; ch < 16; ++ch)
                sts_u4(q_s + (ch >> 3) * kSlab + c * 128 + ((((ch & 7) ^ (c & 7))) << 4), __ldg(src + ch));
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_full);
            qx += rq.len;
        };
        if (!sec) stage_next_q();

        // One pass over a tile's scores (tensor memory, 64 columns at a time): probabilities
        // exp2(d), d = x - mref (x: the score in the exp2 domain), of the tokens [lo, hi) as
        // bf16 into P row c, their sum, and the largest d.  MASK: some token of the tile is
        // outside [lo, hi) for some row of the warp; CAP: soft-cap.
        const uint32_t p_row = p_s + c * 128;
        auto tile_pass = [&](auto mask_t, auto cap_t, int sb, int lo, int hi, float mref, float &dmax,
                             float &ls) {
            constexpr bool MASK = decltype(mask_t)::value;
            constexpr bool CAP = decltype(cap_t)::value;
            float dm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            float lsa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int hh = 0; hh < (HALVES ? 1 : 2); ++hh) {
                const int h = HALVES ? half : hh;  // HALVES: this warp's 64 tokens only
                float v[64];
                tmem_ld<32>(tmem + 128 * sb + 64 * h + t_lane, v);
                tmem_ld<32>(tmem + 128 * sb + 64 * h + 32 + t_lane, v + 32);
                tmem_wait_ld();
                // tokens 64h .. 64h + 63 are slab h of P buffer sb: eight 16-byte chunks
                const uint32_t row = p_row + static_cast<uint32_t>(2 * sb + h) * kSlab;
#pragma unroll
                for (int q8 = 0; q8 < 8; ++q8) {
                    uint32_t pk[4];
#pragma unroll
                    for (int i2 = 0; i2 < 4; ++i2) {
                        float pe[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int i = 8 * q8 + 2 * i2 + e;
                            float d;
                            if constexpr (CAP)
                                d = a.soft_cap * tanhf(v[i] * qs / a.soft_cap) * a.post_scale - mref;
                            else
                                d = fmaf(v[i], qs, -mref);
                            if constexpr (MASK) d = (64 * h + i >= lo && 64 * h + i < hi) ? d : -INFINITY;
                            dm[i & 3] = fmaxf(dm[i & 3], d);
                            pe[e] = fast_exp2(d);
                            lsa[i & 3] += pe[e];
                        }
                        pk[i2] = pack2<__nv_bfloat16>(pe[0], pe[1]);
                    }
                    sts_u4(row + ((q8 ^ (c & 7)) << 4), make_uint4(pk[0], pk[1], pk[2], pk[3]));
                }
            }
            dmax = fmaxf(fmaxf(dm[0], dm[1]), fmaxf(dm[2], dm[3]));
            ls = (lsa[0] + lsa[1]) + (lsa[2] + lsa[3]);
        };
        auto run_pass = [&](int sb, int lo, int hi, float mref, float &dmax, float &ls) {
            // warp-uniform choice (the pass holds warp-collective tensor-memory loads)
            const bool mask = __any_sync(0xffffffffu, HALVES ? (lo > 64 * half || hi < 64 * half + 64)
                                                             : (lo > 0 || hi < kTcTokens));
            using T = std::true_type;
            using F = std::false_type;
            if (cap) {
                if (mask)
                    tile_pass(T{}, T{}, sb, lo, hi, mref, dmax, ls);
                else
                    tile_pass(F{}, T{}, sb, lo, hi, mref, dmax, ls);
            } else {
                if (mask)
                    tile_pass(T{}, F{}, sb, lo, hi, mref, dmax, ls);
                else
                    tile_pass(F{}, F{}, sb, lo, hi, mref, dmax, ls);
            }
        };
        // the largest score (exp2 domain) of row c among the tile's tokens [lo, hi), -inf if
        // none (the soft-cap is increasing, so it is applied to the largest product)
        auto tile_max = [&](int sb, int lo, int hi) {
            float m = -INFINITY;
#pragma unroll 1
            for (int k = HALVES ? 2 * half : 0; k < (HALVES ? 2 * half + 2 : 4); ++k) {
                float v[32];
                tmem_ld<32>(tmem + 128 * sb + 32 * k + t_lane, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (32 * k + i >= lo && 32 * k + i < hi) m = fmaxf(m, v[i] * qs);
            }
            if (cap && m != -INFINITY) m = a.soft_cap * tanhf(m / a.soft_cap) * a.post_scale;
            return m;
        };
        float m_run = -INFINITY;  // exponent reference of row c (lazy running max; -inf: none yet)
        float l_run = 0.f;        // normaliser of row c relative to m_run
        bool bad = false;         // a wait of this warp gave up
        for (TileIt it = tile_begin(sch); it.live;) {
            const int ti = it.ti;
            [[maybe_unused]] const int ri = it.ri;  // run index within this CTA (HALVES hand-over)
            const int sb = ti & 1;
            const Run r = it.r;
            const int ng = min(kTcGroups, r.len - it.tg0);
            const bool run_end = it.tg0 + kTcGroups >= r.len;
            const int len = sm_len[r.s];
            const int ws = tc_win_start(a, len);
            const int t0 = (ws / kRows + r.g + it.tg0) * kRows;  // position of the tile's token 0
            // row c attends to the tile's tokens [lo, hi); V rows outside [lo, vhi) -- no row's --
            // are cleared (a zero probability does not cancel a NaN on the tensor pipe)
            const int lo = max(ws - t0, 0);
            const int vhi = min(len - t0, ng * kRows);
            const int hi = min(vhi, len - qshift - t0);
            bool ok = warp_wait(&s_full[sb], (ti >> 1) & 1, wl, abort, kPtSuspendNs);
            // the probability buffer is free once the value MMAs of tile ti - 2 completed
            if (ok && ti >= 2) ok = warp_wait(&o_done[sb], ((ti - 2) >> 1) & 1, wl, abort, kPtSuspendNs);
            if (!ok) {
                bad = true;
                break;
            }
            tc_fence_after();
            // ---------------- probabilities against the current reference; a tile whose
            // scores pass it by more than 2^kPtLazyMax (or a row's first scores) moves it,
            // rescaling l and O, and is done again
            float dmax, ls;
            run_pass(sb, lo, hi, m_run == -INFINITY ? 0.f : m_run, dmax, ls);
            const bool need = (m_run == -INFINITY) ? dmax > -INFINITY : dmax > kPtLazyMax;
            if (__any_sync(0xffffffffu, need)) {
                const float mn = fmaxf(m_run, tile_max(sb, lo, hi));
                const float alpha = (mn == m_run) ? 1.f : fast_exp2(m_run - mn);
                m_run = mn;
                l_run *= alpha;
                if (it.tg0 > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    // O holds this run's earlier tiles: once the previous tile's value MMAs
                    // are complete, scale row c's O by alpha
                    if (!warp_wait(&o_done[(ti - 1) & 1], ((ti - 1) >> 1) & 1, wl, abort, kPtSuspendNs)) {
                        bad = true;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) {
                        float o[32];
                        tmem_ld<32>(t_om + 32 * k + t_lane, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(t_om + 32 * k + t_lane, o);
                    }
                    tmem_wait_st();
                }
                run_pass(sb, lo, hi, m_run == -INFINITY ? 0.f : m_run, dmax, ls);
            }
            l_run += ls;
            if (!sec && (lo > 0 || vhi < kTcTokens)) {
                // clear V rows [0, lo) and [vhi, 128) once the tile's V copies have landed
                const int vslot = ti % NV;
                if (!warp_wait(&v_full[vslot], (ti / NV) & 1, wl, abort, kPtSuspendNs)) {
                    bad = true;
                    break;
                }
                const uint32_t vt = smem_u32(sm_vring) + static_cast<uint32_t>(vslot) * kTcTile;
                for (int idx = c; idx < kTcTokens * 16; idx += NQ) {
                    const int j = idx >> 4;
                    if (j < lo || j >= vhi) sts_u4(vt + tile_chunk_off(j, idx & 15), make_uint4(0, 0, 0, 0));
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

            if constexpr (HALVES) {
                if (sec) {
                    // second half: hand (reference, normaliser) of row c to warp 4 + (warp & 3)
                    // (read before it stages the next run's q, so before this warp's
                    // next run can end and write them again)
                    sm_ml[c] = m_run;
                    sm_ml[NQ + c] = l_run;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ml_full[warp & 3]);
                    m_run = -INFINITY;
                    l_run = 0.f;
                    continue;
                }
            }
            // ---------------- end of the run: row c of O, normalised, out
            if (!warp_wait(&o_done[sb], (ti >> 1) & 1, wl, abort, kPtSuspendNs)) {
                bad = true;
                break;
            }
            // HALVES: the two halves of row c against their common maximum mm
            float mm = m_run, lsum = l_run;
            [[maybe_unused]] float fa = 1.f, fb = 0.f;
            if constexpr (HALVES) {
                if (!warp_wait(&ml_full[warp & 3], ri & 1, wl, abort, kPtSuspendNs)) {
                    bad = true;
                    break;
                }
                const float mb = sm_ml[c], lb = sm_ml[NQ + c];
                mm = fmaxf(m_run, mb);
                fa = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mm);
                fb = mb == -INFINITY ? 0.f : fast_exp2(mb - mm);
                lsum = l_run * fa + lb * fb;
            }
            tc_fence_after();
            const long long unit = static_cast<long long>(r.s) * Hkv + r.h;
            float *part = a.partials + (unit * kMaxSplits + r.piece) * slot_floats;
            const long long out_row = qo_row(r.s, r.h, c, Hkv, NQ, a.qfold, a.seq_div) * D;
            const float inv = lsum > 0.f ? 1.0f / (lsum + a.norm_eps) : 0.f;
#pragma unroll 1
            for (int k = 0; k < 4; ++k) {
                float o[32];
                tmem_ld<32>(t_o + 32 * k + t_lane, o);
                if constexpr (HALVES) {
                    float ob[32];
                    tmem_ld<32>(t_o + 128 + 32 * k + t_lane, ob);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], fa, ob[i] * fb);
                } else {
                    tmem_wait_ld();
                }
                if (r.pieces == 1) {
                    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(a.out) + out_row + 32 * k);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        dst[q4] = make_uint4(pack2<__nv_bfloat16>(o[8 * q4] * inv, o[8 * q4 + 1] * inv),
                                             pack2<__nv_bfloat16>(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv),
                                             pack2<__nv_bfloat16>(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv),
                                             pack2<__nv_bfloat16>(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv));
                } else {
                    float4 *dst = reinterpret_cast<float4 *>(part + 2 * NQ + c * D + 32 * k);
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4)
                        dst[q4] = make_float4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            if (r.pieces > 1) {
                // Each row warp of each piece arrives on the unit's counter once its rows of
                // the partial are written; the last of the pieces x NW arrivals merges all
                // rows (log-sum-exp), so no warp waits for another.
                part[c] = mm;
                part[NQ + c] = lsum;
                __threadfence();
                __syncwarp();
                int old = 0;
                if (lane == 0) old = atomicAdd(&a.counters[unit], 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == r.pieces * NW - 1) {
                    __threadfence();
                    const float *base = a.partials + unit * kMaxSplits * slot_floats;
                    // lane l takes head-dim columns 4l .. 4l + 3 of every row; four rows at a
                    // time so their loads are in flight together
                    for (int h0 = 0; h0 < NQ; h0 += 4) {
                        float M[4], Ls[4];
                        float4 As[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            M[u] = -INFINITY;
                            Ls[u] = 0.f;
                            As[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                        for (int pc = 0; pc < r.pieces; ++pc)
#pragma unroll
                            for (int u = 0; u < 4; ++u) M[u] = fmaxf(M[u], __ldcg(base + pc * slot_floats + h0 + u));
                        for (int pc = 0; pc < r.pieces; ++pc) {
                            const float *pp = base + pc * slot_floats;
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const float mc = __ldcg(pp + h0 + u);
                                const float f = (mc == -INFINITY || M[u] == -INFINITY) ? 0.f : fast_exp2(mc - M[u]);
                                Ls[u] += __ldcg(pp + NQ + h0 + u) * f;
                                const float4 a4 = __ldcg(reinterpret_cast<const float4 *>(pp + 2 * NQ + (h0 + u) * D) + lane);
                                As[u].x += a4.x * f;
                                As[u].y += a4.y * f;
                                As[u].z += a4.z * f;
                                As[u].w += a4.w * f;
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float iu = Ls[u] > 0.f ? 1.0f / (Ls[u] + a.norm_eps) : 0.f;
                            __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(a.out) +
                                                 qo_row(r.s, r.h, h0 + u, Hkv, NQ, a.qfold, a.seq_div) * D + 4 * lane;
                            *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2<__nv_bfloat16>(As[u].x * iu, As[u].y * iu),
                                                                         pack2<__nv_bfloat16>(As[u].z * iu, As[u].w * iu));
                        }
                    }
                    if (lane == 0) atomicExch(&a.counters[unit], 0);
                }
            }
            m_run = -INFINITY;
            l_run = 0.f;
            stage_next_q();
        }
        if (bad && lane == 0) *abort = 1;
    } else if (warp < 2) {
        // ========================================================= warps 0, 1 (not rows)
        zero_empty();
    }

    // ------------------------------------------------------------ teardown
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 3) tmem_dealloc(tmem, kPtCols);
}

}  // namespace gk
