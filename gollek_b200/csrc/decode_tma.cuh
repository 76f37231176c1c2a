// decode_tma.cuh -- persistent, warp-specialised paged decode attention for sm_100a.
//
// Work: the unit is a group of ROWS tokens of one (sequence, kv-head): 16, or 32 for
// int8 KV with bf16 q and pages of >= 16 tokens (a stage then carries as many bytes as
// a 16-bit one and the per-group costs are paid half as often).  The prologue of every
// CTA derives, from the context lengths, the linear order of all groups
// (sequence-major, then kv-head, then position) and cuts it into gridDim.x contiguous
// ranges of equal cost (stream-K style): every CTA moves about the same number of KV
// bytes, whatever the length mix.  A range covers runs of consecutive groups of one
// (sequence, kv-head); a run that does not cover its whole (sequence, kv-head) is a
// split-K piece.
//
// One CTA = NC consumer warps + 1 producer warp, one CTA per SM.
//   Producer: works in lane-parallel waves of up to 32 groups, one stage per lane:
//   each lane reads its group's block-table entries (two waves ahead), polls its
//   stage's empty mbarrier (non-blocking) and issues TMA tile loads (SWIZZLE_128B, this
//   CTA only) of the group's K and V rows, completing on the stage's full mbarrier;
//   int8 scales come by bulk copy, through registers (per page) or by 4-byte cp.async.
//   (Measured: waves beat per-lane rolling ownership, whose lanes then look up their
//   next groups one at a time, divergently.)
//   Consumer warp w owns a ring of SPW stages and takes groups w, w+NC, ... of the
//   CTA's sequence of groups.  Owning its stages means a warp waits on each stage
//   barrier in phase order, so parity waits cannot alias.
//   (FFMA consumer, fp32 KV.)  Score pass: lane l handles token l%16 over head-dim half l/16 against the G
//   query heads of the GQA group (q staged as fp32 in shared memory, broadcast
//   reads), packed fp32x2 FMAs, halves joined by one shuffle.  Online softmax in the
//   exp2 domain.  Value pass: lanes 0-15 take even rows and 16-31 odd rows, each lane
//   owning head_dim/16 columns for all G heads.
//   At a run's end the NC warp states merge through shared memory; a whole
//   (sequence, kv-head) writes its output, a piece writes an fp32 partial (m, l, acc),
//   and the CTA completing the last piece merges all of them (log-sum-exp) and
//   resets the arrival counter, so the scratch stays zeroed between calls.
//
// Stage layout: 128-byte-wide column slabs of ROWS rows; 16-byte chunk c of
// row r sits at chunk position c ^ (r & 7), which is what TMA's 128-byte swizzle
// writes.  The 8 lanes of a quarter-warp read 8 rows of one logical chunk, or 8
// chunks of one row: 8 distinct bank groups either way.
#pragma once

#include <type_traits>

#include "decode_common.cuh"

#ifndef GK_WAVE
#define GK_WAVE 32
#endif
#ifndef GK_POLL_SLEEP_NS
#define GK_POLL_SLEEP_NS 20  // producer's sleep between polls of busy stages
#endif

namespace gk {

template <typename KV>
struct KvType;
template <>
struct KvType<__nv_bfloat16> {
    static constexpr int kBytes = 2;
    static constexpr bool kQuant = false;
};
template <>
struct KvType<__half> {
    static constexpr int kBytes = 2;
    static constexpr bool kQuant = false;
};
template <>
struct KvType<float> {
    static constexpr int kBytes = 4;
    static constexpr bool kQuant = false;
};
template <>
struct KvType<int8_t> {
    static constexpr int kBytes = 1;
    static constexpr bool kQuant = true;
};

// Decode 4 bytes of KV elements into floats (the CUDA-core consumer reads fp32 KV).
template <typename KV>
__device__ __forceinline__ void decode_word(uint32_t w, float *f);
template <>
__device__ __forceinline__ void decode_word<float>(uint32_t w, float *f) {
    f[0] = __uint_as_float(w);
}

// c += A(16x16, row) * B(16x8, col) with fp32 accumulation.
template <typename KV>
__device__ __forceinline__ void mma_16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    if constexpr (std::is_same<KV, __half>::value)
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
            "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
            "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four signed bytes -> two f16x2 words holding the integers 1152 + b exactly: byte b
// becomes the f16 1024 + (b ^ 0x80) (0x64 exponent byte over the biased byte as
// mantissa).  lo = bytes 0, 1; hi = bytes 2, 3 (lower byte in the low half).  A dot
// product over these carries 1152 times the sum of the other operand, which the caller
// removes once in fp32.
__device__ __forceinline__ void i8x4_to_f16x2_biased(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;
    lo = __byte_perm(u, 0x64646464u, 0x4140);
    hi = __byte_perm(u, 0x64646464u, 0x4342);
}

// 2^e as a float, exact, for e in [-126, 127].
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((127 + e) << 23); }

// Scores may exceed the running max used as the exponent reference by this much (log2
// units) before the reference moves.
constexpr float kLazyMax = 8.f;

// Unbiased exponent of a positive finite float (x in [2^e, 2^(e+1))); normals only.
__device__ __forceinline__ int exp_of(float x) { return static_cast<int>((__float_as_uint(x) >> 23) & 0xffu) - 127; }

// Byte offset in a swizzled stage tile (slabs of ROWS rows) of byte `b` of row `r`.
template <int ROWS = kRows>
__device__ __forceinline__ uint32_t swz(int r, int b) {
    return static_cast<uint32_t>((b >> 7) * (ROWS * 128) + r * 128 +
                                 ((((b >> 4) & 7) ^ (r & 7)) << 4) + (b & 15));
}

// q row layout in shared memory: each head's D floats with 4 floats of padding after
// every 64, so the two head-dim halves of the score pass sit in different banks.
__host__ __device__ constexpr int q_off(int D, int hh, int d) {
    return hh * (D + 4 * (D / 64)) + d + 4 * (d / 64);
}

// Shared-memory carve-up, identical on host and device.
struct DecodeSmem {
    uint32_t stages, q, p, comb, scales, prefix, cprefix, lens, rstart, misc, bars, total;
};

__host__ __device__ inline DecodeSmem decode_smem_layout(int kv_bytes, bool quant, int D, int G,
                                                         int NC, int stages, int num_seqs,
                                                         int num_ctas, int rows) {
    DecodeSmem L;
    const uint32_t tile = static_cast<uint32_t>(D * kv_bytes / 128) * rows * 128;
    uint32_t o = 0;
    L.stages = o;
    o += stages * 2 * tile;
    L.q = o;
    o += align_up(G * (D + 4 * (D / 64)) * 4, 16);
    L.p = o;
    o += NC * rows * align_up(G, 4) * 4;
    L.comb = o;
    o += NC * G * (D + 2) * 4;
    o = align_up(o, 16);  // int8 scale slots take 16-byte bulk copies
    L.scales = o;
    o += quant ? stages * 2 * rows * 4 : 0;
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
    o += stages * 2 * 8;
    L.total = o + 1024;  // slack to align the base to 1024 bytes
    return L;
}

// SPLIT (tensor-pipe consumers): q is wider than the MMA type (fp32 q, or any q with
// f16 KV or int8 KV) and enters the score MMA as hi + lo halves.  ROWS: tokens per
// group and stage (32 only for int8 KV; the launch sets DecodeArgs::group_rows to it).
// PAIR (int8, 16-token pages, 32-token groups): the unit is a (sequence, kv-head pair) and a
// stage holds both heads of each page -- one 4 KB TMA box per page instead of two 2 KB ones
// (the copy path's rate is set by boxes, not bytes, for boxes this small).  Consumer warps
// 2i and 2i+1 share stage ring i, each computing one head of the pair over the same groups;
// a unit's output rows are its two heads' G rows each (a.num_kv_heads counts pairs).
template <typename KV, int D, int G, int NC, bool SPLIT, int ROWS = kRows, bool PAIR = false>
__global__ void __launch_bounds__((NC + 1) * 32, 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
    constexpr int KB = KvType<KV>::kBytes;
    constexpr bool QUANT = KvType<KV>::kQuant;
    constexpr bool I8MMA = std::is_same<KV, int8_t>::value && D == 128;  // int8 on the tensor pipe
    constexpr int HP = PAIR ? 2 : 1;         // kv-heads per unit and stage
    constexpr int UG = G * HP;               // output rows per unit
    constexpr int NP = NC / HP;              // stage-ring owners (warp pairs in PAIR mode)
    constexpr int TROWS = ROWS * HP;         // rows of one K (or V) stage tile
    constexpr int ROW_BYTES = D * KB;
    constexpr int NSLAB = ROW_BYTES / 128;
    constexpr int SLAB = TROWS * 128;        // bytes of one 128-byte column slab
    constexpr int TILE = NSLAB * SLAB;
    constexpr int HALF_CH = ROW_BYTES / 32;  // 16-byte chunks per head-dim half
    constexpr int EPC = 16 / KB;             // elements per chunk
    constexpr int EPW = 4 / KB;              // elements per 32-bit word
    constexpr int EPL = D / 16;              // value-pass columns per lane
    constexpr int LANE_BYTES = EPL * KB;     // value-pass bytes per lane per row
    constexpr int GP = (G + 3) / 4 * 4;      // p row stride (floats)
    constexpr int QROW = D + 4 * (D / 64);
    constexpr int CONS = NC * 32;
    static_assert(ROW_BYTES % 128 == 0, "row must be a whole number of 128-byte slabs");
    static_assert(EPL % 2 == 0 && EPC % 4 == 0 && D % 64 == 0, "vector widths");
    static_assert(NSLAB * 2 * 2 <= 32, "TMA loads of one stage (<= 2 pages) fit a warp");
    static_assert(ROWS == kRows || (I8MMA && ROWS == 32), "32-token groups: int8 KV only");
    static_assert(!PAIR || (I8MMA && ROWS == 32 && NC % 2 == 0 && !SPLIT), "pairs: int8, 32-token groups");

    extern __shared__ __align__(16) uint8_t smem_raw[];
    // Align to 1024 bytes by pointer arithmetic on the shared array (keeps the
    // shared address space visible to the compiler).
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const DecodeSmem L =
        decode_smem_layout(KB, QUANT, D, G, NC, a.num_stages, a.num_seqs, gridDim.x, TROWS);
    uint8_t *sm_stage = smem + L.stages;
    float *sm_q = reinterpret_cast<float *>(smem + L.q);
    float *sm_p = reinterpret_cast<float *>(smem + L.p);
    float *sm_comb = reinterpret_cast<float *>(smem + L.comb);
    float *sm_scale = reinterpret_cast<float *>(smem + L.scales);
    int *sm_prefix = reinterpret_cast<int *>(smem + L.prefix);
    int *sm_cprefix = reinterpret_cast<int *>(smem + L.cprefix);  // per-sequence cost prefix
    int *sm_len = reinterpret_cast<int *>(smem + L.lens);  // context lengths, clamped to the table
    long long *sm_rstart = reinterpret_cast<long long *>(smem + L.rstart);  // CTA range starts
    volatile int *sm_misc = reinterpret_cast<volatile int *>(smem + L.misc);
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty_bar = full_bar + a.num_stages;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int S = a.num_seqs;
    const int Hkv = a.num_kv_heads;
    const int NS = a.num_stages;
    const int SPW = NS / NP;
    const unsigned wait_limit = a.wait_limit ? a.wait_limit : kWaitLimit;
    const unsigned poll_limit = a.wait_limit ? a.wait_limit : kPollLimit;
    auto stage_of = [&](int gi) { return (gi % NP) * SPW + (gi / NP) % SPW; };
    auto round_of = [&](int gi) { return (gi / NP) / SPW; };

    // ------------------------------------------------------------ prologue
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full_bar[i], (QUANT && a.scale_mode == 2) ? 2 : 1);
            mbar_init(&empty_bar[i], HP);  // every warp of the ring's owner releases
        }
        fence_barrier_init();
        sm_misc[0] = 0;  // "this CTA merges the partials" flag
        sm_misc[1] = 0;  // max groups of one sequence (reduction)
        sm_misc[3] = 0;  // consumer abort flag
    }
    if (warp == NC && lane == 0) {
        prefetch_tensormap(&tm_k);
        prefetch_tensormap(&tm_v);
    }
    __syncthreads();

    const Schedule sch = schedule_prologue(a, sm_prefix, sm_cprefix, sm_len, sm_rstart, &sm_misc[1],
                                           reinterpret_cast<int *>(sm_comb));
    const long long x_beg = sch.x_beg;
    const long long x_end = sch.x_end;
    auto run_at = [&](long long x) { return sch.run_at(x); };
    auto run_pieces = [&](Run &r) { sch.pieces(r); };

    if (warp == NC) {
        // ========================================================= producer
        // Lane-parallel waves: lane i of a wave owns CTA-local group gbase + i, one
        // stage per lane (wave size <= number of stages).  Each lane waits for its own
        // stage to be free and issues its own TMA loads, without waiting for the other
        // lanes.  The next wave's page ids are looked up (block-table loads in flight)
        // while the current wave waits and issues, so a wave starts with its ids ready.
        const int R = a.block_size < ROWS ? a.block_size : ROWS;  // token rows of a page in a group
        const int npg = ROWS / R;                                 // pages per stage (<= 2)
        const int RB = R * HP;                                    // rows per TMA box (both heads)
        const int W = NS < GK_WAVE ? NS : GK_WAVE;  // groups per producer wave
        struct GroupLoc {
            int h, t0, row_off, pid0, pid1, stage, round, len, win_start, gi;
            unsigned loaded;
            float ks[2 * HP], vs[2 * HP];  // per-(page, head) int8 scales of the group's pages
        };
        auto locate_group = [&](long long x, int gi) {
            GroupLoc q;
            const Run r = run_at(x);
            const int len = sm_len[r.s];
            q.len = len;
            q.win_start = (a.window > 0 && len > a.window) ? len - a.window : 0;
            q.h = r.h;
            q.stage = stage_of(gi);
            q.round = round_of(gi);
            q.gi = gi;
            q.t0 = (q.win_start / ROWS + r.g) * ROWS;
            const int p_first = q.t0 / a.block_size;
            q.row_off = a.block_size < ROWS ? 0 : q.t0 % a.block_size;
            const int pages_in_seq = (len + a.block_size - 1) / a.block_size;
            const int *bt = a.block_tables + static_cast<long long>(r.s / a.seq_div) * a.max_blocks;
            q.pid0 = q.pid1 = 0;
            q.loaded = 0;
            for (int j = 0; j < npg; ++j) {
                const int pg = p_first + j;
                if (pg < pages_in_seq && (pg + 1) * a.block_size > q.win_start) {
                    const int e = __ldg(bt + pg);
                    if (j)
                        q.pid1 = e;
                    else
                        q.pid0 = e;
                    q.loaded |= 1u << j;
                }
            }
            return q;
        };
        auto checked = [&](int e) {
            if (e < 0 || (a.num_blocks > 0 && e >= a.num_blocks)) {
                raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
                return 0;
            }
            return e;
        };
        // Per-page int8 scales go through registers: loaded one wave ahead of their
        // wave's issue and stored to the stage's scale slots before the barrier is armed.
        const bool page_scales = QUANT && a.scale_mode == 1;
        auto load_scales = [&](GroupLoc &q, bool act) {
            if constexpr (QUANT) {
                if (!page_scales || !act) return;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (j >= npg || !((q.loaded >> j) & 1)) continue;
#pragma unroll
                    for (int hh = 0; hh < HP; ++hh) {
                        const long long so =
                            static_cast<long long>(checked(j ? q.pid1 : q.pid0)) * a.scale_page_stride +
                            static_cast<long long>(q.h * HP + hh) * a.scale_head_stride;
                        q.ks[j * HP + hh] = __ldg(a.k_scales + so);
                        q.vs[j * HP + hh] = __ldg(a.v_scales + so);
                    }
                }
            }
        };
        // one group's copies into its stage (the stage is free)
        auto issue = [&](const GroupLoc &q) {
            // test-only fault injection: leave one group's stage unfilled (its consumer's
            // bounded wait then gives up; nothing else changes)
            if (a.fault_skip_group >= 0 && blockIdx.x == 0 && q.gi == a.fault_skip_group) return;
            const int stage = q.stage;
            const int pid0 = checked(q.pid0), pid1 = checked(q.pid1);
            const unsigned loaded = q.loaded;
            uint8_t *kdst = sm_stage + static_cast<uint32_t>(stage) * 2 * TILE;
            uint8_t *vdst = kdst + TILE;
            if constexpr (QUANT) {
                if (page_scales) {  // slot j * HP + hh: page j, head hh of the unit
                    float *ks = sm_scale + stage * 2 * TROWS;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        if (j >= npg || !((loaded >> j) & 1)) continue;
#pragma unroll
                        for (int hh = 0; hh < HP; ++hh) {
                            ks[j * HP + hh] = q.ks[j * HP + hh];
                            ks[TROWS + j * HP + hh] = q.vs[j * HP + hh];
                        }
                    }
                }
            }
            const uint32_t scale_tx = (QUANT && a.scale_mode == 0) ? 2u * RB * 4u : 0u;
            mbar_arrive_expect_tx(&full_bar[stage], static_cast<uint32_t>(__popc(loaded)) *
                                                        (2u * NSLAB * RB * 128u + scale_tx));
            for (int j = 0; j < npg; ++j) {
                if (!((loaded >> j) & 1)) continue;
                const long long y = static_cast<long long>(j ? pid1 : pid0) * a.page_rows +
                                    static_cast<long long>(q.h) * HP * a.block_size + q.row_off;
                if (a.box3d) {  // ROWS rows x all slabs in one box each for K and V
                    tma_load_3d(kdst, &tm_k, 0, static_cast<int>(y), 0, &full_bar[stage]);
                    tma_load_3d(vdst, &tm_v, 0, static_cast<int>(y), 0, &full_bar[stage]);
                    continue;
                }
#pragma unroll
                for (int slab = 0; slab < NSLAB; ++slab) {
                    tma_load_2d(kdst + slab * SLAB + j * RB * 128, &tm_k, slab * (128 / KB),
                                static_cast<int>(y), &full_bar[stage]);
                    tma_load_2d(vdst + slab * SLAB + j * RB * 128, &tm_v, slab * (128 / KB),
                                static_cast<int>(y), &full_bar[stage]);
                }
            }
            if constexpr (QUANT) {
                float *ks = sm_scale + stage * 2 * TROWS;
                if (a.scale_mode == 0) {
                    // per-token scales: R contiguous floats per page and head (RB for the two
                    // heads of a pair, adjacent when the head stride is R), one bulk copy each
                    for (int j = 0; j < npg; ++j) {
                        if (!((loaded >> j) & 1)) continue;
                        const long long so = static_cast<long long>(j ? pid1 : pid0) * a.scale_page_stride +
                                             static_cast<long long>(q.h) * HP * a.scale_head_stride + q.row_off;
                        bulk_load(ks + j * RB, a.k_scales + so, RB * 4u, &full_bar[stage]);
                        bulk_load(ks + TROWS + j * RB, a.v_scales + so, RB * 4u, &full_bar[stage]);
                    }
                } else if (a.scale_mode == 2) {
                    for (int tk = 0; tk < ROWS; ++tk) {
                        const int t = q.t0 + tk;
                        const int j = tk / R;
                        if (t >= q.win_start && t < q.len && ((loaded >> j) & 1)) {
                            const long long so = static_cast<long long>(j ? pid1 : pid0) * a.scale_page_stride +
                                                 static_cast<long long>(q.h) * a.scale_head_stride +
                                                 static_cast<long long>(t % a.block_size) * a.scale_token_stride;
                            cp_async_4(ks + tk, a.k_scales + so);
                            cp_async_4(ks + TROWS + tk, a.v_scales + so);
                        }
                    }
                    cp_async_mbar_arrive_noinc(&full_bar[stage]);
                }
            }
        };
        int gbase = 0;
        bool aborted = false;
        int abort_wave = 0;         // first group of the wave that gave up
        unsigned abort_pending = 0; // its lanes whose group was never issued
        long long xw = x_beg;
        int nw = static_cast<int>(min(static_cast<long long>(W), x_end - xw));
        // cur: this wave (ids and scales ready); nxt: next wave (ids ready, scales in
        // flight); the wave after that is looked up at the top of each round.
        GroupLoc cur{}, nxt{};
        if (lane < nw) cur = locate_group(xw + lane, gbase + lane);
        load_scales(cur, lane < nw);
        long long xn = xw + nw;
        int gn = gbase + nw;
        int nw_next = static_cast<int>(min(static_cast<long long>(W), x_end - xn));
        if (lane < nw_next) nxt = locate_group(xn + lane, gn + lane);
        while (xw < x_end) {
            const long long xnn = xn + nw_next;
            const int gnn = gn + nw_next;
            const int nw_nn = static_cast<int>(min(static_cast<long long>(W), x_end - xnn));
            GroupLoc nn{};
            if (lane < nw_nn) nn = locate_group(xnn + lane, gnn + lane);
            load_scales(nxt, lane < nw_next);

            // Issue this wave: every lane polls its own stage (non-blocking, so lanes whose
            // stage is free issue at once) until all have issued.
            bool pending = lane < nw;
            bool ok = true;
            for (unsigned spins = 0;; ++spins) {
                if (pending && (cur.round == 0 || mbar_test(&empty_bar[cur.stage], (cur.round - 1) & 1))) {
                    issue(cur);
                    pending = false;
                }
                if (!__any_sync(0xffffffffu, pending)) break;
                if (spins > poll_limit) {
                    if (pending) {
                        raise_status(GOLLEK_STATUS_TIMEOUT);
                        ok = false;
                    }
                    break;
                }
#if GK_POLL_SLEEP_NS > 0
                __nanosleep(GK_POLL_SLEEP_NS);
#endif
            }
            const unsigned pend = __ballot_sync(0xffffffffu, pending);
            const int wave_first = gbase;
            xw = xn;
            gbase = gn;
            nw = nw_next;
            cur = nxt;
            xn = xnn;
            gn = gnn;
            nw_next = nw_nn;
            nxt = nn;
            if (!__all_sync(0xffffffffu, ok)) {
                aborted = true;
                abort_wave = wave_first;
                abort_pending = pend;
                break;
            }
        }
        // Let every copy already issued land before the CTA's shared memory is released:
        // consumers that gave up (their own wait, or another warp's) skip their stages, so
        // the last copy into each stage may still be in flight.  Stage s's last issued
        // group is among the last NS groups -- or, for a lane of the wave that gave up
        // before issuing, the group NS before it in the same stage (waiting on the
        // unissued group's phase would alias that copy's predecessor phase).  In a normal
        // run every such phase has completed and each wait returns at once.
        {
            const int k = lane;
            if (k < NS && k < gbase) {
                int g = gbase - 1 - k;
                if (aborted && g >= abort_wave && ((abort_pending >> (g - abort_wave)) & 1u)) g -= NS;
                if (g >= 0) mbar_wait(&full_bar[stage_of(g)], round_of(g) & 1, wait_limit);
            }
        }
        return;
    }

    // ============================================================ consumers
    // Control flow below depends only on state the consumer warps write before a
    // named barrier, so all NC warps take the same barriers.
    const int half = lane >> 4;
    const int li = lane & 15;
    const uint32_t p_base = smem_u32(sm_p) + warp * ROWS * GP * 4;
    volatile int *cons_abort = sm_misc + 3;
    const int ow = warp / HP;  // owner of this warp's stage ring
    const int hsel = warp % HP;  // PAIR: the head of the pair this warp computes

    // Sequences with nothing to attend to: zeros, written by CTA s % grid.
    for (int s = blockIdx.x; s < S; s += gridDim.x) {
        if (sm_prefix[s + 1] != sm_prefix[s]) continue;
        for (int o = tid; o < Hkv * UG * D; o += CONS)
            store_out(a.out, static_cast<long long>(s) * Hkv * UG * D + o, 0.f, a.q_bf16);
    }

    // bf16 q with bf16 KV: q's words are the score MMA's A fragments as they are, so the
    // next run's q can be loaded into registers while the current run merges.
    constexpr bool kQPrefetch = std::is_same<KV, __nv_bfloat16>::value && !SPLIT && G <= 8;
    uint32_t qnext[kQPrefetch ? D / 16 : 1][2];
    bool have_qnext = false;
    int gidx = 0;        // CTA-local index of the run's first group
    int my_slot = 0;     // this warp's next stage (of SPW) and its phase parity
    uint32_t my_phase = 0;
    for (long long x = x_beg; x < x_end;) {
        Run r = run_at(x);
        run_pieces(r);
        x += r.len;
        SeqWin sw;
        sw.len = sm_len[r.s];
        sw.win_start = (a.window > 0 && sw.len > a.window) ? sw.len - a.window : 0;
        sw.g_lo = sw.win_start / ROWS;
        sw.n = sm_prefix[r.s + 1] - sm_prefix[r.s];

        if constexpr (KB == 2) {
            // ======== 16-bit KV: dot products on the tensor pipe (mma.sync m16n8k16,
            // fp32 accumulate).  Scores S = Q K^T with the G heads as rows (padded to
            // 16); values O^T = V^T P^T with head_dim as rows, the heads as the 8
            // columns, so the probabilities go from the score accumulators straight
            // into the B operand.
            static_assert(ROWS == 16, "16-bit consumer: 16-token groups");
            static_assert(G <= 16, "16-bit consumer: at most 16 rows");
            // G = 16 (folded multi-query calls only): rows g + 8 are live too; their
            // probabilities feed a second value MMA whose 8 columns are rows 8..15.
            constexpr bool R2 = G > 8;
            constexpr int KS = D / 16;  // k-steps of the score MMA = m-tiles of the value MMA
            const int g = lane >> 2;    // fragment row group
            const int t = lane & 3;     // fragment column pair
            // q as A fragments (row g = head g; rows g+8 are zero), split hi + lo when the
            // input is wider than the MMA type so the scores stay fp32-accurate.
            uint32_t qa[KS][2], ql[SPLIT ? KS : 1][2];
            uint32_t qb[R2 ? KS : 1][2], qlb[(R2 && SPLIT) ? KS : 1][2];  // rows g + 8
            float qmul = a.q_scale;  // score multiplier (f16 KV: times the power of two taken out of q)
            if (kQPrefetch && have_qnext) {
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    qa[kk][0] = qnext[kk][0];
                    qa[kk][1] = qnext[kk][1];
                }
            } else {
                constexpr int NH = R2 ? 2 : 1;  // row halves loaded: g, and g + 8 with 16 rows
                float qx[NH][KS][2][2];
#pragma unroll
                for (int rh = 0; rh < NH; ++rh) {
                    const int gr = g + 8 * rh;
                    const long long qrow = qo_row(r.s, r.h, gr < G ? gr : 0, Hkv, G, a.qfold, a.seq_div) * D;
#pragma unroll
                    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const int d = 16 * kk + 2 * t + 8 * hf;
                            float x0 = 0.f, x1 = 0.f;
                            if (gr < G) {
                                if (a.q_bf16) {
                                    const __nv_bfloat162 v2 =
                                        *reinterpret_cast<const __nv_bfloat162 *>(
                                            reinterpret_cast<const __nv_bfloat16 *>(a.q) + qrow + d);
                                    x0 = __low2float(v2);
                                    x1 = __high2float(v2);
                                } else {
                                    const float2 v2 = *reinterpret_cast<const float2 *>(
                                        reinterpret_cast<const float *>(a.q) + qrow + d);
                                    x0 = v2.x;
                                    x1 = v2.y;
                                }
                            }
                            qx[rh][kk][hf][0] = x0;
                            qx[rh][kk][hf][1] = x1;
                        }
                    }
                }
                float down = 1.f;
                if constexpr (std::is_same<KV, __half>::value) {
                    // keep |q| below the f16 maximum: take a power of two out of q and put it
                    // back on the scores
                    float mx = 0.f;
#pragma unroll
                    for (int rh = 0; rh < NH; ++rh)
#pragma unroll
                        for (int kk = 0; kk < KS; ++kk)
#pragma unroll
                            for (int hf = 0; hf < 2; ++hf)
                                mx = fmaxf(mx, fmaxf(fabsf(qx[rh][kk][hf][0]), fabsf(qx[rh][kk][hf][1])));
                    mx = warp_max(mx);
                    const int eq = mx >= 16384.f ? min(exp_of(mx) - 14, 126) : 0;
                    down = pow2i(-eq);
                    qmul = a.q_scale * pow2i(eq);
                }
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const float x0 = qx[0][kk][hf][0] * down, x1 = qx[0][kk][hf][1] * down;
                        qa[kk][hf] = pack2<KV>(x0, x1);
                        if constexpr (SPLIT) {
                            const float2 back = unpack2<KV>(qa[kk][hf]);
                            ql[kk][hf] = pack2<KV>(x0 - back.x, x1 - back.y);
                        }
                        if constexpr (R2) {
                            const float y0 = qx[NH - 1][kk][hf][0] * down, y1 = qx[NH - 1][kk][hf][1] * down;
                            qb[kk][hf] = pack2<KV>(y0, y1);
                            if constexpr (SPLIT) {
                                const float2 back = unpack2<KV>(qb[kk][hf]);
                                qlb[kk][hf] = pack2<KV>(y0 - back.x, y1 - back.y);
                            }
                        }
                    }
                }
            }
            float m_run = -INFINITY;  // running max of head g (quad-uniform)
            float l_run = 0.f;        // this lane's share of head g's normaliser
            float o[KS][4];           // O^T fragments: d = 16*mt + g (+8), heads 2t, 2t+1
            float m_run2 = -INFINITY, l_run2 = 0.f;  // the same for row g + 8 (R2)
            float o2[R2 ? KS : 1][4];                // heads 8 + 2t, 9 + 2t (R2)
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
#pragma unroll
            for (int mt = 0; mt < (R2 ? KS : 1); ++mt) o2[mt][0] = o2[mt][1] = o2[mt][2] = o2[mt][3] = 0.f;
            // Folded multi-query rows: row g is query g / (G / qfold), which sees the
            // positions before len - qshift.
            const int qshift = (a.qfold > 1 && g < G) ? a.qfold - 1 - g / (G / a.qfold) : 0;
            const int qshift2 = (R2 && a.qfold > 1) ? a.qfold - 1 - (g + 8) / (G / a.qfold) : 0;
            // ldmatrix row address of lane: token r + 8*(i>>1), 8 columns at 8*(i&1)
            const int lm_tok = (lane & 7) + 8 * (lane >> 4);
            const int lm_col = 8 * ((lane >> 3) & 1);

            for (int j = ((ow - gidx) % NP + NP) % NP; j < r.len; j += NP) {
                const int stage = ow * SPW + my_slot;
                // every lane tests the phase (and the abort flag, read alongside); if it is
                // not complete the warp spins together (bounded), giving up early once
                // another warp has given up
                bool ok = mbar_try_wait(&full_bar[stage], my_phase) & !*cons_abort;
                if (!__all_sync(0xffffffffu, ok)) ok = warp_wait(&full_bar[stage], my_phase, wait_limit, cons_abort);
                if (++my_slot == SPW) {
                    my_slot = 0;
                    my_phase ^= 1;
                }
                if (!ok) {
                    *cons_abort = 1;
                    continue;
                }
                const uint32_t kt = smem_u32(sm_stage) + static_cast<uint32_t>(stage) * 2 * TILE;
                const uint32_t vt = kt + TILE;
                const int t0 = (sw.g_lo + r.g + j) * kRows;
                const int v_lo = max(sw.win_start - t0, 0);
                const int v_hi = min(sw.len - t0, kRows);
                if (v_lo > 0 || v_hi < kRows) {
                    // Rows outside the window may hold anything (NaN included) and a zero
                    // probability does not cancel a NaN on the tensor pipe: clear them.
                    constexpr int CHR = ROW_BYTES / 16;
                    for (int idx = lane; idx < kRows * CHR; idx += 32) {
                        const int rr = idx / CHR;
                        if (rr < v_lo || rr >= v_hi)
                            sts_u4(vt + swz(rr, (idx - rr * CHR) * 16), make_uint4(0, 0, 0, 0));
                    }
                    __syncwarp();
                }
                // ---------------- K and V fragments to registers, then free the stage at
                // once: the producer refills it while this warp computes.
                uint32_t kb[KS][4], vb[KS][4];
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    ldsm_x4(kt + swz(lm_tok, (16 * kk + lm_col) * 2), kb[kk]);
                    ldsm_x4_trans(vt + swz(lm_tok, (16 * kk + lm_col) * 2), vb[kk]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_bar[stage]);
                // ---------------- scores (two accumulator chains per n-tile)
                float s[2][4], s2[2][4];
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) s[nt][e] = s2[nt][e] = 0.f;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    float(*acc)[4] = (kk & 1) ? s2 : s;
                    const uint32_t b0 = R2 ? qb[R2 ? kk : 0][0] : 0u, b1 = R2 ? qb[R2 ? kk : 0][1] : 0u;
                    mma_16816<KV>(acc[0], qa[kk][0], b0, qa[kk][1], b1, kb[kk][0], kb[kk][1]);
                    mma_16816<KV>(acc[1], qa[kk][0], b0, qa[kk][1], b1, kb[kk][2], kb[kk][3]);
                    if constexpr (SPLIT) {
                        const uint32_t c0 = R2 ? qlb[(R2 && SPLIT) ? kk : 0][0] : 0u;
                        const uint32_t c1 = R2 ? qlb[(R2 && SPLIT) ? kk : 0][1] : 0u;
                        mma_16816<KV>(acc[0], ql[kk][0], c0, ql[kk][1], c1, kb[kk][0], kb[kk][1]);
                        mma_16816<KV>(acc[1], ql[kk][0], c0, ql[kk][1], c1, kb[kk][2], kb[kk][3]);
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < (R2 ? 4 : 2); ++e) s[nt][e] += s2[nt][e];
                // ---------------- online softmax for head g over tokens 8nt + 2t + e
                // (folded queries: row g's query sees qshift fewer positions than the last)
                const int row_hi = min(v_hi, sw.len - qshift - t0);
                float p[2][2];
                float mloc = -INFINITY;
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int tk = 8 * nt + 2 * t + e;
                        float x2 = s[nt][e];
                        if (a.soft_cap > 0.f) {
                            x2 *= qmul;
                            x2 = a.soft_cap * tanhf(x2 / a.soft_cap) * a.post_scale;
                        } else {
                            x2 *= qmul;
                        }
                        x2 = (tk >= v_lo && tk < row_hi) ? x2 : -INFINITY;
                        p[nt][e] = x2;
                        mloc = fmaxf(mloc, x2);
                    }
                // lazy running max (kLazyMax): the reference moves, and o and l are
                // rescaled, only when a score passes it by more than 2^kLazyMax
                if (__any_sync(0xffffffffu, mloc > m_run + kLazyMax)) {
                    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 1));
                    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 2));
                    const float mn = fmaxf(m_run, mloc);
                    const float alpha = (mn == m_run) ? 1.f : fast_exp2(m_run - mn);
                    m_run = mn;
                    l_run *= alpha;
                    if (__any_sync(0xffffffffu, alpha != 1.f)) {
                        const float al0 = __shfl_sync(0xffffffffu, alpha, 8 * t);      // head 2t
                        const float al1 = __shfl_sync(0xffffffffu, alpha, 8 * t + 4);  // head 2t+1
#pragma unroll
                        for (int mt = 0; mt < KS; ++mt) {
                            o[mt][0] *= al0;
                            o[mt][1] *= al1;
                            o[mt][2] *= al0;
                            o[mt][3] *= al1;
                        }
                    }
                }
                const float mref = (m_run == -INFINITY) ? 0.f : m_run;
                float psum = 0.f;
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        p[nt][e] = fast_exp2(p[nt][e] - mref);
                        psum += p[nt][e];
                    }
                l_run += psum;
                const uint32_t pb0 = pack2<KV>(p[0][0], p[0][1]);
                const uint32_t pb1 = pack2<KV>(p[1][0], p[1][1]);
                // ---------------- values
#pragma unroll
                for (int mt = 0; mt < KS; ++mt)
                    mma_16816<KV>(o[mt], vb[mt][0], vb[mt][1], vb[mt][2], vb[mt][3], pb0, pb1);
                if constexpr (R2) {
                    // ---------------- rows g + 8: the same softmax on accumulator entries
                    // 2, 3, then the value MMA for columns (heads) 8..15
                    const int row_hi2 = min(v_hi, sw.len - qshift2 - t0);
                    float p2[2][2];
                    float mloc2 = -INFINITY;
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int tk = 8 * nt + 2 * t + e;
                            float x2 = s[nt][2 + e] * qmul;
                            if (a.soft_cap > 0.f) x2 = a.soft_cap * tanhf(x2 / a.soft_cap) * a.post_scale;
                            x2 = (tk >= v_lo && tk < row_hi2) ? x2 : -INFINITY;
                            p2[nt][e] = x2;
                            mloc2 = fmaxf(mloc2, x2);
                        }
                    if (__any_sync(0xffffffffu, mloc2 > m_run2 + kLazyMax)) {
                        mloc2 = fmaxf(mloc2, __shfl_xor_sync(0xffffffffu, mloc2, 1));
                        mloc2 = fmaxf(mloc2, __shfl_xor_sync(0xffffffffu, mloc2, 2));
                        const float mn2 = fmaxf(m_run2, mloc2);
                        const float alpha2 = (mn2 == m_run2) ? 1.f : fast_exp2(m_run2 - mn2);
                        m_run2 = mn2;
                        l_run2 *= alpha2;
                        if (__any_sync(0xffffffffu, alpha2 != 1.f)) {
                            const float al0 = __shfl_sync(0xffffffffu, alpha2, 8 * t);      // head 8 + 2t
                            const float al1 = __shfl_sync(0xffffffffu, alpha2, 8 * t + 4);  // head 9 + 2t
#pragma unroll
                            for (int mt = 0; mt < KS; ++mt) {
                                o2[mt][0] *= al0;
                                o2[mt][1] *= al1;
                                o2[mt][2] *= al0;
                                o2[mt][3] *= al1;
                            }
                        }
                    }
                    const float mref2 = (m_run2 == -INFINITY) ? 0.f : m_run2;
                    float psum2 = 0.f;
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            p2[nt][e] = fast_exp2(p2[nt][e] - mref2);
                            psum2 += p2[nt][e];
                        }
                    l_run2 += psum2;
                    const uint32_t pc0 = pack2<KV>(p2[0][0], p2[0][1]);
                    const uint32_t pc1 = pack2<KV>(p2[1][0], p2[1][1]);
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt)
                        mma_16816<KV>(o2[mt], vb[mt][0], vb[mt][1], vb[mt][2], vb[mt][3], pc0, pc1);
                }
            }

            gidx += r.len;

            // ---------------- next run's q, in flight while this run merges
            if constexpr (kQPrefetch) {
                have_qnext = x < x_end;
                if (have_qnext) {
                    const Run rn = run_at(x);
                    const uint32_t *qw = reinterpret_cast<const uint32_t *>(a.q) +
                                         qo_row(rn.s, rn.h, g < G ? g : 0, Hkv, G, a.qfold, a.seq_div) * (D / 2);
#pragma unroll
                    for (int kk = 0; kk < KS; ++kk) {
                        qnext[kk][0] = g < G ? __ldg(qw + 8 * kk + t) : 0u;
                        qnext[kk][1] = g < G ? __ldg(qw + 8 * kk + 4 + t) : 0u;
                    }
                }
            }
            // ---------------- this warp's state -> shared memory
            float *cw = sm_comb + warp * G * (D + 2);
            l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
            l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
            if (t == 0 && g < G) {
                cw[g] = m_run;
                cw[G + g] = l_run;
            }
            if constexpr (R2) {
                l_run2 += __shfl_xor_sync(0xffffffffu, l_run2, 1);
                l_run2 += __shfl_xor_sync(0xffffffffu, l_run2, 2);
                if (t == 0) {
                    cw[g + 8] = m_run2;
                    cw[G + g + 8] = l_run2;
                }
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    const int d0 = 16 * mt + g;
                    cw[2 * G + (8 + 2 * t) * D + d0] = o2[mt][0];
                    cw[2 * G + (8 + 2 * t) * D + d0 + 8] = o2[mt][2];
                    cw[2 * G + (9 + 2 * t) * D + d0] = o2[mt][1];
                    cw[2 * G + (9 + 2 * t) * D + d0 + 8] = o2[mt][3];
                }
            }

#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int d0 = 16 * mt + g;
                if (2 * t < G) {
                    cw[2 * G + (2 * t) * D + d0] = o[mt][0];
                    cw[2 * G + (2 * t) * D + d0 + 8] = o[mt][2];
                }
                if (2 * t + 1 < G) {
                    cw[2 * G + (2 * t + 1) * D + d0] = o[mt][1];
                    cw[2 * G + (2 * t + 1) * D + d0 + 8] = o[mt][3];
                }
            }
        } else if constexpr (I8MMA) {
            // ======== int8 KV on the tensor pipe.  The bytes become exact f16 integers
            // 1152 + b in registers (i8x4_to_f16x2_biased) and meet q in f16 MMAs with fp32
            // accumulation; the bias is removed once in fp32 (1152 * sum(q) from each score,
            // 1152 * the probability mass from each value accumulator).
            // The per-token K scale multiplies the fp32 scores.  The V scale enters the
            // probabilities relative to a power of two 2^ev that the value accumulators
            // carry (o holds O * 2^-ev), so the f16 probabilities stay in range whatever
            // the scale; ev moves only when a group's largest scale leaves [2^(ev-2), 2^(ev+3)).
            // Head-dim order inside the MMAs: quad lane t owns dims [32t, 32t+32); k-step
            // kk takes dims 32t+4kk+{0,1,2,3} as MMA columns {2t, 2t+1, 2t+8, 2t+9}, so one
            // K word is one B fragment pair, and q is loaded in the same order.  Value rows
            // (head_dim) likewise: lane row group g owns dims [16g, 16g+16); m-tile mt row
            // g is dim 16g+2mt and row g+8 is dim 16g+2mt+1.
            // A group of ROWS tokens is NT score n-tiles of 8 tokens and VK value k-steps
            // of 16 tokens; 16-token groups keep two accumulator chains per n-tile.
            // Token sets (SETS = 2, GQA groups of <= 4 rows, q unsplit): the 8 MMA rows hold
            // the G rows twice -- rows [0, G) against the even 8-token n-tiles, rows
            // [G, 2G) against the odd ones -- by stacking the two n-tiles' K along the
            // MMA's k dimension with each row's q zero over the other set's k-steps.  A
            // score MMA then yields 2G useful rows instead of G, so every lane's
            // accumulators hold live scores and the online softmax does half the work per
            // lane; the value MMA takes the odd set's probabilities by one shuffle.
            constexpr int KS = D / 16;
            constexpr int NT = ROWS / 8;
            constexpr int VK = ROWS / 16;
            constexpr int CH = NT >= 4 ? 1 : 2;
            constexpr int SETS = (G <= 4 && !SPLIT) ? 2 : 1;
            constexpr int NTC = NT / SETS;  // score accumulator tiles (8 * SETS tokens each)
            constexpr int RU = G * SETS;    // MMA rows in use
            static_assert(D == 128, "int8 tensor-pipe path: head_dim 128");
            static_assert(NT % SETS == 0 && VK == NTC * SETS / 2, "token-set tiling");
            const int g = lane >> 2;
            const int t = lane & 3;
            const int gm = g % G;                 // row of the model (head or folded query row)
            const int myset = (g / G) % SETS;     // the n-tiles this lane's row scores
            const bool row_used = g < RU;
            const int R = a.block_size < ROWS ? a.block_size : ROWS;
            // stage row of the group's token tau (PAIR: pages of 16 rows of each head, the
            // two heads of a page adjacent, so row = 32 * page + 16 * head + slot)
            auto srow = [&](int tau) { return PAIR ? ((tau >> 4) << 5) + (hsel << 4) + (tau & 15) : tau; };
            uint32_t qa[KS][2], ql[SPLIT ? KS : 1][2];
            // the A operand of set js: this lane's q on its own set's k-steps, zero on the
            // other's (one AND per register as the MMAs are issued)
            uint32_t qmask[SETS];
#pragma unroll
            for (int js = 0; js < SETS; ++js) qmask[js] = myset == js ? 0xffffffffu : 0u;
            float qmul;         // score multiplier: q_scale times the power of two taken out of q
            float qsum = 0.f;   // head g's sum of the f16 q values the MMAs see
            {
                float qf[32];
                const long long qrow =
                    qo_row(r.s, r.h * HP + hsel, row_used ? gm : 0, Hkv * HP, G, a.qfold, a.seq_div) * D + 32 * t;
                if (row_used) {
                    if (a.q_bf16) {
                        const uint4 *src = reinterpret_cast<const uint4 *>(
                            reinterpret_cast<const __nv_bfloat16 *>(a.q) + qrow);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint4 w = __ldg(src + i);
                            qf[8 * i + 0] = bf16_lo(w.x);
                            qf[8 * i + 1] = bf16_hi(w.x);
                            qf[8 * i + 2] = bf16_lo(w.y);
                            qf[8 * i + 3] = bf16_hi(w.y);
                            qf[8 * i + 4] = bf16_lo(w.z);
                            qf[8 * i + 5] = bf16_hi(w.z);
                            qf[8 * i + 6] = bf16_lo(w.w);
                            qf[8 * i + 7] = bf16_hi(w.w);
                        }
                    } else {
                        const float4 *src = reinterpret_cast<const float4 *>(
                            reinterpret_cast<const float *>(a.q) + qrow);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 w = __ldg(src + i);
                            qf[4 * i + 0] = w.x;
                            qf[4 * i + 1] = w.y;
                            qf[4 * i + 2] = w.z;
                            qf[4 * i + 3] = w.w;
                        }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) qf[i] = 0.f;
                }
                // keep |q| below the f16 maximum: take a power of two out of q and put
                // it back on the scores
                float mx = 0.f;
#pragma unroll
                for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(qf[i]));
                mx = warp_max(mx);
                const int eq = mx >= 16384.f ? min(exp_of(mx) - 14, 126) : 0;
                const float down = pow2i(-eq);
                qmul = a.q_scale * pow2i(eq);
#pragma unroll
                for (int kk = 0; kk < KS; ++kk)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const float x0 = qf[4 * kk + 2 * hf] * down;
                        const float x1 = qf[4 * kk + 2 * hf + 1] * down;
                        const uint32_t qh = pack2<__half>(x0, x1);
                        qa[kk][hf] = qh;
                        const float2 back = unpack2<__half>(qh);
                        qsum += back.x + back.y;
                        if constexpr (SPLIT) {
                            ql[kk][hf] = pack2<__half>(x0 - back.x, x1 - back.y);
                            const float2 lo2 = unpack2<__half>(ql[kk][hf]);
                            qsum += lo2.x + lo2.y;
                        }
                    }
                qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
                qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
            }
            const float qbias = 1152.f * qsum;  // the biased K bytes add this to head g's scores
            float m_run = -INFINITY;  // running max of head g (quad-uniform)
            float l_run = 0.f;        // this lane's share of head g's normaliser
            float ps_run = 0.f;       // this lane's share of head g's probability mass in o
            // folded multi-query rows: row g's query sees the positions before len - qshift
            const int qshift = (a.qfold > 1 && row_used) ? a.qfold - 1 - gm / (G / a.qfold) : 0;
            int ev = 0;               // o holds O * 2^-ev
            bool ev_set = false;
            float o[KS][4];
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

            for (int j = ((ow - gidx) % NP + NP) % NP; j < r.len; j += NP) {
                const int stage = ow * SPW + my_slot;
                // every lane tests the phase (and the abort flag, read alongside); if it is
                // not complete the warp spins together (bounded), giving up early once
                // another warp has given up
                bool ok = mbar_try_wait(&full_bar[stage], my_phase) & !*cons_abort;
                if (!__all_sync(0xffffffffu, ok)) ok = warp_wait(&full_bar[stage], my_phase, wait_limit, cons_abort);
                if (++my_slot == SPW) {
                    my_slot = 0;
                    my_phase ^= 1;
                }
                if (!ok) {
                    *cons_abort = 1;
                    continue;
                }
                const uint32_t kt = smem_u32(sm_stage) + static_cast<uint32_t>(stage) * 2 * TILE;
                const uint32_t vt = kt + TILE;
                const int t0 = (sw.g_lo + r.g + j) * ROWS;
                const int v_lo = max(sw.win_start - t0, 0);
                const int v_hi = min(sw.len - t0, ROWS);
                // ---------------- raw K words and the scales to registers (int8 rows outside
                // the window are finite integers: no clearing); the V words follow the score
                // MMAs, so K and V words are never live together
                uint4 kr[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf)
                        kr[nt][hf] = lds_u4(kt + swz<TROWS>(srow(g + 8 * nt), 32 * t + 16 * hf));
                const uint32_t sc = smem_u32(sm_scale) + static_cast<uint32_t>(stage) * 2 * TROWS * 4;
                // scales of this lane's tokens 8nt + 2t + e (nt = nc * SETS + myset): one per
                // page (slot = token / R), or per token
                auto read_scales = [&](float (*dst)[2], uint32_t base) {
                    if (a.scale_mode == 1) {
#pragma unroll
                        for (int nc = 0; nc < NTC; ++nc) {
                            const int nt = nc * SETS + myset;
                            float f;
                            asm volatile("ld.shared.f32 %0, [%1];"
                                         : "=f"(f)
                                         : "r"(base + static_cast<uint32_t>(((8 * nt) / R) * HP + hsel) * 4));
                            dst[nc][0] = dst[nc][1] = f;
                        }
                    } else {  // tokens 2t, 2t+1 of each n-tile are adjacent
#pragma unroll
                        for (int nc = 0; nc < NTC; ++nc) {
                            const int nt = nc * SETS + myset;
                            const uint2 w2 = lds_u2(base + srow(8 * nt + 2 * t) * 4);
                            dst[nc][0] = __uint_as_float(w2.x);
                            dst[nc][1] = __uint_as_float(w2.y);
                        }
                    }
                };
                float ksc[NTC][2], vsc[NTC][2];
                read_scales(ksc, sc);
                // ---------------- scores
                float s[CH][NTC][4];
#pragma unroll
                for (int c = 0; c < CH; ++c)
#pragma unroll
                    for (int nc = 0; nc < NTC; ++nc)
#pragma unroll
                        for (int e = 0; e < 4; ++e) s[c][nc][e] = 0.f;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    float(*acc)[4] = s[kk % CH];
#pragma unroll
                    for (int js = 0; js < SETS; ++js) {
                        // (volatile: keep the AND here -- hoisted out of the group loop, the
                        // masked copies would need 16 more registers than the budget has)
                        uint32_t a0 = qa[kk][0], a2 = qa[kk][1];
                        if constexpr (SETS == 2) {
                            asm volatile("and.b32 %0, %0, %1;" : "+r"(a0) : "r"(qmask[js]));
                            asm volatile("and.b32 %0, %0, %1;" : "+r"(a2) : "r"(qmask[js]));
                        }
#pragma unroll
                        for (int nc = 0; nc < NTC; ++nc) {
                            const uint4 &q4 = kr[nc * SETS + js][kk >> 2];
                            const uint32_t w = (kk & 3) == 0 ? q4.x : (kk & 3) == 1 ? q4.y : (kk & 3) == 2 ? q4.z : q4.w;
                            uint32_t b0, b1;
                            i8x4_to_f16x2_biased(w, b0, b1);
                            mma_16816<__half>(acc[nc], a0, 0u, a2, 0u, b0, b1);
                            if constexpr (SPLIT) mma_16816<__half>(acc[nc], ql[kk][0], 0u, ql[kk][1], 0u, b0, b1);
                        }
                    }
                }
                // ---------------- V words and scales to registers, then free the stage
                uint4 vr[VK][4];
#pragma unroll
                for (int vk = 0; vk < VK; ++vk)
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        vr[vk][i] = lds_u4(vt + swz<TROWS>(srow(16 * vk + 2 * t + (i & 1) + 8 * (i >> 1)), 16 * g));
                read_scales(vsc, sc + TROWS * 4);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_bar[stage]);
                if constexpr (CH == 2) {
#pragma unroll
                    for (int nc = 0; nc < NTC; ++nc)
#pragma unroll
                        for (int e = 0; e < 2; ++e) s[0][nc][e] += s[1][nc][e];
                }
                // ---------------- online softmax for head g over tokens 8nt + 2t + e
                // (vmax spans the group's window, the same for every row, so the V-scale
                // exponent stays warp-uniform; row g's own causal bound masks its scores)
                const int row_hi = min(v_hi, sw.len - qshift - t0);
                float p[NTC][2];
                bool valid[NTC][2];
                float mloc = -INFINITY;
                float vmax = 0.f;
                bool vout = false;  // an in-window V scale outside [2^(ev-2), 2^(ev+3))
                const float vband_lo = pow2i(max(-126, ev - 2)), vband_hi = pow2i(min(127, ev + 3));
#pragma unroll
                for (int nc = 0; nc < NTC; ++nc)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int tk = 8 * (nc * SETS + myset) + 2 * t + e;
                        if (tk >= v_lo && tk < v_hi) {
                            vmax = fmaxf(vmax, vsc[nc][e]);
                            vout |= !(vsc[nc][e] >= vband_lo && vsc[nc][e] < vband_hi);
                        }
                        valid[nc][e] = row_used && tk >= v_lo && tk < row_hi;
                        p[nc][e] = (s[0][nc][e] - qbias) * (qmul * ksc[nc][e]);
                    }
                if (a.soft_cap > 0.f) {
#pragma unroll
                    for (int nc = 0; nc < NTC; ++nc)
#pragma unroll
                        for (int e = 0; e < 2; ++e)
                            p[nc][e] = a.soft_cap * tanhf(p[nc][e] / a.soft_cap) * a.post_scale;
                }
#pragma unroll
                for (int nc = 0; nc < NTC; ++nc)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        p[nc][e] = valid[nc][e] ? p[nc][e] : -INFINITY;
                        mloc = fmaxf(mloc, p[nc][e]);
                    }
                // probabilities relative to mref, V scales relative to 2^ev, as the value
                // MMA's B fragments: n-tile nt holds tokens 8nt + 2t, 8nt + 2t + 1 of head g,
                // i.e. k rows 2t, 2t+1 (+8) of k-step nt / 2 (two sets: this lane holds
                // n-tile 2nc + myset; the odd one comes from the lane 4G above)
                uint32_t pb[NTC];
                auto probs = [&](float mref, float vmul, float &psum, float &pmass) {
                    psum = 0.f;
                    pmass = 0.f;
#pragma unroll
                    for (int nc = 0; nc < NTC; ++nc) {
                        float pv[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const float pe = fast_exp2(p[nc][e] - mref);
                            psum += pe;
                            pv[e] = valid[nc][e] ? pe * (vsc[nc][e] * vmul) : 0.f;
                        }
                        pb[nc] = pack2<__half>(pv[0], pv[1]);
                        const float2 pr = unpack2<__half>(pb[nc]);
                        pmass += pr.x + pr.y;
                    }
                };
                // Lazy running max: a group whose scores stay within 2^kLazyMax of the row's
                // running max and whose V scales stay inside the exponent band keeps both
                // references (probabilities up to 2^kLazyMax * 8 stay far inside f16; the
                // final normalisation is relative to the same reference, so the result is
                // unchanged), and needs no cross-lane reduction and no rescale.
                const bool slow = mloc > m_run + kLazyMax || vout || !ev_set;
                if (__any_sync(0xffffffffu, slow)) {
                    // reduce over the quad's tokens and, with two sets, over the other set's
                    // row of the same head (lane + or - 4G): every (row, head) pair then agrees
                    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 1));
                    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 2));
                    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
                    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
                    if constexpr (SETS == 2) {
                        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 4 * G));
                        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 4 * G));
                    }
                    const float mn = fmaxf(m_run, mloc);
                    const float alpha = (mn == m_run) ? 1.f : fast_exp2(m_run - mn);
                    const float mref = (mn == -INFINITY) ? 0.f : mn;
                    m_run = mn;
                    // the V-scale exponent (warp-uniform: every quad sees the same tokens)
                    int ev_new = ev;
                    if (vmax > 0.f && vmax < INFINITY) {
                        const int e0 = exp_of(vmax);
                        if (!ev_set || e0 < ev - 2 || e0 > ev + 2) ev_new = max(-100, min(100, e0));
                    }
                    float psum, pmass;
                    probs(mref, pow2i(-ev_new), psum, pmass);
                    l_run = l_run * alpha + psum;
                    const float fac = ev_set ? alpha * pow2i(max(-126, min(127, ev - ev_new))) : alpha;
                    ps_run = ps_run * fac + pmass;
                    ev = ev_new;
                    ev_set = true;
                    if (__any_sync(0xffffffffu, fac != 1.f)) {
                        const float al0 = __shfl_sync(0xffffffffu, fac, 8 * t);      // head 2t
                        const float al1 = __shfl_sync(0xffffffffu, fac, 8 * t + 4);  // head 2t+1
#pragma unroll
                        for (int mt = 0; mt < KS; ++mt) {
                            o[mt][0] *= al0;
                            o[mt][1] *= al1;
                            o[mt][2] *= al0;
                            o[mt][3] *= al1;
                        }
                    }
                } else {
                    float psum, pmass;
                    probs(m_run == -INFINITY ? 0.f : m_run, pow2i(-ev), psum, pmass);
                    l_run += psum;
                    ps_run += pmass;
                }
                // ---------------- values: per k-step, rows 2t, 2t+1 (a0, a1) and 2t+8, 2t+9 (a2, a3)
#pragma unroll
                for (int vk = 0; vk < VK; ++vk) {
                    uint32_t pb0, pb1;
                    if constexpr (SETS == 2) {
                        pb0 = pb[vk];
                        pb1 = __shfl_down_sync(0xffffffffu, pb[vk], 4 * G);
                    } else {
                        pb0 = pb[2 * vk];
                        pb1 = pb[2 * vk + 1];
                    }
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        const uint4 *v4 = vr[vk];
                        const uint32_t ra = w == 0 ? v4[0].x : w == 1 ? v4[0].y : w == 2 ? v4[0].z : v4[0].w;
                        const uint32_t rb = w == 0 ? v4[1].x : w == 1 ? v4[1].y : w == 2 ? v4[1].z : v4[1].w;
                        const uint32_t rc = w == 0 ? v4[2].x : w == 1 ? v4[2].y : w == 2 ? v4[2].z : v4[2].w;
                        const uint32_t rd = w == 0 ? v4[3].x : w == 1 ? v4[3].y : w == 2 ? v4[3].z : v4[3].w;
                        uint32_t a0e, a1e, a0o, a1o, a2e, a3e, a2o, a3o;
                        i8x4_to_f16x2_biased(__byte_perm(ra, rb, 0x5140), a0e, a1e);  // dims 4w, 4w+1
                        i8x4_to_f16x2_biased(__byte_perm(ra, rb, 0x7362), a0o, a1o);  // dims 4w+2, 4w+3
                        i8x4_to_f16x2_biased(__byte_perm(rc, rd, 0x5140), a2e, a3e);
                        i8x4_to_f16x2_biased(__byte_perm(rc, rd, 0x7362), a2o, a3o);
                        mma_16816<__half>(o[2 * w], a0e, a1e, a2e, a3e, pb0, pb1);
                        mma_16816<__half>(o[2 * w + 1], a0o, a1o, a2o, a3o, pb0, pb1);
                    }
                }
            }
            gidx += r.len;

            // ---------------- this warp's state -> shared memory (O = o * 2^ev)
            float *cw = sm_comb + warp * G * (D + 2);
            l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
            l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
            if constexpr (SETS == 2) l_run += __shfl_xor_sync(0xffffffffu, l_run, 4 * G);
            if (t == 0 && g < G) {
                cw[g] = m_run;
                cw[G + g] = l_run;
            }
            // the biased V bytes added 1152 times each head's probability mass to o
            ps_run += __shfl_xor_sync(0xffffffffu, ps_run, 1);
            ps_run += __shfl_xor_sync(0xffffffffu, ps_run, 2);
            if constexpr (SETS == 2) ps_run += __shfl_xor_sync(0xffffffffu, ps_run, 4 * G);
            const float bias0 = 1152.f * __shfl_sync(0xffffffffu, ps_run, 8 * t);      // head 2t
            const float bias1 = 1152.f * __shfl_sync(0xffffffffu, ps_run, 8 * t + 4);  // head 2t+1
            const float om = pow2i(ev);
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int d0 = 16 * g + 2 * mt;
                if (2 * t < G) {
                    cw[2 * G + (2 * t) * D + d0] = (o[mt][0] - bias0) * om;
                    cw[2 * G + (2 * t) * D + d0 + 1] = (o[mt][2] - bias0) * om;
                }
                if (2 * t + 1 < G) {
                    cw[2 * G + (2 * t + 1) * D + d0] = (o[mt][1] - bias1) * om;
                    cw[2 * G + (2 * t + 1) * D + d0 + 1] = (o[mt][3] - bias1) * om;
                }
            }
        } else {
            // ======== fp32 KV on the CUDA cores (packed FFMA).
            static_assert(std::is_same<KV, float>::value && ROWS == 16,
                          "the CUDA-core consumer serves fp32 KV in 16-token groups");
            // Stage q (G heads of this kv-head's group), scaled, as fp32.
            {
                const long long qbase = (static_cast<long long>(r.s) * Hkv + r.h) * G * D;
                for (int i = tid; i < G * D; i += CONS) {
                    // folded multi-query rows sit apart in q ([S, Tq, Hq, D])
                    const long long qi = a.qfold > 1
                                             ? qo_row(r.s, r.h, i / D, Hkv, G, a.qfold, a.seq_div) * D + (i % D)
                                             : qbase + i;
                    const float v = a.q_bf16
                                        ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.q)[qi])
                                        : reinterpret_cast<const float *>(a.q)[qi];
                    sm_q[q_off(D, i / D, i % D)] = v * a.q_scale;
                }
            }
            named_barrier(1, CONS);

            float m[G], l[G];
            float2 acc[G][EPL / 2];
    #pragma unroll
            for (int hh = 0; hh < G; ++hh) {
                m[hh] = -INFINITY;
                l[hh] = 0.f;
    #pragma unroll
                for (int e = 0; e < EPL / 2; ++e) acc[hh][e] = make_float2(0.f, 0.f);
            }

            // this warp's groups of the run: CTA-local indices gidx + j with (gidx + j) % NC == warp
            for (int j = ((ow - gidx) % NP + NP) % NP; j < r.len; j += NP) {
                const int stage = ow * SPW + my_slot;
                bool ok = mbar_try_wait(&full_bar[stage], my_phase) & !*cons_abort;
                if (!__all_sync(0xffffffffu, ok)) ok = warp_wait(&full_bar[stage], my_phase, wait_limit, cons_abort);
                if (++my_slot == SPW) {
                    my_slot = 0;
                    my_phase ^= 1;
                }
                if (!ok) {
                    *cons_abort = 1;
                    continue;
                }
                const uint32_t kt = smem_u32(sm_stage) + static_cast<uint32_t>(stage) * 2 * TILE;
                const uint32_t vt = kt + TILE;
                const int t0 = (sw.g_lo + r.g + j) * kRows;
                const int v_lo = max(sw.win_start - t0, 0);
                const int v_hi = min(sw.len - t0, kRows);

                // ---------------- score pass: lane = (token li, head-dim half)
                float sc[G];
                {
                    float2 dot[G];
    #pragma unroll
                    for (int hh = 0; hh < G; ++hh) dot[hh] = make_float2(0.f, 0.f);
                    const uint32_t qh = smem_u32(sm_q) + q_off(D, 0, half * (D / 2)) * 4;
    #pragma unroll
                    for (int ch = 0; ch < HALF_CH; ++ch) {
                        const uint4 raw = lds_u4(kt + swz(li, (half * HALF_CH + ch) * 16));
                        float kf[EPC];
                        decode_word<KV>(raw.x, kf + 0 * EPW);
                        decode_word<KV>(raw.y, kf + 1 * EPW);
                        decode_word<KV>(raw.z, kf + 2 * EPW);
                        decode_word<KV>(raw.w, kf + 3 * EPW);
    #pragma unroll
                        for (int hh = 0; hh < G; ++hh) {
    #pragma unroll
                            for (int e = 0; e < EPC; e += 4) {
                                const float4 qv = lds_f4(qh + (hh * QROW + ch * EPC + e) * 4);
                                dot[hh] = __ffma2_rn(make_float2(qv.x, qv.y),
                                                     make_float2(kf[e], kf[e + 1]), dot[hh]);
                                dot[hh] = __ffma2_rn(make_float2(qv.z, qv.w),
                                                     make_float2(kf[e + 2], kf[e + 3]), dot[hh]);
                            }
                        }
                    }
                    const bool valid = li >= v_lo && li < v_hi;
    #pragma unroll
                    for (int hh = 0; hh < G; ++hh) {
                        float x2 = dot[hh].x + dot[hh].y;
                        x2 += __shfl_xor_sync(0xffffffffu, x2, 16);
                        if (a.soft_cap > 0.f) x2 = a.soft_cap * tanhf(x2 / a.soft_cap) * a.post_scale;
                        sc[hh] = valid ? x2 : -INFINITY;
                    }
                    if (a.qfold > 1) {  // folded row hh: its query sees the positions before len - qshift
                        const int gm = G / a.qfold;
    #pragma unroll
                        for (int hh = 0; hh < G; ++hh)
                            if (t0 + li >= sw.len - (a.qfold - 1 - hh / gm)) sc[hh] = -INFINITY;
                    }
                }

                // ---------------- online softmax (exp2 domain), per head over the 16 tokens
                bool rescale = false;
                float alpha[G], pw[GP];
    #pragma unroll
                for (int hh = 0; hh < G; ++hh) {
                    float mx = sc[hh];
    #pragma unroll
                    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    const float mn = fmaxf(m[hh], mx);
                    alpha[hh] = (mn == m[hh]) ? 1.f : fast_exp2(m[hh] - mn);
                    rescale |= (mn != m[hh]);
                    m[hh] = mn;
                    const float mref = (mn == -INFINITY) ? 0.f : mn;
                    const float p = fast_exp2(sc[hh] - mref);
                    l[hh] = l[hh] * alpha[hh] + (half == 0 ? p : 0.f);
                    pw[hh] = p;
                }
    #pragma unroll
                for (int hh = G; hh < GP; ++hh) pw[hh] = 0.f;
                if (half == 0) {
    #pragma unroll
                    for (int hh = 0; hh < GP; hh += 4)
                        sts_f4(p_base + (li * GP + hh) * 4,
                               make_float4(pw[hh], pw[hh + 1], pw[hh + 2], pw[hh + 3]));
                }
                if (rescale) {
    #pragma unroll
                    for (int hh = 0; hh < G; ++hh) {
                        const float2 al = make_float2(alpha[hh], alpha[hh]);
    #pragma unroll
                        for (int e = 0; e < EPL / 2; ++e) acc[hh][e] = __fmul2_rn(acc[hh][e], al);
                    }
                }
                __syncwarp();

                // ---------------- value pass: lanes 0-15 even rows, 16-31 odd rows
                auto value_row = [&](int rr) {
                    float vf[EPL];
                    const int b0 = li * LANE_BYTES;
                    if constexpr (LANE_BYTES >= 16) {
    #pragma unroll
                        for (int k = 0; k < LANE_BYTES / 16; ++k) {
                            const uint4 raw = lds_u4(vt + swz(rr, b0 + 16 * k));
                            decode_word<KV>(raw.x, vf + (4 * k + 0) * EPW);
                            decode_word<KV>(raw.y, vf + (4 * k + 1) * EPW);
                            decode_word<KV>(raw.z, vf + (4 * k + 2) * EPW);
                            decode_word<KV>(raw.w, vf + (4 * k + 3) * EPW);
                        }
                    } else {
                        static_assert(LANE_BYTES == 8 || LANE_BYTES >= 16, "value-pass width");
                        const uint2 raw = lds_u2(vt + swz(rr, b0));
                        decode_word<KV>(raw.x, vf + 0 * EPW);
                        decode_word<KV>(raw.y, vf + 1 * EPW);
                    }
                    float pv[GP];
    #pragma unroll
                    for (int hh = 0; hh < GP; hh += 4) {
                        const float4 t = lds_f4(p_base + (rr * GP + hh) * 4);
                        pv[hh] = t.x;
                        pv[hh + 1] = t.y;
                        pv[hh + 2] = t.z;
                        pv[hh + 3] = t.w;
                    }
    #pragma unroll
                    for (int hh = 0; hh < G; ++hh) {
                        const float2 pp = make_float2(pv[hh], pv[hh]);
    #pragma unroll
                        for (int e = 0; e < EPL / 2; ++e)
                            acc[hh][e] = __ffma2_rn(pp, make_float2(vf[2 * e], vf[2 * e + 1]), acc[hh][e]);
                    }
                };
                if (v_lo == 0 && v_hi == kRows) {  // a full group: fixed trip count, unrolled
    #pragma unroll
                    for (int i = 0; i < kRows / 2; ++i) value_row(2 * i + half);
                } else {
                    for (int rr = v_lo + half; rr < v_hi; rr += 2) value_row(rr);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_bar[stage]);
            }
            gidx += r.len;

            // ---------------- merge the NC warp states of this run
            {
                float *cw = sm_comb + warp * G * (D + 2);
    #pragma unroll
                for (int hh = 0; hh < G; ++hh) {
                    const float lw = warp_sum(l[hh]);
    #pragma unroll
                    for (int e = 0; e < EPL / 2; ++e) {
                        acc[hh][e].x += __shfl_xor_sync(0xffffffffu, acc[hh][e].x, 16);
                        acc[hh][e].y += __shfl_xor_sync(0xffffffffu, acc[hh][e].y, 16);
                    }
                    if (lane == 0) {
                        cw[hh] = m[hh];
                        cw[G + hh] = lw;
                    }
                    if (half == 0) {
    #pragma unroll
                        for (int e = 0; e < EPL / 2; ++e) {
                            cw[2 * G + hh * D + li * EPL + 2 * e] = acc[hh][e].x;
                            cw[2 * G + hh * D + li * EPL + 2 * e + 1] = acc[hh][e].y;
                        }
                    }
                }
            }
        }
        named_barrier(1, CONS);
        if (*cons_abort) {
            // A wait gave up in this CTA: stop cleanly, but let every split-K piece this
            // CTA still owns (this run and the rest of its range) arrive on its counter,
            // so that whoever arrives last resets the counter and the scratch is zeroed
            // for the next call.  The last arriver merges whatever partials it finds; the
            // call's result is void anyway (GOLLEK_STATUS_TIMEOUT is raised).
            if (tid == 0) {
                auto arrive_only = [&](const Run &rr) {
                    if (rr.pieces <= 1) return;
                    int *c = &a.counters[rr.s * Hkv + rr.h];
                    if (atomicAdd(c, 1) == rr.pieces - 1) atomicExch(c, 0);
                };
                arrive_only(r);
                for (long long y = x; y < x_end;) {
                    Run rn = run_at(y);
                    run_pieces(rn);
                    y += rn.len;
                    arrive_only(rn);
                }
            }
            break;
        }

        const long long out_row = (static_cast<long long>(r.s) * Hkv + r.h) * UG * D;
        // element o of the (s, h) state [G][D] in out (folded queries: [S, qfold, Hq, D])
        auto out_at = [&](int o) -> long long {
            return a.qfold > 1 ? qo_row(r.s, r.h, o / D, Hkv, G, a.qfold, a.seq_div) * D + (o % D) : out_row + o;
        };
        const int slot_floats = 2 * UG + UG * D;
        float *part = nullptr;
        if (r.pieces > 1)
            part = a.partials +
                   (static_cast<long long>(r.s * Hkv + r.h) * kMaxSplits + r.piece) * slot_floats;
        for (int o = tid; o < UG * D; o += CONS) {
            const int ro = o / D;          // row of the unit
            const int hs = ro / G;         // PAIR: the head of the pair it belongs to
            const int gr = ro - hs * G;    // its row among that head's warp states
            const int oo = gr * D + (o - ro * D);
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NC; ++w)
                if (w % HP == hs) M = fmaxf(M, sm_comb[w * G * (D + 2) + gr]);
            float Ls = 0.f, As = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < NC; ++w) {
                    if (w % HP != hs) continue;
                    const float *cw = sm_comb + w * G * (D + 2);
                    const float mw = cw[gr];
                    const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
                    Ls += cw[G + gr] * f;
                    As += cw[2 * G + oo] * f;
                }
            }
            if (r.pieces == 1) {
                const float v = Ls > 0.f ? As * (1.0f / (Ls + a.norm_eps)) : 0.f;
                store_out(a.out, out_at(o), v, a.q_bf16);
            } else {
                part[2 * UG + o] = As;
                if ((o % D) == 0) {
                    part[ro] = M;
                    part[UG + ro] = Ls;
                }
            }
        }
        if (r.pieces > 1) {
            __threadfence();
            named_barrier(1, CONS);
            if (tid == 0) {
                const int old = atomicAdd(&a.counters[r.s * Hkv + r.h], 1);
                sm_misc[0] = (old == r.pieces - 1) ? 1 : 0;
            }
            named_barrier(1, CONS);
            if (sm_misc[0]) {
                __threadfence();
                const float *base =
                    a.partials + static_cast<long long>(r.s * Hkv + r.h) * kMaxSplits * slot_floats;
                for (int o = tid; o < UG * D; o += CONS) {
                    const int ro = o / D;
                    float M = -INFINITY;
                    for (int c = 0; c < r.pieces; ++c) M = fmaxf(M, __ldcg(base + c * slot_floats + ro));
                    float Ls = 0.f, As = 0.f;
                    if (M != -INFINITY) {
                        for (int c = 0; c < r.pieces; ++c) {
                            const float *pc = base + c * slot_floats;
                            const float mc = __ldcg(pc + ro);
                            const float f = (mc == -INFINITY) ? 0.f : fast_exp2(mc - M);
                            Ls += __ldcg(pc + UG + ro) * f;
                            As += __ldcg(pc + 2 * UG + o) * f;
                        }
                    }
                    const float v = Ls > 0.f ? As * (1.0f / (Ls + a.norm_eps)) : 0.f;
                    store_out(a.out, out_at(o), v, a.q_bf16);
                }
                if (tid == 0) atomicExch(&a.counters[r.s * Hkv + r.h], 0);
            }
        } else {
            // Every thread has read the warp states of this run before any warp writes
            // the next run's (a warp with no group in the next run gets there quickly).
            named_barrier(1, CONS);
        }
    }
}

}  // namespace gk
