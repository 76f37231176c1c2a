// tc_tiles.cuh -- what the tensor-memory kernels (decode_tc.cuh, prefill_tc.cuh) share:
// the walk over a CTA's tiles and the producer warp that copies K or V tiles into a ring.
//
// A run of one (sequence, kv-head) of the stream-K schedule (decode_common.cuh) is cut
// into tiles of up to 8 groups = 128 tokens.  One group (16 tokens x 128 head-dim bf16 =
// 4 KB) is [row half][64-column slab][8 rows][128 bytes], written by one 4-D TMA box in
// the 128-byte swizzle, so every 8-token core group of a tile sits 2 KB after the previous
// one and the two column slabs of a core group are 1 KB apart: the canonical
// 128B-swizzled operand layout, K-major along head_dim (K as a score operand) and
// MN-major along head_dim (V as a value operand).
#pragma once

#include "decode_common.cuh"
#include "tcgen05.cuh"

namespace gk {

constexpr int kTcGroups = 8;                            // 16-token groups per tile
constexpr int kTcTokens = kTcGroups * kRows;            // 128
constexpr uint32_t kTcGroupBytes = kRows * 256;         // 4 KB: K or V of one group
constexpr uint32_t kTcTile = kTcGroups * kTcGroupBytes; // 32 KB: K or V of one tile

// Byte offset of 16-byte chunk `ch` (head_dim 8*ch .. 8*ch+7) of token `tok` in a K or V
// tile (group layout above).
__device__ __forceinline__ uint32_t tile_chunk_off(int tok, int ch) {
    const int r8 = tok & 7;
    return static_cast<uint32_t>((tok >> 3) * 2048 + (ch >> 3) * 1024 + r8 * 128 + (((ch & 7) ^ r8) << 4));
}

// Tiles of a CTA in order: the runs of its range, each cut into <= 8-group tiles.
struct TileIt {
    long long x;  // first unit of the current run
    Run r;
    int tg0;      // first group of the tile within the run
    int ri;       // run index within this CTA
    int ti;       // tile index within this CTA
    bool live;
};

__device__ __forceinline__ TileIt tile_begin(const Schedule &sch) {
    TileIt t;
    t.x = sch.x_beg;
    t.tg0 = 0;
    t.ri = 0;
    t.ti = 0;
    t.live = t.x < sch.x_end;
    if (t.live) {
        t.r = sch.run_at(t.x);
        sch.pieces(t.r);
    }
    return t;
}

__device__ __forceinline__ void tile_next(const Schedule &sch, TileIt &t) {
    ++t.ti;
    t.tg0 += kTcGroups;
    if (t.tg0 >= t.r.len) {
        t.x += t.r.len;
        ++t.ri;
        t.tg0 = 0;
        t.live = t.x < sch.x_end;
        if (t.live) {
            t.r = sch.run_at(t.x);
            sch.pieces(t.r);
        }
    }
}

__device__ __forceinline__ int tc_win_start(const DecodeArgs &a, int len) {
    return (a.window > 0 && len > a.window) ? len - a.window : 0;
}

// Producer warp of one ring (K or V): per tile, lane i looks up group i's page (two tiles
// ahead, so the block-table loads are in flight while the current tile waits for its
// slot) and, once the slot is free, issues the group's TMA box (suspend_ns > 0: each test
// of the slot may suspend the lane that long, see mbar_wait_or_abort).
// Gives up (raising *abort) if a wait for a free slot runs out or another warp gave up;
// every copy it issued has landed when it returns.
__device__ inline void tc_producer(const DecodeArgs &a, const Schedule &sch, const int *sm_len,
                                   volatile int *abort, const CUtensorMap *map, uint8_t *ring,
                                   uint64_t *full, uint64_t *empty, int NR, int lane,
                                   uint32_t suspend_ns = 0) {
    const int R = a.block_size < kRows ? a.block_size : kRows;  // rows per TMA box
    const int npg = kRows / R;                                  // pages per group (<= 2)
    struct Loc {
        int pid0, pid1, row_off;
        unsigned loaded;
    };
    auto locate = [&](const TileIt &t) {
        Loc l{0, 0, 0, 0u};
        if (!t.live) return l;
        const int ng = min(kTcGroups, t.r.len - t.tg0);
        if (lane < ng) {
            const int len = sm_len[t.r.s];
            const int ws = tc_win_start(a, len);
            const int t0 = (ws / kRows + t.r.g + t.tg0 + lane) * kRows;
            const int p_first = t0 / a.block_size;
            l.row_off = a.block_size < kRows ? 0 : t0 % a.block_size;
            const int pages_in_seq = (len + a.block_size - 1) / a.block_size;
            const int *bt = a.block_tables + static_cast<long long>(t.r.s / a.seq_div) * a.max_blocks;
            for (int j = 0; j < npg; ++j) {
                const int pg = p_first + j;
                if (pg < pages_in_seq && (pg + 1) * a.block_size > ws) {
                    const int e = __ldg(bt + pg);
                    if (j)
                        l.pid1 = e;
                    else
                        l.pid0 = e;
                    l.loaded |= 1u << j;
                }
            }
        }
        return l;
    };
    int issued = 0;
    TileIt ia = tile_begin(sch);
    Loc la = locate(ia);
    TileIt ib = ia;
    if (ib.live) tile_next(sch, ib);
    Loc lb = locate(ib);
    while (ia.live) {
        if (*abort) break;
        // test-only fault injection: CTA 0 stops issuing at this tile (the copies are
        // simply never made, so a consumer's bounded wait gives up; nothing else changes)
        if (a.fault_skip_group >= 0 && blockIdx.x == 0 && ia.ti == a.fault_skip_group) break;
        TileIt ic = ib;
        if (ic.live) tile_next(sch, ic);
        const Loc lc = locate(ic);
        const int slot = ia.ti % NR;
        const int rnd = ia.ti / NR;
        uint32_t bytes = static_cast<uint32_t>(__popc(la.loaded)) * R * 256u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
        bool ok = true;
        if (rnd > 0) {
            if (lane == 0)
                ok = mbar_wait_or_abort(&empty[slot], (rnd - 1) & 1, abort, suspend_ns ? kSuspendTries : kWaitLimit,
                                        suspend_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        if (!ok) {
            if (lane == 0) *abort = 1;
            break;
        }
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], bytes);
        __syncwarp();
        if (la.loaded) {
            uint8_t *dst = ring + static_cast<uint32_t>(slot) * kTcTile + lane * kTcGroupBytes;
#pragma unroll 1
            for (int j = 0; j < npg; ++j) {
                if (!((la.loaded >> j) & 1)) continue;
                int e = j ? la.pid1 : la.pid0;
                if (e < 0 || (a.num_blocks > 0 && e >= a.num_blocks)) {
                    raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
                    e = 0;
                }
                const long long y = static_cast<long long>(e) * a.page_rows +
                                    static_cast<long long>(ia.r.h) * a.block_size + la.row_off;
                tma_load_4d(dst + j * R * 256, map, 0, 0, 0, static_cast<int>(y >> 3), &full[slot]);
            }
        }
        ++issued;
        ia = ib;
        la = lb;
        ib = ic;
        lb = lc;
    }
    // every copy issued lands before the CTA's shared memory is released
    if (lane == 0)
        for (int k = max(0, issued - NR); k < issued; ++k) mbar_wait(&full[k % NR], (k / NR) & 1);
    __syncwarp();
}

}  // namespace gk
