// decode_tma.cuh -- persistent, warp-specialised paged decode attention for sm_100a.
//
// One CTA = NC consumer warps + 1 producer warp, resident for the whole launch
// (grid = SMs x CTAs-per-SM).  The unit of work is an item (sequence, kv-head,
// split-K chunk of 32-token groups).  Every CTA derives the same item list from
// the context lengths in a prologue (a block-wide scan kept in shared memory) and
// takes items b, b+grid, b+2*grid, ...
//
// Producer warp: for each 32-token group of its items, reads the block table,
// and issues 2-D TMA tile loads (SWIZZLE_128B, no multicast) of the K and V rows
// of the group's pages into a ring of shared-memory stages, completing on the
// stage's mbarrier.  For int8 KV it also cp.async-copies the per-token scales.
//
// Consumer warps: group j of an item goes to warp j % NC.  Score pass: lane z owns
// token row z of the stage and dots it against the G query heads of the GQA group
// (q staged in shared memory as fp32, read by broadcast), with packed fp32x2 FMAs.
// Online softmax per head across the warp (exp2 domain).  Value pass: lanes 0-15
// take even rows, 16-31 odd rows, each lane owning head_dim/16 columns of all G
// heads.  At the end of an item the NC warp states merge through shared memory;
// a single-chunk item writes the output, a multi-chunk item writes an fp32
// partial (m, l, acc) and the CTA that completes the last chunk of a
// (sequence, kv-head) merges all partials (split-K log-sum-exp reduce) and resets
// the arrival counter, so the workspace stays zeroed between calls.
//
// The swizzled layout: each stage tile is stored as 128-byte-wide column slabs of
// 32 rows; 16-byte chunk c of row r sits at chunk position c ^ (r & 7).  Lanes of a
// quarter-warp read 8 different rows of the same logical chunk, or 8 chunks of one
// row, and hit 8 distinct bank groups either way.
#pragma once

#include "common.cuh"

namespace gk {

constexpr int kRows = 32;          // tokens per stage (one per lane in the score pass)
constexpr int kSlabBytes = kRows * 128;
constexpr int kMaxSplits = 64;     // split-K chunks per (sequence, kv-head) at most
constexpr int kMaxFastSeqs = 16384;

struct DecodeArgs {
    void *out;
    const void *q;
    const float *k_scales;
    const float *v_scales;
    const int *block_tables;
    const int *context_lens;
    float *partials;   // split-K partial states: [slot][G*2 + G*D] fp32
    int *counters;     // [num_seqs * num_kv_heads] arrival counters, zero between calls
    long long page_rows;  // rows of head_dim elements between consecutive pages
    long long scale_page_stride, scale_head_stride, scale_token_stride;
    int num_seqs, num_kv_heads, block_size, max_blocks, num_blocks;
    int window;           // <= 0: no sliding window
    int q_bf16;           // 1: q/out bf16, 0: fp32
    int num_stages;
    int min_chunk_groups;
    int items_per_cta;
    float q_scale;        // applied to q when staged: scale*log2(e), or scale with soft-cap
    float soft_cap;       // > 0: cap*tanh(score/cap)
    float post_scale;     // log2(e) with soft-cap, else 1
    float norm_eps;       // 1e-9 (engine path) or 0 (legacy fp32 path)
};

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

// Decode 4 bytes of KV elements into floats (bf16/f16: 2, f32: 1, int8: 4).
template <typename KV>
__device__ __forceinline__ void decode_word(uint32_t w, float *f);
template <>
__device__ __forceinline__ void decode_word<__nv_bfloat16>(uint32_t w, float *f) {
    f[0] = bf16_lo(w);
    f[1] = bf16_hi(w);
}
template <>
__device__ __forceinline__ void decode_word<__half>(uint32_t w, float *f) {
    float2 v = __half22float2(*reinterpret_cast<__half2 *>(&w));
    f[0] = v.x;
    f[1] = v.y;
}
template <>
__device__ __forceinline__ void decode_word<float>(uint32_t w, float *f) {
    f[0] = __uint_as_float(w);
}
template <>
__device__ __forceinline__ void decode_word<int8_t>(uint32_t w, float *f) {
    // Signed byte b -> float: bias to b+128 in [0,255], place it in the low mantissa
    // byte of 2^23, subtract 2^23 + 128.  Exact.
    const uint32_t u = w ^ 0x80808080u;
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    float2 a = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                           __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)));
    float2 b = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                           __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)));
    a = __fadd2_rn(a, bias);
    b = __fadd2_rn(b, bias);
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

// Byte offset in a swizzled stage tile of byte `b` of row `r`.
__device__ __forceinline__ uint32_t swz(int r, int b) {
    return static_cast<uint32_t>((b >> 7) * kSlabBytes + r * 128 + ((((b >> 4) & 7) ^ (r & 7)) << 4) +
                                 (b & 15));
}

__device__ __forceinline__ void store_out(void *out, long long idx, float v, int bf16) {
    if (bf16)
        reinterpret_cast<__nv_bfloat16 *>(out)[idx] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float *>(out)[idx] = v;
}

// Shared-memory carve-up, identical on host and device.
struct DecodeSmem {
    uint32_t stages, q, p, comb, scales, prefix, misc, bars, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline DecodeSmem decode_smem_layout(int kv_bytes, bool quant, int D, int G,
                                                         int NC, int stages, int num_seqs) {
    DecodeSmem L;
    const uint32_t tile = static_cast<uint32_t>(D * kv_bytes / 128) * kSlabBytes;
    uint32_t o = 0;
    L.stages = o;
    o += stages * 2 * tile;
    L.q = o;
    o += G * D * 4;
    L.p = o;
    o += NC * kRows * G * 4;
    L.comb = o;
    o += NC * G * (D + 2) * 4;
    L.scales = o;
    o += quant ? stages * 2 * kRows * 4 : 0;
    L.prefix = o;
    o += (num_seqs + 1) * 4;
    o = align_up(o, 16);
    L.misc = o;
    o += 64;
    L.bars = o;
    o += stages * 2 * 8;
    L.total = o + 1024;  // slack to align the base to 1024 bytes
    return L;
}

// Split-K plan of one sequence: its 32-token groups [g_lo, g_hi) in chunks of cs.
struct SeqPlan {
    int len, win_start, g_lo, n_groups, chunk;
};

__device__ __forceinline__ SeqPlan seq_plan(const DecodeArgs &a, int s, int base_chunk) {
    SeqPlan sp;
    int len = a.context_lens[s];
    const int cap = a.max_blocks * a.block_size;
    if (len < 0) len = 0;
    if (len > cap) len = cap;
    sp.len = len;
    sp.win_start = (a.window > 0 && len > a.window) ? len - a.window : 0;
    sp.g_lo = sp.win_start / kRows;
    sp.n_groups = len > 0 ? (len + kRows - 1) / kRows - sp.g_lo : 0;
    const int need = (sp.n_groups + kMaxSplits - 1) / kMaxSplits;
    sp.chunk = base_chunk > need ? base_chunk : need;
    return sp;
}

template <typename KV, int D, int G, int NC>
__global__ void __launch_bounds__((NC + 1) * 32, 2)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
    constexpr int KB = KvType<KV>::kBytes;
    constexpr bool QUANT = KvType<KV>::kQuant;
    constexpr int ROW_BYTES = D * KB;
    constexpr int NSLAB = ROW_BYTES / 128;
    constexpr int TILE = NSLAB * kSlabBytes;
    constexpr int CH = ROW_BYTES / 16;     // 16-byte chunks per row
    constexpr int EPC = 16 / KB;           // elements per chunk
    constexpr int EPL = D / 16;            // value-pass columns per lane
    constexpr int LANE_BYTES = EPL * KB;   // value-pass bytes per lane per row
    constexpr int NT = (NC + 1) * 32;
    constexpr int CONS = NC * 32;
    constexpr int EPW = 4 / KB;            // elements per 32-bit word
    static_assert(ROW_BYTES % 128 == 0, "row must be a whole number of 128-byte slabs");
    static_assert(EPL % 2 == 0 && EPC % 4 == 0, "vector widths");
    static_assert(NSLAB * 2 * 4 <= 32, "TMA loads of one group (<= 4 pages) fit a warp");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const DecodeSmem L = decode_smem_layout(KB, QUANT, D, G, NC, a.num_stages, a.num_seqs);
    uint8_t *sm_stage = smem + L.stages;
    float *sm_q = reinterpret_cast<float *>(smem + L.q);
    float *sm_p = reinterpret_cast<float *>(smem + L.p);
    float *sm_comb = reinterpret_cast<float *>(smem + L.comb);
    float *sm_scale = reinterpret_cast<float *>(smem + L.scales);
    int *sm_prefix = reinterpret_cast<int *>(smem + L.prefix);
    volatile int *sm_misc = reinterpret_cast<volatile int *>(smem + L.misc);
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty_bar = full_bar + a.num_stages;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int S = a.num_seqs;
    const int Hkv = a.num_kv_heads;
    const int NS = a.num_stages;  // NC * SPW: consumer warp w owns stages [w*SPW, w*SPW+SPW)
    const int SPW = NS / NC;
    // Group gidx belongs to warp gidx % NC and lands in that warp's stage ring.  A stage
    // is only ever waited on by its owner warp, in order, so no mbarrier wait is more
    // than one phase ahead of the barrier (parity waits cannot alias).
    auto stage_of = [&](int gi) { return (gi % NC) * SPW + (gi / NC) % SPW; };
    auto round_of = [&](int gi) { return (gi / NC) / SPW; };

    // ------------------------------------------------------------ prologue
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full_bar[i], QUANT ? 1 + 32 : 1);
            mbar_init(&empty_bar[i], 1);
        }
        fence_barrier_init();
        sm_misc[0] = 0;  // abort flag
        sm_misc[1] = 0;  // "this CTA merges the partials" flag
        sm_misc[2] = 0;  // total groups (reduction)
    }
    if (warp == NC && lane == 0) {
        prefetch_tensormap(&tm_k);
        prefetch_tensormap(&tm_v);
    }
    __syncthreads();

    // Total groups over all sequences -> uniform chunk size.
    int my_groups = 0;
    for (int s = tid; s < S; s += NT) {
        my_groups += seq_plan(a, s, 1).n_groups;
        const int raw = a.context_lens[s];
        if (raw < 0 || raw > a.max_blocks * a.block_size) raise_status(GOLLEK_STATUS_BAD_POSITION);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_groups += __shfl_xor_sync(0xffffffffu, my_groups, o);
    if (lane == 0) atomicAdd(const_cast<int *>(&sm_misc[2]), my_groups);
    __syncthreads();
    const long long total_units = static_cast<long long>(sm_misc[2]) * Hkv;
    const long long target = static_cast<long long>(gridDim.x) * a.items_per_cta;
    int base_chunk = static_cast<int>((total_units + target - 1) / (target > 0 ? target : 1));
    if (base_chunk < a.min_chunk_groups) base_chunk = a.min_chunk_groups;
    if (base_chunk < 1) base_chunk = 1;

    // Exclusive prefix over per-sequence split counts (contiguous segment per thread).
    {
        const int seg = (S + NT - 1) / NT;
        const int s0 = tid * seg;
        const int s1 = min(S, s0 + seg);
        int sum = 0;
        for (int s = s0; s < s1; ++s) {
            SeqPlan sp = seq_plan(a, s, base_chunk);
            int splits = sp.n_groups > 0 ? (sp.n_groups + sp.chunk - 1) / sp.chunk : 1;
            sm_prefix[s] = splits;
            sum += splits;
        }
        // inclusive warp scan of per-thread sums
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int *warp_tot = reinterpret_cast<int *>(sm_comb);  // scratch before first use
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (tid == 0) {
            int run = 0;
            for (int w = 0; w <= NC; ++w) {
                int t = warp_tot[w];
                warp_tot[w] = run;
                run += t;
            }
            sm_prefix[S] = run;
        }
        __syncthreads();
        int run = warp_tot[warp] + incl - sum;
        for (int s = s0; s < s1; ++s) {
            int v = sm_prefix[s];
            sm_prefix[s] = run;
            run += v;
        }
        __syncthreads();
    }
    const int num_items = sm_prefix[S] * Hkv;

    // Item -> (sequence, kv-head, chunk).
    auto locate = [&](int item, int &s, int &h, int &c) {
        const int u = item / Hkv;
        h = item - u * Hkv;
        int lo = 0, hi = S - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (sm_prefix[mid] <= u)
                lo = mid;
            else
                hi = mid - 1;
        }
        s = lo;
        c = u - sm_prefix[lo];
    };

    if (warp == NC) {
        // ========================================================= producer
        // Pages of one group: BS < 32 -> 32/BS whole pages (R = BS rows each);
        // BS >= 32 -> one 32-row slice of a page.
        const int R = a.block_size < kRows ? a.block_size : kRows;
        const int npg = kRows / R;  // <= 4 (BS >= 8)
        int gidx = 0;
        bool aborted = false;
        for (int item = blockIdx.x; item < num_items && !aborted; item += gridDim.x) {
            int s, h, c;
            locate(item, s, h, c);
            const SeqPlan sp = seq_plan(a, s, base_chunk);
            const int g_beg = sp.g_lo + c * sp.chunk;
            const int g_end = min(sp.g_lo + sp.n_groups, g_beg + sp.chunk);
            const int *bt = a.block_tables + static_cast<long long>(s) * a.max_blocks;
            const int pages_in_seq = (sp.len + a.block_size - 1) / a.block_size;
            int batch_base = -(1 << 30);
            int batch_entry = 0;  // lane i: block-table entry batch_base + i
            for (int g = g_beg; g < g_end; ++g, ++gidx) {
                const int stage = stage_of(gidx);
                const int round = round_of(gidx);
                if (round > 0) {
                    bool ok = true;
                    if (lane == 0) ok = mbar_wait(&empty_bar[stage], (round - 1) & 1);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) {
                        aborted = true;
                        break;
                    }
                }
                const int t0 = g * kRows;
                const int p_first = t0 / a.block_size;
                const int row_off = a.block_size < kRows ? 0 : t0 % a.block_size;
                if (p_first < batch_base || p_first + npg - 1 >= batch_base + 32) {
                    batch_base = p_first;
                    const int e = batch_base + lane;
                    batch_entry = (e < pages_in_seq) ? __ldg(bt + e) : 0;
                }
                // lane j < npg resolves page j of the group
                const int pg = p_first + lane;
                const bool need = lane < npg && pg < pages_in_seq &&
                                  (pg + 1) * a.block_size > sp.win_start;
                int entry = __shfl_sync(0xffffffffu, batch_entry, (pg - batch_base) & 31);
                if (need && (entry < 0 || (a.num_blocks > 0 && entry >= a.num_blocks))) {
                    raise_status(GOLLEK_STATUS_BAD_BLOCK_ID);
                    entry = 0;
                }
                const unsigned loaded = __ballot_sync(0xffffffffu, need);
                uint8_t *kdst = sm_stage + static_cast<uint32_t>(stage) * 2 * TILE;
                uint8_t *vdst = kdst + TILE;
                if (lane == 0)
                    mbar_arrive_expect_tx(&full_bar[stage],
                                          static_cast<uint32_t>(__popc(loaded)) * 2u * NSLAB * R * 128u);
                __syncwarp();
                // one lane per (page, slab, K/V) TMA load: npg * NSLAB * 2 <= 32
                {
                    const int j = lane / (NSLAB * 2);
                    const int rem = lane - j * NSLAB * 2;
                    const int pj = __shfl_sync(0xffffffffu, entry, j & 31);
                    if (j < npg && ((loaded >> j) & 1)) {
                        const int slab = rem >> 1;
                        const int isv = rem & 1;
                        const long long y = static_cast<long long>(pj) * a.page_rows +
                                            static_cast<long long>(h) * a.block_size + row_off;
                        uint8_t *dst = (isv ? vdst : kdst) + slab * kSlabBytes + j * R * 128;
                        tma_load_2d(dst, isv ? &tm_v : &tm_k, slab * (128 / KB),
                                    static_cast<int>(y), &full_bar[stage]);
                    }
                }
                if constexpr (QUANT) {
                    const int t = t0 + lane;
                    const int j = lane / R;
                    const int pj = __shfl_sync(0xffffffffu, entry, j);
                    float *ks = sm_scale + stage * 2 * kRows;
                    if (t >= sp.win_start && t < sp.len && ((loaded >> j) & 1)) {
                        const long long so =
                            static_cast<long long>(pj) * a.scale_page_stride +
                            static_cast<long long>(h) * a.scale_head_stride +
                            static_cast<long long>(t % a.block_size) * a.scale_token_stride;
                        cp_async_4(ks + lane, a.k_scales + so);
                        cp_async_4(ks + kRows + lane, a.v_scales + so);
                    }
                    cp_async_mbar_arrive_noinc(&full_bar[stage]);
                }
            }
        }
        if (aborted) {
            // Let every copy already issued land before the CTA's shared memory is released.
            for (int k = 0; k < NS && k < gidx; ++k) {
                const int gi = gidx - 1 - k;
                if (lane == 0) mbar_wait(&full_bar[stage_of(gi)], round_of(gi) & 1);
            }
        }
        return;
    }

    // ============================================================ consumers
    // Control flow below depends only on state the consumer warps themselves write
    // before a named barrier, so all NC warps take the same barriers.
    const int half = lane >> 4;
    const int li = lane & 15;
    float *my_p = sm_p + warp * kRows * G;
    volatile int *cons_abort = sm_misc + 3;
    if (tid == 0) *cons_abort = 0;
    named_barrier(1, CONS);
    int gidx = 0;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
        int s, h, c;
        locate(item, s, h, c);
        const SeqPlan sp = seq_plan(a, s, base_chunk);
        const int g_beg = sp.g_lo + c * sp.chunk;
        const int g_end = min(sp.g_lo + sp.n_groups, g_beg + sp.chunk);
        const int splits = sm_prefix[s + 1] - sm_prefix[s];

        // Stage q (G heads of this kv-head's group), scaled, as fp32.
        {
            const long long qbase = (static_cast<long long>(s) * Hkv + h) * G * D;
            for (int i = tid; i < G * D; i += CONS) {
                float v = a.q_bf16 ? __bfloat162float(
                                         reinterpret_cast<const __nv_bfloat16 *>(a.q)[qbase + i])
                                   : reinterpret_cast<const float *>(a.q)[qbase + i];
                sm_q[i] = v * a.q_scale;
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

        for (int g = g_beg; g < g_end; ++g, ++gidx) {
            if (gidx % NC != warp) continue;
            if (*cons_abort) continue;
            const int stage = stage_of(gidx);
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&full_bar[stage], round_of(gidx) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                *cons_abort = 1;
                continue;
            }
            const uint8_t *kt = sm_stage + static_cast<uint32_t>(stage) * 2 * TILE;
            const uint8_t *vt = kt + TILE;
            const int t0 = g * kRows;
            const int v_lo = max(sp.win_start - t0, 0);
            const int v_hi = min(sp.len - t0, kRows);

            // ---------------- score pass: lane = token row
            float sc[G];
            {
                float2 dot[G];
#pragma unroll
                for (int hh = 0; hh < G; ++hh) dot[hh] = make_float2(0.f, 0.f);
#pragma unroll 2
                for (int ch = 0; ch < CH; ++ch) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(kt + swz(lane, ch * 16));
                    float kf[EPC];
                    decode_word<KV>(raw.x, kf + 0 * EPW);
                    decode_word<KV>(raw.y, kf + 1 * EPW);
                    decode_word<KV>(raw.z, kf + 2 * EPW);
                    decode_word<KV>(raw.w, kf + 3 * EPW);
#pragma unroll
                    for (int hh = 0; hh < G; ++hh) {
#pragma unroll
                        for (int e = 0; e < EPC; e += 4) {
                            const float4 qv =
                                *reinterpret_cast<const float4 *>(sm_q + hh * D + ch * EPC + e);
                            dot[hh] = __ffma2_rn(make_float2(qv.x, qv.y),
                                                 make_float2(kf[e], kf[e + 1]), dot[hh]);
                            dot[hh] = __ffma2_rn(make_float2(qv.z, qv.w),
                                                 make_float2(kf[e + 2], kf[e + 3]), dot[hh]);
                        }
                    }
                }
                const bool valid = lane >= v_lo && lane < v_hi;
                float kscale = 1.f;
                if constexpr (QUANT) kscale = sm_scale[stage * 2 * kRows + lane];
#pragma unroll
                for (int hh = 0; hh < G; ++hh) {
                    float x = (dot[hh].x + dot[hh].y) * kscale;
                    if (a.soft_cap > 0.f) x = a.soft_cap * tanhf(x / a.soft_cap) * a.post_scale;
                    sc[hh] = valid ? x : -INFINITY;
                }
            }

            // ---------------- online softmax (exp2 domain), per head across the warp
            bool rescale = false;
            float alpha[G];
            float vscale = 1.f;
            if constexpr (QUANT) vscale = sm_scale[stage * 2 * kRows + kRows + lane];
#pragma unroll
            for (int hh = 0; hh < G; ++hh) {
                const float mx = warp_max(sc[hh]);
                const float mn = fmaxf(m[hh], mx);
                alpha[hh] = (mn == m[hh]) ? 1.f : fast_exp2(m[hh] - mn);
                rescale |= (mn != m[hh]);
                m[hh] = mn;
                const float mref = (mn == -INFINITY) ? 0.f : mn;
                const float p = fast_exp2(sc[hh] - mref);
                l[hh] = l[hh] * alpha[hh] + p;
                my_p[lane * G + hh] = p * vscale;
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
            for (int r = v_lo + half; r < v_hi; r += 2) {
                float vf[EPL];
                const int b0 = li * LANE_BYTES;
                if constexpr (LANE_BYTES >= 16) {
#pragma unroll
                    for (int k = 0; k < LANE_BYTES / 16; ++k) {
                        const uint4 raw = *reinterpret_cast<const uint4 *>(vt + swz(r, b0 + 16 * k));
                        decode_word<KV>(raw.x, vf + (4 * k + 0) * EPW);
                        decode_word<KV>(raw.y, vf + (4 * k + 1) * EPW);
                        decode_word<KV>(raw.z, vf + (4 * k + 2) * EPW);
                        decode_word<KV>(raw.w, vf + (4 * k + 3) * EPW);
                    }
                } else {
                    static_assert(LANE_BYTES == 8 || LANE_BYTES >= 16, "value-pass width");
                    const uint2 raw = *reinterpret_cast<const uint2 *>(vt + swz(r, b0));
                    decode_word<KV>(raw.x, vf + 0 * EPW);
                    decode_word<KV>(raw.y, vf + 1 * EPW);
                }
                float pv[G];
                if constexpr (G % 4 == 0) {
#pragma unroll
                    for (int hh = 0; hh < G; hh += 4) {
                        const float4 t = *reinterpret_cast<const float4 *>(my_p + r * G + hh);
                        pv[hh] = t.x;
                        pv[hh + 1] = t.y;
                        pv[hh + 2] = t.z;
                        pv[hh + 3] = t.w;
                    }
                } else {
#pragma unroll
                    for (int hh = 0; hh < G; ++hh) pv[hh] = my_p[r * G + hh];
                }
#pragma unroll
                for (int hh = 0; hh < G; ++hh) {
                    const float2 pp = make_float2(pv[hh], pv[hh]);
#pragma unroll
                    for (int e = 0; e < EPL / 2; ++e)
                        acc[hh][e] = __ffma2_rn(pp, make_float2(vf[2 * e], vf[2 * e + 1]), acc[hh][e]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[stage]);
        }

        // ---------------- merge the NC warp states of this item
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
        named_barrier(1, CONS);
        if (*cons_abort) break;  // a wait gave up in this CTA: stop cleanly

        const long long out_row = (static_cast<long long>(s) * Hkv + h) * G * D;
        const int slot_floats = 2 * G + G * D;
        float *part = nullptr;
        if (splits > 1)
            part = a.partials +
                   (static_cast<long long>(sm_prefix[s] + c) * Hkv + h) * slot_floats;
        for (int o = tid; o < G * D; o += CONS) {
            const int hh = o / D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NC; ++w) M = fmaxf(M, sm_comb[w * G * (D + 2) + hh]);
            float Ls = 0.f, As = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < NC; ++w) {
                    const float *cw = sm_comb + w * G * (D + 2);
                    const float mw = cw[hh];
                    const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
                    Ls += cw[G + hh] * f;
                    As += cw[2 * G + o] * f;
                }
            }
            if (splits == 1) {
                const float v = Ls > 0.f ? As * (1.0f / (Ls + a.norm_eps)) : 0.f;
                store_out(a.out, out_row + o, v, a.q_bf16);
            } else {
                part[2 * G + o] = As;
                if ((o % D) == 0) {
                    part[hh] = M;
                    part[G + hh] = Ls;
                }
            }
        }
        if (splits > 1) {
            __threadfence();
            named_barrier(1, CONS);
            if (tid == 0) {
                const int old = atomicAdd(&a.counters[s * Hkv + h], 1);
                sm_misc[1] = (old == splits - 1) ? 1 : 0;
            }
            named_barrier(1, CONS);
            if (sm_misc[1]) {
                __threadfence();
                const float *base = a.partials +
                                    (static_cast<long long>(sm_prefix[s]) * Hkv + h) * slot_floats;
                const long long step = static_cast<long long>(Hkv) * slot_floats;
                for (int o = tid; o < G * D; o += CONS) {
                    const int hh = o / D;
                    float M = -INFINITY;
                    for (int cc = 0; cc < splits; ++cc) M = fmaxf(M, __ldcg(base + cc * step + hh));
                    float Ls = 0.f, As = 0.f;
                    if (M != -INFINITY) {
                        for (int cc = 0; cc < splits; ++cc) {
                            const float *pc = base + cc * step;
                            const float mc = __ldcg(pc + hh);
                            const float f = (mc == -INFINITY) ? 0.f : fast_exp2(mc - M);
                            Ls += __ldcg(pc + G + hh) * f;
                            As += __ldcg(pc + 2 * G + o) * f;
                        }
                    }
                    const float v = Ls > 0.f ? As * (1.0f / (Ls + a.norm_eps)) : 0.f;
                    store_out(a.out, out_row + o, v, a.q_bf16);
                }
                if (tid == 0) atomicExch(&a.counters[s * Hkv + h], 0);
            }
        }
    }
}

}  // namespace gk
