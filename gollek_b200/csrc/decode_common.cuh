// decode_common.cuh -- what the persistent decode kernels share: the argument block,
// the token group (16 tokens; 32 in the int8 kernel) as the unit of work, and the
// stream-K schedule that cuts the groups of all (sequence, kv-head) pairs into one
// contiguous range per CTA.
//
// Linear group space: unit x = prefix[s] * Hkv + h * n_s + g, where n_s is the number
// of groups in sequence s's attention window and g the group within it.  CTA ranges
// are cut in cost space, where each (sequence, kv-head) costs its groups plus a run
// cost (kRunCost 16-token groups), so a CTA that starts many runs gets fewer groups.
// A range covers runs of consecutive groups of one (sequence, kv-head); a run that does
// not cover its whole (sequence, kv-head) is a split-K piece, merged by the CTA that
// finishes last.
#pragma once

#include "common.cuh"

namespace gk {

constexpr int kRows = 16;          // tokens per group (DecodeArgs::group_rows may be 32)
constexpr int kSlabBytes = kRows * 128;
constexpr int kMaxSplits = 64;     // split-K pieces per (sequence, kv-head) at most
constexpr int kMaxFastSeqs = 16384;
constexpr int kMinRunGroups = 8;   // smallest per-CTA range, in groups
constexpr int kMaxStagesPerWarp = 6;  // stage ring of one consumer warp, at most
// Cost of starting a run (a q load, a merge of the warp states, maybe a split-K
// exchange), in 16-token groups; CTAs are balanced on groups + kRunCost per run.
#ifndef GK_RUN_COST
#define GK_RUN_COST 16
#endif
constexpr int kRunCost = GK_RUN_COST;

struct DecodeArgs {
    void *out;
    const void *q;
    const float *k_scales;
    const float *v_scales;
    const int *block_tables;
    const int *context_lens;
    float *partials;   // split-K partial states: [(s*Hkv+h)*kMaxSplits + piece][2G + G*D]
    int *counters;     // [num_seqs * num_kv_heads] arrival counters, zero between calls
    long long page_rows;  // rows of head_dim elements between consecutive pages
    long long scale_page_stride, scale_head_stride, scale_token_stride;
    int num_seqs, num_kv_heads, block_size, max_blocks, num_blocks;
    int window;           // <= 0: no sliding window
    int q_bf16;           // 1: q/out bf16, 0: fp32
    int num_stages;       // stage ring length (tensor-memory kernel: K tiles)
    int num_vstages;      // tensor-memory kernel: V tiles
    int box3d;            // 1: one 3-D TMA box (all 128-byte slabs of 16 rows) per page
    int seq_div;          // block-table row of sequence s is s / seq_div (queries of one sequence)
    int qfold;            // > 1: the G rows of (s, h) are qfold queries x G/qfold heads of one
                          // chunk of seq_div chunks (qo_row); the chunk's query i < qfold sees
                          // the positions before len - (qfold - 1 - i)
    int group_rows;       // tokens per group: 16, or 32 (int8 kernel with 32-token stages)
    int scale_mode;       // int8: 0 per-token scales by bulk copy, 1 one scale per page, 2 general
    float q_scale;        // applied to q when staged: scale*log2(e), or scale with soft-cap
    float soft_cap;       // > 0: cap*tanh(score/cap)
    float post_scale;     // log2(e) with soft-cap, else 1
    float norm_eps;       // 1e-9 (engine path) or 0 (legacy fp32 path)
    unsigned wait_limit;  // bounded waits: try_waits / polls before giving up (0: the default)
    int fault_skip_group; // test only (-1 = off): CTA 0's producer never issues this CTA-local
                          // group, so the consumer's bounded wait for it gives up
};

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

// Row of q/out (in units of head_dim elements) holding row g of the G rows of (decode
// sequence v, kv-head h).  Decode: q/out [S, Hkv*G, D], row (v*Hkv + h)*G + g.  Folded
// multi-query (F = qfold > 1): sequence s has C = seq_div chunks v = s*C + c of F queries,
// the G rows of a chunk are its F queries x G/F heads, and q/out are [S, C*F, Hkv*G/F, D].
__device__ __forceinline__ long long qo_row(int v, int h, int g, int Hkv, int G, int F, int C) {
    if (F <= 1) return (static_cast<long long>(v) * Hkv + h) * G + g;
    const int gm = G / F;
    const int s = v / C;
    const int qi = g / gm;
    const int i = (v - s * C) * F + qi;
    return ((static_cast<long long>(s) * C * F + i) * Hkv + h) * gm + (g - qi * gm);
}

__device__ __forceinline__ void store_out(void *out, long long idx, float v, int bf16) {
    if (bf16)
        reinterpret_cast<__nv_bfloat16 *>(out)[idx] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float *>(out)[idx] = v;
}

// Window of one sequence: groups [g_lo, g_lo + n) of group_rows tokens cover
// [win_start, len).
struct SeqWin {
    int len, win_start, g_lo, n;
};

__device__ __forceinline__ SeqWin seq_win(const DecodeArgs &a, int s) {
    SeqWin w;
    int len = a.context_lens[s];
    const int cap = a.max_blocks * a.block_size;
    len = len < 0 ? 0 : (len > cap ? cap : len);
    w.len = len;
    w.win_start = (a.window > 0 && len > a.window) ? len - a.window : 0;
    const int gr = a.group_rows;
    w.g_lo = w.win_start / gr;
    w.n = len > 0 ? (len + gr - 1) / gr - w.g_lo : 0;
    return w;
}

// A run: the groups [g, g + len) of (sequence s, kv-head h) inside this CTA's range;
// piece / pieces: its split-K index and the number of CTAs sharing (s, h).
struct Run {
    int s, h, g, len, piece, pieces;
    long long sh_start, sh_end;
};

struct Schedule {
    const int *prefix;         // [S+1] exclusive prefix of window group counts (shared)
    const long long *rstart;   // [g_eff+1] CTA range starts (shared)
    int S, Hkv, g_eff;
    long long total, x_beg, x_end;

    // the CTA whose range holds group x: the last b with range_start(b) <= x
    __device__ __forceinline__ int owner(long long x) const {
        int lo = 0, hi = g_eff - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (rstart[mid] <= x)
                lo = mid;
            else
                hi = mid - 1;
        }
        return lo;
    }
    // the run holding unit x (clipped to this CTA's range); piece fields unset
    __device__ __forceinline__ Run run_at(long long x) const {
        Run r;
        int lo = 0, hi = S - 1;
        while (lo < hi) {  // last s with prefix[s]*Hkv <= x
            const int mid = (lo + hi + 1) >> 1;
            if (static_cast<long long>(prefix[mid]) * Hkv <= x)
                lo = mid;
            else
                hi = mid - 1;
        }
        r.s = lo;
        const int n = prefix[lo + 1] - prefix[lo];  // > 0: x lies inside sequence lo
        const int y = static_cast<int>(x - static_cast<long long>(prefix[lo]) * Hkv);
        r.h = y / n;
        r.g = y - r.h * n;
        const long long sh_start =
            static_cast<long long>(prefix[lo]) * Hkv + static_cast<long long>(r.h) * n;
        const long long sh_end = sh_start + n;
        r.len = static_cast<int>(min(sh_end, x_end) - x);
        r.sh_start = sh_start;
        r.sh_end = sh_end;
        return r;
    }
    __device__ __forceinline__ void pieces(Run &r) const {
        const int first = owner(r.sh_start);
        r.piece = static_cast<int>(blockIdx.x) - first;
        r.pieces = owner(r.sh_end - 1) - first + 1;
    }
};

// Builds the schedule in shared memory; every thread of the CTA calls it (it holds
// __syncthreads).  On entry *max_n == 0 is visible to all threads.  scratch: >= 64
// ints of shared memory, free until the function returns.  Raises BAD_POSITION for a
// context length outside [0, max_blocks * block_size] (then clamped).
__device__ inline Schedule schedule_prologue(const DecodeArgs &a, int *sm_prefix, int *sm_cprefix,
                                             int *sm_len, long long *sm_rstart, volatile int *max_n,
                                             int *scratch) {
    const int NT = blockDim.x;
    const int nwarps = NT >> 5;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int S = a.num_seqs;
    const int Hkv = a.num_kv_heads;
    const int run_cost = kRunCost * kRows / a.group_rows;  // in this launch's groups
    // Exclusive prefix of per-sequence group counts (contiguous segment per thread).
    {
        const int seg = (S + NT - 1) / NT;
        const int s0 = min(S, tid * seg);
        const int s1 = min(S, s0 + seg);
        int sum = 0, csum = 0, mx = 0;
        for (int s = s0; s < s1; ++s) {
            const int raw = a.context_lens[s];
            if (raw < 0 || raw > a.max_blocks * a.block_size) raise_status(GOLLEK_STATUS_BAD_POSITION);
            const SeqWin w0 = seq_win(a, s);
            sm_len[s] = w0.len;
            const int n = w0.n;
            sm_prefix[s] = n;
            sm_cprefix[s] = n > 0 ? n + run_cost : 0;
            sum += n;
            csum += n > 0 ? n + run_cost : 0;
            mx = max(mx, n);
        }
        int incl = sum, cincl = csum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            const int cv = __shfl_up_sync(0xffffffffu, cincl, o);
            if (lane >= o) {
                incl += v;
                cincl += cv;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        int *warp_tot = scratch;
        int *warp_ctot = scratch + 32;
        if (lane == 31) {
            warp_tot[warp] = incl;
            warp_ctot[warp] = cincl;
        }
        if (lane == 0) atomicMax(const_cast<int *>(max_n), mx);
        __syncthreads();
        if (tid == 0) {
            int run = 0, crun = 0;
            for (int w = 0; w < nwarps; ++w) {
                const int t = warp_tot[w], ct = warp_ctot[w];
                warp_tot[w] = run;
                warp_ctot[w] = crun;
                run += t;
                crun += ct;
            }
            sm_prefix[S] = run;
            sm_cprefix[S] = crun;
        }
        __syncthreads();
        int run = warp_tot[warp] + incl - sum;
        int crun = warp_ctot[warp] + cincl - csum;
        for (int s = s0; s < s1; ++s) {
            const int v = sm_prefix[s], cv = sm_cprefix[s];
            sm_prefix[s] = run;
            sm_cprefix[s] = crun;
            run += v;
            crun += cv;
        }
        __syncthreads();
    }
    Schedule sch;
    sch.prefix = sm_prefix;
    sch.rstart = sm_rstart;
    sch.S = S;
    sch.Hkv = Hkv;
    sch.total = static_cast<long long>(sm_prefix[S]) * Hkv;
    const long long tcost = static_cast<long long>(sm_cprefix[S]) * Hkv;
    long long per_cost = (tcost + gridDim.x - 1) / gridDim.x;
    const long long per_floor = (*max_n + kMaxSplits - 3) / (kMaxSplits - 2);
    if (per_cost < per_floor) per_cost = per_floor;
    if (per_cost < kMinRunGroups) per_cost = kMinRunGroups;
    sch.g_eff = static_cast<int>(min(static_cast<long long>(gridDim.x), (tcost + per_cost - 1) / per_cost));
    // group position where cost c falls (the run's first group for cost inside its
    // start-up share)
    auto x_of_cost = [&](long long c) -> long long {
        if (c >= tcost) return sch.total;
        int lo = 0, hi = S - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (static_cast<long long>(sm_cprefix[mid]) * Hkv <= c)
                lo = mid;
            else
                hi = mid - 1;
        }
        const int n = sm_prefix[lo + 1] - sm_prefix[lo];
        const int m = n + run_cost;
        const int y = static_cast<int>(c - static_cast<long long>(sm_cprefix[lo]) * Hkv);
        const int h = y / m;
        const int v = y - h * m;
        return static_cast<long long>(sm_prefix[lo]) * Hkv + static_cast<long long>(h) * n +
               (v > run_cost ? v - run_cost : 0);
    };
    for (int b = tid; b <= static_cast<int>(gridDim.x); b += NT)
        sm_rstart[b] = b >= sch.g_eff ? sch.total : x_of_cost(static_cast<long long>(b) * per_cost);
    __syncthreads();
    sch.x_beg = sm_rstart[blockIdx.x];
    sch.x_end = sm_rstart[blockIdx.x + 1];
    return sch;
}

}  // namespace gk
