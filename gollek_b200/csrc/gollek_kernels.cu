// gollek_kernels.cu -- host side of libgollek_kernels.so: argument checks, kernel
// selection, TMA descriptors, per-(device, stream) scratch and the C ABI declared
// in include/gollek_kernels.h.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <utility>

#include "common.cuh"
#include "decode_generic.cuh"
#include "decode_tc.cuh"
#include "decode_tma.cuh"
#include "kv_append.cuh"
#include "kv_migrate.cuh"
#include "prefill_tc.cuh"

namespace gk {
namespace {

thread_local std::string t_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    cudaGetLastError();  // clear a non-sticky error so the next call starts clean
    return fail(static_cast<int>(e), "%s: %s", what, cudaGetErrorString(e));
}

#define GK_CUDA(call, what)                        \
    do {                                           \
        cudaError_t e_ = (call);                   \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (dev >= 0 && dev != prev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// ----------------------------------------------------------- driver entry points

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        cudaGetLastError();
    });
    return g_encode;
}

PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
std::once_flag g_range_once;

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
    std::call_once(g_range_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
        cudaGetLastError();
    });
    return g_range;
}

// ------------------------------------------------------------------ device info

std::mutex g_mu;
std::map<int, int> g_sm_count;
// (device, stream, thread) -> scratch.  The thread is part of the key only for the
// per-thread default stream, whose handle is the same constant on every thread.
std::map<std::tuple<int, void *, size_t>, std::pair<void *, size_t>> g_ws;

int sm_count(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_sm_count.find(dev);
    if (it != g_sm_count.end()) return it->second;
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n;
    return n;
}

// Library-owned split-K scratch for (device, stream), zero-filled when (re)allocated;
// *cap_out receives its size.
int library_workspace(int dev, void *stream, size_t bytes, void **out, size_t *cap_out = nullptr) {
    const size_t tkey = stream == static_cast<void *>(cudaStreamPerThread)
                            ? std::hash<std::thread::id>()(std::this_thread::get_id())
                            : 0;
    std::lock_guard<std::mutex> lk(g_mu);
    auto &slot = g_ws[std::make_tuple(dev, stream, tkey)];
    if (slot.second < bytes) {
        if (slot.first) {
            cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
            cudaFree(slot.first);
            slot = {nullptr, 0};
        }
        void *p = nullptr;
        GK_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(split-K workspace)");
        GK_CUDA(cudaMemsetAsync(p, 0, bytes, static_cast<cudaStream_t>(stream)),
                "cudaMemsetAsync(split-K workspace)");
        slot = {p, bytes};
    }
    *out = slot.first;
    if (cap_out) *cap_out = slot.second;
    return GOLLEK_OK;
}

int dtype_bytes(int dt) {
    switch (dt) {
        case GOLLEK_DTYPE_F32:
            return 4;
        case GOLLEK_DTYPE_BF16:
        case GOLLEK_DTYPE_F16:
            return 2;
        case GOLLEK_DTYPE_I8:
            return 1;
        default:
            return 0;
    }
}

// Split-K scratch of W bytes: the arrival counters (int per (sequence, kv-head), zero
// between calls) fill the first W/128 bytes, the partial states follow.  The counter
// region depends on W alone, so one workspace can serve calls of any sizes: no call's
// partials ever land where another call's counters live.  Every call that fits in W has
// its counters inside the region (each (sequence, kv-head) needs >= 64 * 12 bytes of
// partials for its 4-byte counter).
size_t ws_counter_region(size_t W) { return (W / 128 + 255) / 256 * 256; }

size_t ws_partials_bytes(int S, int Hq, int Hkv, int D) {
    const int G = Hq / Hkv;
    const size_t slot = static_cast<size_t>(2 * G + G * D) * 4;
    return static_cast<size_t>(S) * Hkv * kMaxSplits * slot;
}

// Smallest W with ws_counter_region(W) + partials <= W.
size_t ws_bytes(int S, int Hq, int Hkv, int D) {
    const size_t P = ws_partials_bytes(S, Hq, Hkv, D);
    return P + P / 64 + 1024;
}

// Multi-query attention as decode: the Tq = C*F queries of sequence s (query i at
// absolute position ctx[s] - Tq + i, PagedAttentionVectorAPI.compute) become C decode
// sequences s*C + c of F queries each (F > 1: folded into the kernel's rows next to the
// GQA heads).  Chunk c's length is that of its last query, ctx[s] - Tq + (c+1)*F, when
// causal, ctx[s] otherwise.
__global__ void prefill_lengths_kernel(const int *ctx, int *lens, int S, int C, int F, int causal) {
    const long long n = static_cast<long long>(S) * C;
    const int Tq = C * F;
    for (long long v = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < n;
         v += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int s = static_cast<int>(v / C), c = static_cast<int>(v % C);
        const int x = ctx[s];
        lens[v] = (causal && x >= 0) ? max(0, x - Tq + (c + 1) * F) : x;  // negative stays: BAD_POSITION
    }
}

size_t prefill_lens_bytes(long long n) { return align_up(static_cast<uint32_t>(n * 4), 256u); }

// ------------------------------------------------------------------ fast path

constexpr uint32_t kSmemBudget = 224 * 1024;

struct Launch {
    const void *fn;
    int kv_bytes;
    bool quant;
};

// Consumer warps per CTA (one CTA per SM).  Nine, or twelve, warps in all put three on
// one SM sub-partition, whose register file then caps a thread at 168 registers; thirteen
// would cap it at 128 and spill.  16-bit KV compiles 8 and 7 consumer warps (the host
// takes the one with more stages in flight: 7 when G = 8, whose per-warp merge buffers
// crowd out stages), int8 and fp32 compile 11 and 8 (their consumers are latency-bound,
// so 11 unless its stages do not fit).
template <typename KV, int D, int G, int NC, bool SPLIT, int ROWS>
const void *fast_kernel() {
    return reinterpret_cast<const void *>(&decode_tma_kernel<KV, D, G, NC, SPLIT, ROWS>);
}

template <typename KV, int D, int NC, bool SPLIT, int ROWS = kRows>
const void *pick_g(int G) {
    switch (G) {
        case 1: return fast_kernel<KV, D, 1, NC, SPLIT, ROWS>();
        case 2: return fast_kernel<KV, D, 2, NC, SPLIT, ROWS>();
        case 4: return fast_kernel<KV, D, 4, NC, SPLIT, ROWS>();
        case 8: return fast_kernel<KV, D, 8, NC, SPLIT, ROWS>();
        default: return nullptr;
    }
}

// Consumer-warp counts compiled for a KV type and head_dim, in preference order.
struct NcList {
    int n;
    int v[2];
};
NcList nc_candidates(int kv, int D) {
    switch (kv) {
        case GOLLEK_DTYPE_BF16: return D == 128 ? NcList{2, {8, 7}} : NcList{1, {8, 0}};
        case GOLLEK_DTYPE_F16: return NcList{1, {8, 0}};
        case GOLLEK_DTYPE_I8:
        case GOLLEK_DTYPE_F32: return NcList{2, {11, 8}};
        default: return NcList{0, {0, 0}};
    }
}

// 16-bit KV computes on the tensor pipe; q wider than the MMA type (fp32 q, or any q
// with f16 KV) is split into hi + lo halves (SPLIT).  int8 KV is turned into f16 on the
// tensor pipe (fp32 q split); fp32 KV runs on packed FFMA.
const void *pick_fast(int kv, int D, int G, bool q_f32, int nc, int rows) {
    if (rows != kRows && kv != GOLLEK_DTYPE_I8) return nullptr;
    switch (kv) {
        case GOLLEK_DTYPE_BF16:
            if (D == 128) {
                if (nc == 8) return q_f32 ? pick_g<__nv_bfloat16, 128, 8, true>(G) : pick_g<__nv_bfloat16, 128, 8, false>(G);
                if (nc == 7) {
                    // 16 rows (folded multi-query calls): 7 consumer warps only, so that no
                    // SM sub-partition holds three warps and a thread may use 255 registers
                    if (G == 16)
                        return q_f32 ? fast_kernel<__nv_bfloat16, 128, 16, 7, true, kRows>()
                                     : fast_kernel<__nv_bfloat16, 128, 16, 7, false, kRows>();
                    return q_f32 ? pick_g<__nv_bfloat16, 128, 7, true>(G) : pick_g<__nv_bfloat16, 128, 7, false>(G);
                }
                return nullptr;
            }
            if (D == 64 && nc == 8)
                return q_f32 ? pick_g<__nv_bfloat16, 64, 8, true>(G) : pick_g<__nv_bfloat16, 64, 8, false>(G);
            return nullptr;
        case GOLLEK_DTYPE_F16:
            if (nc != 8) return nullptr;
            return D == 128 ? pick_g<__half, 128, 8, true>(G) : D == 64 ? pick_g<__half, 64, 8, true>(G) : nullptr;
        case GOLLEK_DTYPE_F32:
            if (nc == 11) return D == 128 ? pick_g<float, 128, 11, false>(G) : D == 64 ? pick_g<float, 64, 11, false>(G) : nullptr;
            if (nc == 8) return D == 128 ? pick_g<float, 128, 8, false>(G) : D == 64 ? pick_g<float, 64, 8, false>(G) : nullptr;
            return nullptr;
        case GOLLEK_DTYPE_I8:
            if (D != 128) return nullptr;
            if (rows == 32) {
                if (q_f32) return nullptr;
                if (nc == 11) return pick_g<int8_t, 128, 11, false, 32>(G);
                if (nc == 8) return pick_g<int8_t, 128, 8, false, 32>(G);
                return nullptr;
            }
            if (nc == 11) return q_f32 ? pick_g<int8_t, 128, 11, true>(G) : pick_g<int8_t, 128, 11, false>(G);
            if (nc == 8) return q_f32 ? pick_g<int8_t, 128, 8, true>(G) : pick_g<int8_t, 128, 8, false>(G);
            return nullptr;
        default:
            return nullptr;
    }
}

CUtensorMapDataType tma_type(int kv) {
    switch (kv) {
        case GOLLEK_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        case GOLLEK_DTYPE_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        case GOLLEK_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct V2 {
    void *out;
    const void *q, *k, *v;
    const float *ks, *vs;
    const int *bt, *ctx;
    int S, Hq, Hkv, D, BS, maxB, num_blocks;
    long long page_stride;
    int q_dtype, kv_dtype;
    long long sps, shs, sts;
    float scale, soft_cap;
    int window;
    float norm_eps;
    void *workspace;
    size_t workspace_bytes;
    void *stream;
    int seq_div;  // > 1: S counts (sequence, query) pairs, block-table row = s / seq_div
    int qfold;    // > 1: folded multi-query call, Hq counts qfold queries x the model's q heads
};

int encode_map(CUtensorMap *m, const void *base, int kv, int D, long long rows, int box_rows) {
    auto enc = encode_fn();
    if (!enc) return fail(GOLLEK_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    const int eb = dtype_bytes(kv);
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * eb};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / eb), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, tma_type(kv), 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GOLLEK_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GOLLEK_OK;
}

// 4-D map over a bf16 pool with head_dim 128 for the tensor-memory kernel: (64 columns,
// 8 rows, 2 column slabs, 8-row blocks), strides 256 B / 128 B / 2 KB, so one box of
// (64, 8, 2, box_rows/8) lands as [row block][slab][8 rows][128 B] in the 128-byte swizzle.
int encode_map4(CUtensorMap *m, const void *base, long long rows, int box_rows) {
    auto enc = encode_fn();
    if (!enc) return fail(GOLLEK_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[4] = {64, 8, 2, static_cast<cuuint64_t>(rows / 8)};
    cuuint64_t strides[3] = {256, 128, 2048};
    cuuint32_t box[4] = {64, 8, 2, static_cast<cuuint32_t>(box_rows / 8)};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GOLLEK_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled (4-D) failed (%d)", (int)r);
    return GOLLEK_OK;
}

// 3-D map for the mma.sync kernel: (128-byte column slab, row, slab index), strides row
// pitch / 128 B, box (128 B, 16 rows, all slabs): one box lands as [slab][16 rows][128 B],
// the kernel's stage layout.
int encode_map3(CUtensorMap *m, const void *base, int kv, int D, long long rows) {
    auto enc = encode_fn();
    if (!enc) return fail(GOLLEK_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    const int eb = dtype_bytes(kv);
    const int nslab = D * eb / 128;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(128 / eb), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(nslab)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * eb, 128};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / eb), static_cast<cuuint32_t>(kRows),
                         static_cast<cuuint32_t>(nslab)};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, tma_type(kv), 3, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GOLLEK_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return GOLLEK_OK;
}

// Tokens per group and stage of the mma.sync kernel: int8 KV (head_dim 128) with bf16 q
// and pages of at least 16 tokens moves 32-token groups, so that a stage holds as many
// bytes as a 16-bit one and the per-group costs (block-table lookup, barriers, softmax
// update) are paid half as often; everything else 16 (fp32 q's hi + lo fragments would
// push 32-token groups past the register budget).
int group_rows(const V2 &p) {
    return (p.kv_dtype == GOLLEK_DTYPE_I8 && p.D == 128 && p.BS >= 16 &&
            p.q_dtype == GOLLEK_DTYPE_BF16) ? 32 : kRows;
}

// Layout conditions shared by the TMA kernels (page tiles, alignment, sizes).
bool tma_layout_ok(const V2 &p, long long page_stride) {
    const int eb = dtype_bytes(p.kv_dtype);
    if (eb == 0) return false;
    const bool bs_ok = (p.BS >= 8 && p.BS <= 32 && 32 % p.BS == 0) || (p.BS > 32 && p.BS % 32 == 0);
    if (!bs_ok) return false;
    if (!aligned16(p.k) || !aligned16(p.v)) return false;
    if (page_stride % p.D != 0 || (page_stride * eb) % 16 != 0) return false;
    if (p.S > kMaxFastSeqs) return false;
    if (p.kv_dtype == GOLLEK_DTYPE_I8 && (!p.ks || !p.vs)) return false;
    if (p.kv_dtype == GOLLEK_DTYPE_I8 && !aligned16(p.q)) return false;  // 16-byte q loads
    if (p.q_dtype != GOLLEK_DTYPE_F32 && p.q_dtype != GOLLEK_DTYPE_BF16) return false;
    const long long rows_per_page = page_stride / p.D;
    if (p.num_blocks > 0 && static_cast<long long>(p.num_blocks) * rows_per_page >= (1LL << 31))
        return false;
    return true;
}

// Eligibility of the mma.sync TMA kernel; returns the function of its first compiled
// warp count or nullptr.
const void *fast_eligible(const V2 &p, int G, long long page_stride) {
    if (!tma_layout_ok(p, page_stride)) return nullptr;
    if (G > 8 && p.qfold <= 1) return nullptr;  // 16-row kernels serve folded multi-query calls
    const NcList c = nc_candidates(p.kv_dtype, p.D);
    for (int i = 0; i < c.n; ++i)
        if (const void *f = pick_fast(p.kv_dtype, p.D, G, p.q_dtype == GOLLEK_DTYPE_F32, c.v[i], group_rows(p)))
            return f;
    return nullptr;
}

// Split-K scratch: the caller's workspace, or the library's per (device, stream) one;
// *cap receives its size (which fixes where the partials start).
int v2_workspace(const V2 &p, int dev, void **ws, size_t *cap) {
    *ws = p.workspace;
    *cap = p.workspace_bytes;
    const size_t need = ws_bytes(p.S, p.Hq, p.Hkv, p.D);
    if (*ws) {
        if (p.workspace_bytes < need)
            return fail(GOLLEK_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed", p.workspace_bytes, need);
        return GOLLEK_OK;
    }
    return library_workspace(dev, p.stream, need, ws, cap);
}

// 2-D tensor maps over the K and V pools: rows of head_dim elements, boxes of 128 bytes
// x min(block_size, group rows) rows.
int v2_maps(const V2 &p, long long page_stride, int group, CUtensorMap *tmk, CUtensorMap *tmv) {
    const long long rows_per_page = page_stride / p.D;
    const long long rows =
        p.num_blocks > 0 ? static_cast<long long>(p.num_blocks) * rows_per_page : (1LL << 31) - 1;
    const int box_rows = p.BS < group ? p.BS : group;
    int rc = encode_map(tmk, p.k, p.kv_dtype, p.D, rows, box_rows);
    if (!rc) rc = encode_map(tmv, p.v, p.kv_dtype, p.D, rows, box_rows);
    return rc;
}

DecodeArgs v2_args(const V2 &p, void *ws, size_t ws_cap, long long page_stride, int stages,
                   int group = kRows) {
    const bool cap = p.soft_cap > 0.f;
    DecodeArgs a;
    a.out = p.out;
    a.q = p.q;
    a.k_scales = p.ks;
    a.v_scales = p.vs;
    a.block_tables = p.bt;
    a.context_lens = p.ctx;
    a.counters = static_cast<int *>(ws);
    a.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + ws_counter_region(ws_cap));
    a.page_rows = page_stride / p.D;
    a.scale_page_stride = p.sps;
    a.scale_head_stride = p.shs;
    a.scale_token_stride = p.sts;
    a.num_seqs = p.S;
    a.num_kv_heads = p.Hkv;
    a.block_size = p.BS;
    a.max_blocks = p.maxB;
    a.num_blocks = p.num_blocks;
    a.window = p.window;
    a.q_bf16 = p.q_dtype == GOLLEK_DTYPE_BF16;
    a.num_stages = stages;
    a.num_vstages = 0;
    a.box3d = 0;
    a.seq_div = p.seq_div > 1 ? p.seq_div : 1;
    a.qfold = p.qfold > 1 ? p.qfold : 1;
    a.group_rows = group;
    a.scale_mode = 2;
    if (p.kv_dtype == GOLLEK_DTYPE_I8) {
        const int R = p.BS < group ? p.BS : group;
        if (p.sts == 1 && (p.sps * 4) % 16 == 0 && (p.shs * 4) % 16 == 0 && aligned16(p.ks) &&
            aligned16(p.vs) && (R * 4) % 16 == 0)
            a.scale_mode = 0;
        else if (p.sts == 0)
            a.scale_mode = 1;
    }
    a.q_scale = cap ? p.scale : p.scale * kLog2e;
    a.soft_cap = p.soft_cap;
    a.post_scale = cap ? kLog2e : 1.f;
    a.norm_eps = p.norm_eps;
    // Test hooks of the failure-detection tests (unset in normal use): a short bound for the
    // kernels' waits, and one group of CTA 0 whose copies are never issued.
    const char *wl = std::getenv("GOLLEK_TEST_WAIT_LIMIT");
    const char *sk = std::getenv("GOLLEK_TEST_SKIP_GROUP");
    a.wait_limit = wl ? static_cast<unsigned>(std::strtoul(wl, nullptr, 10)) : 0u;
    a.fault_skip_group = sk ? std::atoi(sk) : -1;
    return a;
}

// Which decode kernel serves bf16 KV: GOLLEK_DECODE_PATH = "auto" (default: the mma.sync
// kernel, and the tensor-memory kernel for what it alone covers, GQA groups of 16), "tc"
// (the tensor-memory kernel wherever it applies) or "mma" (never the tensor-memory kernel).
enum class DecodePath { kAuto, kTc, kMma };
DecodePath decode_path() {
    const char *e = std::getenv("GOLLEK_DECODE_PATH");
    if (e && std::strcmp(e, "tc") == 0) return DecodePath::kTc;
    if (e && std::strcmp(e, "mma") == 0) return DecodePath::kMma;
    return DecodePath::kAuto;
}

template <int G, bool SPLIT>
const void *tc_kernel() {
    return reinterpret_cast<const void *>(&decode_tc_kernel<G, SPLIT>);
}

const void *pick_tc(int G, bool split) {
    switch (G) {
        case 1: return split ? tc_kernel<1, true>() : tc_kernel<1, false>();
        case 2: return split ? tc_kernel<2, true>() : tc_kernel<2, false>();
        case 4: return split ? tc_kernel<4, true>() : tc_kernel<4, false>();
        case 8: return split ? tc_kernel<8, true>() : tc_kernel<8, false>();
        case 16: return split ? tc_kernel<16, true>() : tc_kernel<16, false>();
        default: return nullptr;
    }
}

constexpr int kNotTaken = 1 << 30;

// The tcgen05 kernel (bf16 KV, head_dim 128, GQA group 1-16): launches it, or returns
// kNotTaken when the case is outside its range.
int try_tc(const V2 &p, int dev, int G, long long page_stride) {
    const DecodePath mode = decode_path();
    if (p.qfold > 1) return kNotTaken;  // folded queries: the mma.sync kernel only
    if (mode == DecodePath::kMma || p.kv_dtype != GOLLEK_DTYPE_BF16 || p.D != 128) return kNotTaken;
    if (mode == DecodePath::kAuto && fast_eligible(p, G, page_stride)) return kNotTaken;
    if (!tma_layout_ok(p, page_stride) || !aligned16(p.q)) return kNotTaken;
    const bool split = p.q_dtype == GOLLEK_DTYPE_F32;
    const void *fn = pick_tc(G, split);
    if (!fn) return kNotTaken;
    const long long rows_per_page = page_stride / p.D;
    if (rows_per_page % 8 != 0) return kNotTaken;
    const int ctas = sm_count(dev);
    // K / V ring lengths in 32 KB tiles: V tiles are held longer (until the probabilities
    // exist), so they get the larger ring
    static const int kRings[][2] = {{2, 4}, {2, 3}, {1, 3}, {2, 2}, {1, 2}};
    int nk = 0, nv = 0;
    TcSmem L{};
    for (const auto &rg : kRings) {
        L = tc_smem_layout(rg[0], rg[1], split, p.S, ctas);
        if (L.total <= 227 * 1024) {
            nk = rg[0];
            nv = rg[1];
            break;
        }
    }
    if (!nk) return kNotTaken;
    void *ws = nullptr;
    size_t ws_cap = 0;
    int rc = v2_workspace(p, dev, &ws, &ws_cap);
    if (rc) return rc;
    const long long rows =
        p.num_blocks > 0 ? static_cast<long long>(p.num_blocks) * rows_per_page : (1LL << 31) - 8;
    const int box_rows = p.BS < kRows ? p.BS : kRows;
    CUtensorMap tmk, tmv;
    rc = encode_map4(&tmk, p.k, rows, box_rows);
    if (!rc) rc = encode_map4(&tmv, p.v, rows, box_rows);
    if (rc) return rc;
    DecodeArgs a = v2_args(p, ws, ws_cap, page_stride, nk);
    a.num_vstages = nv;
    GK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total),
            "cudaFuncSetAttribute");
    void *args[] = {&tmk, &tmv, &a};
    GK_CUDA(cudaLaunchKernel(fn, dim3(ctas), dim3(kTcThreads), args, L.total,
                             static_cast<cudaStream_t>(p.stream)),
            "decode_tc_kernel launch");
    return GOLLEK_OK;
}

// 32 or 64 rows per (sequence or chunk, kv-head) unit with bf16 KV and bf16 q, head_dim
// 128 -- folded multi-query calls (F queries x G heads), and decode with G = 32 or 64 q
// heads per kv head (multi-query-attention models) -- on the tensor-memory kernel whose MMA
// rows are those rows (prefill_tc.cuh), so one pass over the pages serves up to 64 rows.
// GOLLEK_PREFILL_TC=0 (read per call) leaves folded calls to the 16-row mma.sync kernel;
// decode with such groups has no other kernel (GOLLEK_ERR_UNSUPPORTED without this one).
bool prefill_tc_enabled() {
    const char *e = std::getenv("GOLLEK_PREFILL_TC");
    return !(e && e[0] == '0');
}

// Two warps per 32 rows, one per half of a tile's tokens (prefill_tc_kernel<G, true>):
// 0.339 against 0.503 ms at Tq = 16 on config 2's pool.  GOLLEK_PREFILL_TC_HALVES=0 (read
// per call) selects one warp per 32 rows.
bool prefill_tc_halves() {
    const char *e = std::getenv("GOLLEK_PREFILL_TC_HALVES");
    return !(e && e[0] == '0');
}

int try_prefill_tc(const V2 &p, int dev, int G, long long page_stride) {
    if (!prefill_tc_enabled()) return kNotTaken;
    // (folded calls come without a window; decode may have one)
    if (p.kv_dtype != GOLLEK_DTYPE_BF16 || p.q_dtype != GOLLEK_DTYPE_BF16 || p.D != 128) return kNotTaken;
    if (G != 32 && G != 64) return kNotTaken;
    if (!tma_layout_ok(p, page_stride) || !aligned16(p.q) || !aligned16(p.out)) return kNotTaken;
    const long long rows_per_page = page_stride / p.D;
    if (rows_per_page % 8 != 0) return kNotTaken;
    const int ctas = sm_count(dev);
    // the largest rings that fit, two warps per 32 rows first; their hand-over area costs
    // 2 * G floats, so a call with slightly more sequences runs the one-warp form
    static const int kRings[][2] = {{2, 3}, {2, 2}, {1, 2}};
    int nk = 0, nv = 0;
    PtSmem L{};
    bool halves = prefill_tc_halves();
    for (int form = 0; form < 2 && !nk; ++form) {
        if (form == 1) {
            if (!halves) break;
            halves = false;
        }
        for (const auto &rg : kRings) {
            L = pt_smem_layout(G, rg[0], rg[1], p.S, ctas, halves);
            if (L.total <= 227 * 1024) {
                nk = rg[0];
                nv = rg[1];
                break;
            }
        }
    }
    if (!nk) return kNotTaken;
    const void *fn = G == 64 ? (halves ? reinterpret_cast<const void *>(&prefill_tc_kernel<64, true>)
                                       : reinterpret_cast<const void *>(&prefill_tc_kernel<64>))
                             : (halves ? reinterpret_cast<const void *>(&prefill_tc_kernel<32, true>)
                                       : reinterpret_cast<const void *>(&prefill_tc_kernel<32>));
    void *ws = nullptr;
    size_t ws_cap = 0;
    int rc = v2_workspace(p, dev, &ws, &ws_cap);
    if (rc) return rc;
    const long long rows =
        p.num_blocks > 0 ? static_cast<long long>(p.num_blocks) * rows_per_page : (1LL << 31) - 8;
    const int box_rows = p.BS < kRows ? p.BS : kRows;
    CUtensorMap tmk, tmv;
    rc = encode_map4(&tmk, p.k, rows, box_rows);
    if (!rc) rc = encode_map4(&tmv, p.v, rows, box_rows);
    if (rc) return rc;
    DecodeArgs a = v2_args(p, ws, ws_cap, page_stride, nk);
    a.num_vstages = nv;
    GK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total),
            "cudaFuncSetAttribute");
    void *args[] = {&tmk, &tmv, &a};
    GK_CUDA(cudaLaunchKernel(fn, dim3(ctas), dim3(kPtThreads), args, L.total,
                             static_cast<cudaStream_t>(p.stream)),
            "prefill_tc_kernel launch");
    return GOLLEK_OK;
}

// int8 KV over 16-token pages in kv-head pairs (decode_tma_kernel<..., PAIR>): one 4 KB TMA
// box per page holds both heads of a pair, so the copy path moves twice the bytes per box.
// Needs bf16 q, an even number of kv heads, decode (no folded queries), and per-token scales
// whose two heads are adjacent (head stride == block size) or per-page scales.
// GOLLEK_I8_PAIR=0 (read per call) keeps the one-head-per-stage kernel.
constexpr int kPairWarps = 10;

template <int G>
const void *pair_kernel() {
    return reinterpret_cast<const void *>(&decode_tma_kernel<int8_t, 128, G, kPairWarps, false, 32, true>);
}

const void *pick_pair(int G) {
    switch (G) {
        case 1: return pair_kernel<1>();
        case 2: return pair_kernel<2>();
        case 4: return pair_kernel<4>();
        case 8: return pair_kernel<8>();
        default: return nullptr;
    }
}

int try_pair(const V2 &p, int dev, int G, long long page_stride) {
    const char *e = std::getenv("GOLLEK_I8_PAIR");
    if (e && std::strcmp(e, "0") == 0) return kNotTaken;
    if (p.kv_dtype != GOLLEK_DTYPE_I8 || p.D != 128 || p.BS != 16 || p.q_dtype != GOLLEK_DTYPE_BF16)
        return kNotTaken;
    if (p.qfold > 1 || p.Hkv % 2 != 0 || group_rows(p) != 32) return kNotTaken;
    if (!tma_layout_ok(p, page_stride)) return kNotTaken;
    const bool per_token = p.sts == 1 && p.shs == p.BS && (p.sps * 4) % 16 == 0 && (p.shs * 4) % 16 == 0 &&
                           aligned16(p.ks) && aligned16(p.vs);
    if (!per_token && p.sts != 0) return kNotTaken;
    const void *fn = pick_pair(G);
    if (!fn) return kNotTaken;
    constexpr int kTrows = 64;  // 2 pages x 2 heads x 16 rows per K (or V) tile
    const uint32_t tile = kTrows * 128;
    const int max_ctas = sm_count(dev) * 2;
    const int np = kPairWarps / 2;
    DecodeSmem L0 = decode_smem_layout(1, true, p.D, G, kPairWarps, 0, p.S, max_ctas, kTrows);
    int spw = static_cast<int>((kSmemBudget > L0.total ? kSmemBudget - L0.total : 0) / (2 * tile * np));
    spw = std::min(spw, kMaxStagesPerWarp);
    if (spw < 1) return kNotTaken;
    const int stages = spw * np;
    DecodeSmem L = decode_smem_layout(1, true, p.D, G, kPairWarps, stages, p.S, max_ctas, kTrows);
    if (L.total > 227 * 1024 || L.q % 16 || L.p % 16 || L.scales % 16 || L.rstart % 8 || L.bars % 8)
        return kNotTaken;
    void *ws = nullptr;
    size_t ws_cap = 0;
    int rc = v2_workspace(p, dev, &ws, &ws_cap);
    if (rc) return rc;
    const long long rows_per_page = page_stride / p.D;
    const long long rows =
        p.num_blocks > 0 ? static_cast<long long>(p.num_blocks) * rows_per_page : (1LL << 31) - 1;
    CUtensorMap tmk, tmv;
    rc = encode_map(&tmk, p.k, p.kv_dtype, p.D, rows, 2 * p.BS);
    if (!rc) rc = encode_map(&tmv, p.v, p.kv_dtype, p.D, rows, 2 * p.BS);
    if (rc) return rc;
    DecodeArgs a = v2_args(p, ws, ws_cap, page_stride, stages, 32);
    a.num_kv_heads = p.Hkv / 2;  // units are kv-head pairs
    a.box3d = 0;
    a.scale_mode = per_token ? 0 : 1;
    GK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total),
            "cudaFuncSetAttribute");
    const int grid = sm_count(dev);
    void *args[] = {&tmk, &tmv, &a};
    GK_CUDA(cudaLaunchKernel(fn, dim3(grid), dim3((kPairWarps + 1) * 32), args, L.total,
                             static_cast<cudaStream_t>(p.stream)),
            "decode_tma_kernel (kv-head pairs) launch");
    return GOLLEK_OK;
}

int run_v2(const V2 &p) {
    int dev = 0;
    GK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    const int G = p.Hq / p.Hkv;
    const long long page_stride =
        p.page_stride > 0 ? p.page_stride : static_cast<long long>(p.Hkv) * p.BS * p.D;
    const float log2e = kLog2e;
    const bool cap = p.soft_cap > 0.f;
    cudaStream_t st = static_cast<cudaStream_t>(p.stream);
    if (p.S == 0) return GOLLEK_OK;

    {
        const int rc = try_prefill_tc(p, dev, G, page_stride);
        if (rc != kNotTaken) return rc;
    }
    {
        const int rc = try_tc(p, dev, G, page_stride);
        if (rc != kNotTaken) return rc;
    }
    {
        const int rc = try_pair(p, dev, G, page_stride);
        if (rc != kNotTaken) return rc;
    }
    const void *fn = fast_eligible(p, G, page_stride);
    if (fn) {
        const int eb = dtype_bytes(p.kv_dtype);
        const bool quant = p.kv_dtype == GOLLEK_DTYPE_I8;
        const int rows = group_rows(p);
        const uint32_t tile = static_cast<uint32_t>(p.D * eb / 128) * rows * 128;
        const int max_ctas = sm_count(dev) * 2;
        // warp count: 16-bit KV takes the candidate with the most stages in flight, int8
        // and fp32 the first that fits
        const NcList cand = nc_candidates(p.kv_dtype, p.D);
        const bool most_stages = eb == 2;
        int nc = 0, stages = 0;
        DecodeSmem L{};
        fn = nullptr;
        for (int ci = 0; ci < cand.n; ++ci) {
            const int c = cand.v[ci];
            const void *f = pick_fast(p.kv_dtype, p.D, G, p.q_dtype == GOLLEK_DTYPE_F32, c, rows);
            if (!f) continue;
            DecodeSmem L0 = decode_smem_layout(eb, quant, p.D, G, c, 0, p.S, max_ctas, rows);
            int spw = static_cast<int>((kSmemBudget > L0.total ? kSmemBudget - L0.total : 0) / (2 * tile * c));
            spw = std::min(std::max(spw, 1), kMaxStagesPerWarp);
            DecodeSmem Lc = decode_smem_layout(eb, quant, p.D, G, c, spw * c, p.S, max_ctas, rows);
            if (Lc.total > 227 * 1024) continue;
            // TMA and bulk-copy destinations and vector accesses need these alignments
            if (Lc.q % 16 || Lc.p % 16 || Lc.scales % 16 || Lc.rstart % 8 || Lc.bars % 8) continue;
            if (!fn || (most_stages && spw * c > stages)) {
                fn = f;
                nc = c;
                stages = spw * c;
                L = Lc;
                if (!most_stages) break;
            }
        }
        if (fn) {
            void *ws = nullptr;
            size_t ws_cap = 0;
            int rc = v2_workspace(p, dev, &ws, &ws_cap);
            if (rc) return rc;
            CUtensorMap tmk, tmv;
            const bool box3d = rows == kRows && p.BS >= kRows && p.D * eb >= 256;
            if (box3d) {
                const long long rows = p.num_blocks > 0 ? static_cast<long long>(p.num_blocks) * (page_stride / p.D)
                                                        : (1LL << 31) - 1;
                rc = encode_map3(&tmk, p.k, p.kv_dtype, p.D, rows);
                if (!rc) rc = encode_map3(&tmv, p.v, p.kv_dtype, p.D, rows);
            } else {
                rc = v2_maps(p, page_stride, rows, &tmk, &tmv);
            }
            if (rc) return rc;
            DecodeArgs a = v2_args(p, ws, ws_cap, page_stride, stages, rows);
            a.box3d = box3d ? 1 : 0;

            GK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total),
                    "cudaFuncSetAttribute");
            int per_sm = 0;
            GK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, (nc + 1) * 32, L.total),
                    "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
            if (per_sm < 1) per_sm = 1;
            const int grid = std::min(sm_count(dev) * per_sm, max_ctas);  // smem sized for max_ctas
            void *args[] = {&tmk, &tmv, &a};
            GK_CUDA(cudaLaunchKernel(fn, dim3(grid), dim3((nc + 1) * 32), args, L.total, st),
                    "decode_tma_kernel launch");
            return GOLLEK_OK;
        }
    }

    // Folded multi-query calls run on the mma.sync kernel or not at all (the caller then
    // runs the queries as separate decode sequences).
    if (p.qfold > 1) return kNotTaken;
    // Generic kernel.
    if (G > kGenMaxG || p.D > kGenMaxJ * 32)
        return fail(GOLLEK_ERR_UNSUPPORTED, "head_dim %d / GQA group %d outside the supported range",
                    p.D, G);
    GenericArgs g;
    g.out = p.out;
    g.q = p.q;
    g.k = p.k;
    g.v = p.v;
    g.k_scales = p.ks;
    g.v_scales = p.vs;
    g.block_tables = p.bt;
    g.context_lens = p.ctx;
    g.page_stride = page_stride;
    g.scale_page_stride = p.sps;
    g.scale_head_stride = p.shs;
    g.scale_token_stride = p.sts;
    g.num_q_heads = p.Hq;
    g.num_kv_heads = p.Hkv;
    g.head_dim = p.D;
    g.block_size = p.BS;
    g.max_blocks = p.maxB;
    g.num_blocks = p.num_blocks;
    g.window = p.window;
    g.q_bf16 = p.q_dtype == GOLLEK_DTYPE_BF16;
    g.kv_dtype = p.kv_dtype;
    g.seq_div = p.seq_div > 1 ? p.seq_div : 1;
    g.q_scale = cap ? p.scale : p.scale * log2e;
    g.soft_cap = p.soft_cap;
    g.post_scale = cap ? log2e : 1.f;
    g.norm_eps = p.norm_eps;
    decode_generic_kernel<<<dim3(p.S, p.Hkv), kGenWarps * 32, 0, st>>>(g);
    GK_CUDA(cudaGetLastError(), "decode_generic_kernel launch");
    return GOLLEK_OK;
}

int check_v2(const V2 &p) {
    if (!p.out || !p.q || !p.k || !p.v || !p.bt || !p.ctx)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (p.S < 0 || p.Hq <= 0 || p.Hkv <= 0 || p.D <= 0 || p.BS <= 0 || p.maxB <= 0 || p.num_blocks < 0)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "non-positive size");
    if (p.Hq % p.Hkv != 0)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "num_q_heads %d not a multiple of num_kv_heads %d",
                    p.Hq, p.Hkv);
    if (p.q_dtype != GOLLEK_DTYPE_F32 && p.q_dtype != GOLLEK_DTYPE_BF16)
        return fail(GOLLEK_ERR_UNSUPPORTED, "q dtype %d (F32 or BF16 only)", p.q_dtype);
    if (p.kv_dtype < GOLLEK_DTYPE_F32 || p.kv_dtype > GOLLEK_DTYPE_I4)
        return fail(GOLLEK_ERR_UNSUPPORTED, "kv dtype %d", p.kv_dtype);
    if ((p.kv_dtype == GOLLEK_DTYPE_I8 || p.kv_dtype == GOLLEK_DTYPE_I4) && (!p.ks || !p.vs))
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "quantised KV needs k_scales and v_scales");
    const long long minimal = static_cast<long long>(p.Hkv) * p.BS * p.D;
    if (p.page_stride != 0 && p.page_stride < minimal)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "page_stride %lld < num_kv_heads*block_size*head_dim",
                    p.page_stride);
    if (static_cast<long long>(p.maxB) * p.BS > (1LL << 30))
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "max_blocks_per_seq * block_size too large");
    return GOLLEK_OK;
}

// After a wait gave up (GOLLEK_STATUS_TIMEOUT) a split-K arrival counter may have been
// left non-zero; zero the counter regions of this device's library-owned workspaces.
// Called with the device current and idle (after a synchronize).
int rezero_library_counters(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto &kv : g_ws) {
        if (std::get<0>(kv.first) != dev || !kv.second.first) continue;
        GK_CUDA(cudaMemset(kv.second.first, 0, ws_counter_region(kv.second.second)),
                "cudaMemset(split-K counters after a timeout)");
    }
    return GOLLEK_OK;
}

int read_and_clear_status(cudaStream_t st, unsigned *out) {
    unsigned v = 0;
    GK_CUDA(cudaMemcpyFromSymbolAsync(&v, g_status, sizeof(v), 0, cudaMemcpyDeviceToHost, st),
            "read status");
    GK_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (v) {
        const unsigned zero = 0;
        GK_CUDA(cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st),
                "clear status");
        GK_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    }
    if (v & GOLLEK_STATUS_TIMEOUT) {
        int dev = 0;
        GK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
        GK_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        const int rc = rezero_library_counters(dev);
        if (rc) return rc;
    }
    *out = v;
    return GOLLEK_OK;
}

int status_to_code(unsigned v) {
    if (v & GOLLEK_STATUS_TIMEOUT) return fail(GOLLEK_ERR_TIMEOUT, "a device-side wait gave up");
    if (v & GOLLEK_STATUS_BAD_BLOCK_ID)
        return fail(GOLLEK_ERR_BAD_BLOCK_ID, "block table entry outside the pool");
    if (v & GOLLEK_STATUS_BAD_POSITION)
        return fail(GOLLEK_ERR_BAD_POSITION, "context length or position beyond the block table");
    return GOLLEK_OK;
}

// ------------------------------------------------------------ no-alloc scratch

// Split-K scratch of gollek_paged_attention_v2_noalloc: a static device array, so that
// entry point never allocates.  Host code cannot use the array's name as a device
// address; noalloc_scratch() looks the address up per device (with it current) and
// caches it for the life of the process.  The cached address belongs to the device's
// primary context: after cudaDeviceReset (which destroys that context) it is stale, so a
// process that resets a device must not call the no-alloc entry point on it again.
__device__ __align__(256) unsigned char g_noalloc_scratch[GOLLEK_NOALLOC_SCRATCH_BYTES];

std::mutex g_na_mu;
std::map<int, void *> g_na_ptr;

int noalloc_scratch(int dev, void **out) {
    std::lock_guard<std::mutex> lk(g_na_mu);
    auto it = g_na_ptr.find(dev);
    if (it != g_na_ptr.end()) {
        *out = it->second;
        return GOLLEK_OK;
    }
    void *p = nullptr;
    GK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    g_na_ptr[dev] = p;
    *out = p;
    return GOLLEK_OK;
}

}  // namespace
}  // namespace gk

using namespace gk;

// =============================================================== C ABI

extern "C" {

int paged_attention_launch(float *out, float *q, float *k_cache, float *v_cache, int *block_tables,
                           int *context_lens, int num_seqs, int num_heads, int head_dim,
                           int block_size, int max_blocks_per_seq, float scale) {
    t_last_error.clear();
    if (gollek_cuda_device_count() == 0) return fail(GOLLEK_ERR_NO_DEVICE, "no CUDA device");
    V2 p{};
    p.out = out;
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.bt = block_tables;
    p.ctx = context_lens;
    p.S = num_seqs;
    p.Hq = num_heads;
    p.Hkv = num_heads;
    p.D = head_dim;
    p.BS = block_size;
    p.maxB = max_blocks_per_seq;
    p.num_blocks = 0;
    p.page_stride = 0;
    p.q_dtype = GOLLEK_DTYPE_F32;
    p.kv_dtype = GOLLEK_DTYPE_F32;
    p.scale = scale;
    p.soft_cap = 0.f;
    p.window = 0;
    p.norm_eps = 0.f;  // the fallback divides by the plain sum (PagedAttentionCpuFallback.java:92-94)
    p.stream = cudaStreamPerThread;
    int rc = check_v2(p);
    if (rc) return rc;
    rc = run_v2(p);
    if (rc) return rc;
    unsigned v = 0;
    rc = read_and_clear_status(cudaStreamPerThread, &v);
    if (rc) return rc;
    return status_to_code(v);
}

int gollek_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int gollek_cuda_device_name(char *buf, int len) {
    if (!buf || len <= 0) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null or empty buffer");
    buf[0] = 0;
    if (gollek_cuda_device_count() == 0) return fail(GOLLEK_ERR_NO_DEVICE, "no CUDA device");
    int dev = 0;
    GK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    cudaDeviceProp prop;
    GK_CUDA(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
    snprintf(buf, static_cast<size_t>(len), "%s", prop.name);
    return GOLLEK_OK;
}

int gollek_paged_attention_v2(void *out, const void *q, const void *k_cache, const void *v_cache,
                              const float *k_scales, const float *v_scales, const int *block_tables,
                              const int *context_lens, int num_seqs, int num_q_heads,
                              int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq,
                              int num_blocks, long long page_stride, int q_dtype, int kv_dtype,
                              long long scale_page_stride, long long scale_head_stride,
                              long long scale_token_stride, float scale, float soft_cap,
                              int sliding_window, void *workspace, size_t workspace_bytes,
                              void *stream) {
    t_last_error.clear();
    V2 p{};
    p.out = out;
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.ks = k_scales;
    p.vs = v_scales;
    p.bt = block_tables;
    p.ctx = context_lens;
    p.S = num_seqs;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.D = head_dim;
    p.BS = block_size;
    p.maxB = max_blocks_per_seq;
    p.num_blocks = num_blocks;
    p.page_stride = page_stride;
    p.q_dtype = q_dtype;
    p.kv_dtype = kv_dtype;
    p.sps = scale_page_stride;
    p.shs = scale_head_stride;
    p.sts = scale_token_stride;
    p.scale = scale;
    p.soft_cap = soft_cap;
    p.window = sliding_window;
    p.norm_eps = 1e-9f;  // AttentionOnlineSoftmax.NORMALIZER_EPSILON
    p.workspace = workspace;
    p.workspace_bytes = workspace_bytes;
    p.stream = stream;
    int rc = check_v2(p);
    if (rc) return rc;
    return run_v2(p);
}

size_t gollek_paged_attention_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads,
                                             int head_dim) {
    if (num_seqs <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || head_dim <= 0)
        return 0;
    return ws_bytes(num_seqs, num_q_heads, num_kv_heads, head_dim);
}

static bool prefill_fold_enabled() {
    const char *e = std::getenv("GOLLEK_PREFILL_FOLD");
    return !(e && e[0] == '0');
}

size_t gollek_paged_attention_prefill_workspace_size(int num_seqs, int num_queries, int num_q_heads,
                                                     int num_kv_heads, int head_dim) {
    if (num_seqs <= 0 || num_queries <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 ||
        head_dim <= 0 || static_cast<long long>(num_seqs) * num_queries > (1 << 30))
        return 0;
    const int n = num_seqs * num_queries;
    return ws_bytes(n, num_q_heads, num_kv_heads, head_dim) + 2 * prefill_lens_bytes(n) + 512;
}

int gollek_paged_attention_prefill(void *out, const void *q, const void *k_cache, const void *v_cache,
                                   const float *k_scales, const float *v_scales, const int *block_tables,
                                   const int *context_lens, int num_seqs, int num_queries,
                                   int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                                   int max_blocks_per_seq, int num_blocks, long long page_stride,
                                   int q_dtype, int kv_dtype, long long scale_page_stride,
                                   long long scale_head_stride, long long scale_token_stride,
                                   float scale, float soft_cap, int sliding_window, int causal,
                                   void *workspace, size_t workspace_bytes, void *stream) {
    t_last_error.clear();
    if (num_queries <= 0) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "num_queries %d < 1", num_queries);
    if (num_seqs < 0 || static_cast<long long>(num_seqs) * num_queries > (1 << 30))
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "num_seqs * num_queries out of range");
    if (!causal && sliding_window > 0 && num_queries > 1)
        return fail(GOLLEK_ERR_UNSUPPORTED,
                    "a sliding window without causal masking over several queries");
    if (!context_lens) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    const int n = num_seqs * num_queries;
    V2 p{};
    p.out = out;
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.ks = k_scales;
    p.vs = v_scales;
    p.bt = block_tables;
    p.ctx = context_lens;  // checked below, replaced by the per-query lengths
    p.S = n;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.D = head_dim;
    p.BS = block_size;
    p.maxB = max_blocks_per_seq;
    p.num_blocks = num_blocks;
    p.page_stride = page_stride;
    p.q_dtype = q_dtype;
    p.kv_dtype = kv_dtype;
    p.sps = scale_page_stride;
    p.shs = scale_head_stride;
    p.sts = scale_token_stride;
    p.scale = scale;
    p.soft_cap = soft_cap;
    p.window = sliding_window;
    p.norm_eps = 1e-9f;  // AttentionOnlineSoftmax.NORMALIZER_EPSILON
    p.stream = stream;
    p.seq_div = num_queries;
    int rc = check_v2(p);
    if (rc) return rc;
    if (n == 0) return GOLLEK_OK;
    int dev = 0;
    GK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    // [counters][partials] ... [per-query lengths at the end]
    const size_t lens_bytes = prefill_lens_bytes(n);
    const size_t need = ws_bytes(n, num_q_heads, num_kv_heads, head_dim) + 2 * lens_bytes + 512;
    void *ws = workspace;
    size_t cap = workspace_bytes;
    if (ws) {
        if (workspace_bytes < need)
            return fail(GOLLEK_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed", workspace_bytes, need);
    } else {
        rc = library_workspace(dev, stream, need, &ws, &cap);
        if (rc) return rc;
    }
    if (ws_counter_region(cap) + ws_partials_bytes(n, num_q_heads, num_kv_heads, head_dim) + lens_bytes > cap)
        return fail(GOLLEK_ERR_WORKSPACE, "workspace of %zu bytes too small", cap);
    int *lens = reinterpret_cast<int *>(static_cast<uint8_t *>(ws) + (cap - lens_bytes) / 256 * 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    p.ctx = lens;
    p.workspace = ws;
    p.workspace_bytes = cap;
    // Page-once chunks: F queries of a sequence times its GQA group G as the rows of one
    // (sequence, kv-head) unit (G*F one of the decode kernel's row counts 2, 4, 8, and 16
    // for bf16 KV with head_dim 128, or 32 or 64 on the tensor-memory kernel with bf16 q),
    // each row with its own causal limit, so a page is read once per F queries instead of
    // once per query.  Causal, no sliding
    // window (its start would differ per row), bf16/f16/fp32 KV or int8 KV with head_dim 128.
    // F is the largest power of two dividing Tq whose rows have a compiled kernel;
    // GOLLEK_PREFILL_FOLD=0 keeps one query per decode sequence.  The partial slots need
    // the same bytes either way.
    const int G = num_q_heads / num_kv_heads;
    const bool foldable = causal && sliding_window <= 0 && prefill_fold_enabled() &&
                          (kv_dtype == GOLLEK_DTYPE_BF16 || kv_dtype == GOLLEK_DTYPE_F16 ||
                           kv_dtype == GOLLEK_DTYPE_F32 ||
                           (kv_dtype == GOLLEK_DTYPE_I8 && head_dim == 128));
    // rows of the kernels: 16 for bf16 KV with head_dim 128 (the mma.sync kernel), else 8;
    // with bf16 q also 32 or 64 (the tensor-memory kernel)
    const bool bf16_128 = kv_dtype == GOLLEK_DTYPE_BF16 && head_dim == 128;
    const int max_rows = bf16_128 ? 16 : 8;
    const bool tc_rows = bf16_128 && q_dtype == GOLLEK_DTYPE_BF16 && prefill_tc_enabled();
    auto next_fold = [&](int below) {
        for (int f = below >> 1; f > 1; f >>= 1)
            if (num_queries % f == 0 && (G * f <= max_rows || (tc_rows && (G * f == 32 || G * f == 64)))) return f;
        return 1;
    };
    int F = foldable ? next_fold(2 * 64) : 1;
    for (;;) {
        const int C = num_queries / F;
        const long long nv = static_cast<long long>(num_seqs) * C;
        const int threads = 256;
        const int blocks = static_cast<int>(std::min<long long>((nv + threads - 1) / threads, 4096));
        prefill_lengths_kernel<<<blocks, threads, 0, st>>>(context_lens, lens, num_seqs, C, F, causal);
        GK_CUDA(cudaGetLastError(), "prefill_lengths_kernel launch");
        p.S = static_cast<int>(nv);
        p.Hq = num_q_heads * F;
        p.seq_div = C;
        p.qfold = F;
        rc = run_v2(p);
        if (rc != kNotTaken || F == 1) return rc;
        t_last_error.clear();
        F = next_fold(F);  // no kernel for these rows: fewer queries per pass (at last one)
    }
}

int gollek_paged_attention_v2_noalloc(void *out, const void *q, const void *k_cache,
                                      const void *v_cache, const float *k_scales,
                                      const float *v_scales, const int *block_tables,
                                      const int *context_lens, int num_seqs, int num_q_heads,
                                      int num_kv_heads, int head_dim, int block_size,
                                      int max_blocks_per_seq, int num_blocks, long long page_stride,
                                      int q_dtype, int kv_dtype, long long scale_page_stride,
                                      long long scale_head_stride, long long scale_token_stride,
                                      float scale, float soft_cap, int sliding_window,
                                      void *stream) {
    t_last_error.clear();
    V2 p{};
    p.out = out;
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.ks = k_scales;
    p.vs = v_scales;
    p.bt = block_tables;
    p.ctx = context_lens;
    p.S = num_seqs;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.D = head_dim;
    p.BS = block_size;
    p.maxB = max_blocks_per_seq;
    p.num_blocks = num_blocks;
    p.page_stride = page_stride;
    p.q_dtype = q_dtype;
    p.kv_dtype = kv_dtype;
    p.sps = scale_page_stride;
    p.shs = scale_head_stride;
    p.sts = scale_token_stride;
    p.scale = scale;
    p.soft_cap = soft_cap;
    p.window = sliding_window;
    p.norm_eps = 1e-9f;
    p.stream = stream;
    int rc = check_v2(p);
    if (rc) return rc;
    if (p.S == 0) return GOLLEK_OK;
    const size_t need = ws_bytes(p.S, p.Hq, p.Hkv, p.D);
    if (need > GOLLEK_NOALLOC_SCRATCH_BYTES)
        return fail(GOLLEK_ERR_WORKSPACE,
                    "no-alloc decode needs %zu bytes of split-K scratch; its static buffer holds %u "
                    "(use gollek_paged_attention_v2 with a workspace)",
                    need, GOLLEK_NOALLOC_SCRATCH_BYTES);
    int dev = 0;
    GK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    void *scratch = nullptr;
    rc = noalloc_scratch(dev, &scratch);
    if (rc) return rc;
    // The arrival counters must start at zero; a previous call leaves them zeroed unless
    // it gave up half way, so clear them on every call.
    GK_CUDA(cudaMemsetAsync(scratch, 0, align_up(static_cast<uint32_t>(p.S) * p.Hkv * 4u, 256u),
                            static_cast<cudaStream_t>(stream)),
            "cudaMemsetAsync(no-alloc scratch counters)");
    p.workspace = scratch;
    p.workspace_bytes = GOLLEK_NOALLOC_SCRATCH_BYTES;
    return run_v2(p);
}

int gollek_kv_append(const void *key, const void *value, int src_dtype, const int *token_seq,
                     const int *token_pos, const int *block_tables, int max_blocks_per_seq,
                     int num_blocks, void *k_cache, void *v_cache, float *k_scales, float *v_scales,
                     int kv_dtype, int num_tokens, int num_kv_heads, int head_dim, int block_size,
                     long long page_stride, long long scale_page_stride, long long scale_head_stride,
                     long long scale_token_stride, void *stream) {
    t_last_error.clear();
    if (!key || !value || !token_pos || !block_tables || !k_cache || !v_cache)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
        max_blocks_per_seq <= 0 || num_blocks < 0)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "non-positive size");
    if (src_dtype != GOLLEK_DTYPE_F32 && src_dtype != GOLLEK_DTYPE_BF16)
        return fail(GOLLEK_ERR_UNSUPPORTED, "source dtype %d (F32 or BF16 only)", src_dtype);
    if (kv_dtype < GOLLEK_DTYPE_F32 || kv_dtype > GOLLEK_DTYPE_I4)
        return fail(GOLLEK_ERR_UNSUPPORTED, "kv dtype %d", kv_dtype);
    const long long ps = page_stride > 0 ? page_stride
                                         : static_cast<long long>(num_kv_heads) * block_size * head_dim;
    if (kv_dtype == GOLLEK_DTYPE_I4 && ((head_dim & 1) || (ps & 1)))
        return fail(GOLLEK_ERR_UNSUPPORTED, "int4 pools need an even head_dim and page stride");
    // The append quantises each row with its own absmax (the reference's per-token scale,
    // PagedKvCacheQuantization.java:66-80).  With scale_token_stride == 0 every row of a
    // page would overwrite the page's one shared scale and silently rescale the rows
    // written before it (rows of one launch would also race on that slot).
    if ((kv_dtype == GOLLEK_DTYPE_I8 || kv_dtype == GOLLEK_DTYPE_I4) && (k_scales || v_scales) &&
        scale_token_stride == 0)
        return fail(GOLLEK_ERR_UNSUPPORTED,
                    "appending to an int8/int4 pool needs per-token scales (scale_token_stride != 0); "
                    "a scale shared by a page's rows cannot take rows one at a time");
    if (num_tokens == 0) return GOLLEK_OK;
    AppendArgs a;
    a.key = key;
    a.value = value;
    a.token_seq = token_seq;
    a.token_pos = token_pos;
    a.block_tables = block_tables;
    a.k = k_cache;
    a.v = v_cache;
    a.k_scales = k_scales;
    a.v_scales = v_scales;
    a.page_stride = ps;
    a.scale_page_stride = scale_page_stride;
    a.scale_head_stride = scale_head_stride;
    a.scale_token_stride = scale_token_stride;
    a.src_bf16 = src_dtype == GOLLEK_DTYPE_BF16;
    a.kv_dtype = kv_dtype;
    a.num_tokens = num_tokens;
    a.num_kv_heads = num_kv_heads;
    a.head_dim = head_dim;
    a.block_size = block_size;
    a.max_blocks = max_blocks_per_seq;
    a.num_blocks = num_blocks;
    const long long rows = static_cast<long long>(num_tokens) * num_kv_heads;
    kv_append_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, static_cast<cudaStream_t>(stream)>>>(a);
    GK_CUDA(cudaGetLastError(), "kv_append_kernel launch");
    return GOLLEK_OK;
}

int gollek_kv_migrate(const void *src_k, const void *src_v, void *dst_k, void *dst_v,
                      const int *src_blocks, const int *dst_blocks, int num_copies,
                      int src_num_blocks, int dst_num_blocks, long long src_block_stride,
                      long long dst_block_stride, long long bytes_per_block, int device,
                      void *stream) {
    t_last_error.clear();
    if (!src_k || !dst_k || !src_blocks || !dst_blocks)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null pointer");
    if ((src_v == nullptr) != (dst_v == nullptr))
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "src_v and dst_v must both be set or both NULL");
    if (num_copies < 0 || bytes_per_block < 0 || src_block_stride < 0 || dst_block_stride < 0 ||
        src_num_blocks < 0 || dst_num_blocks < 0)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "negative size");
    if ((src_num_blocks > 0 && bytes_per_block > src_block_stride) ||
        (dst_num_blocks > 0 && bytes_per_block > dst_block_stride))
        return fail(GOLLEK_ERR_INVALID_ARGUMENT,
                    "bytes_per_block %lld exceeds a block stride of a bounded pool", bytes_per_block);
    if (num_copies == 0 || bytes_per_block == 0) return GOLLEK_OK;
    DeviceGuard guard(device);
    MigrateArgs a;
    a.src[0] = static_cast<const uint8_t *>(src_k);
    a.src[1] = static_cast<const uint8_t *>(src_v);
    a.dst[0] = static_cast<uint8_t *>(dst_k);
    a.dst[1] = static_cast<uint8_t *>(dst_v);
    a.src_blocks = src_blocks;
    a.dst_blocks = dst_blocks;
    a.src_stride = src_block_stride;
    a.dst_stride = dst_block_stride;
    a.bytes = bytes_per_block;
    a.tensors = src_v ? 2 : 1;
    a.src_num_blocks = src_num_blocks;
    a.dst_num_blocks = dst_num_blocks;
    a.segs_per_block = (bytes_per_block + kSegBytes - 1) / kSegBytes;
    a.num_units = static_cast<long long>(num_copies) * a.tensors * a.segs_per_block;
    const bool vec = aligned16(src_k) && aligned16(dst_k) && (!src_v || (aligned16(src_v) && aligned16(dst_v))) &&
                     bytes_per_block % 16 == 0 && src_block_stride % 16 == 0 && dst_block_stride % 16 == 0;
    const long long grid = std::min<long long>(a.num_units, static_cast<long long>(sm_count(device)) * 4);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (vec)
        kv_migrate_kernel_v16<<<static_cast<unsigned>(grid), 512, 0, st>>>(a);
    else
        kv_migrate_kernel_bytes<<<static_cast<unsigned>(grid), 256, 0, st>>>(a);
    GK_CUDA(cudaGetLastError(), "kv_migrate launch");
    return GOLLEK_OK;
}

int gollek_kv_block_checksum(const void *pool, const int *blocks, int n, int num_blocks,
                             long long block_stride, long long bytes_per_block,
                             unsigned long long *checksums, void *stream) {
    t_last_error.clear();
    if (!pool || !blocks || !checksums) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null pointer");
    if (n < 0 || num_blocks < 0 || bytes_per_block % 8 != 0 ||
        (reinterpret_cast<uintptr_t>(pool) & 7u) || block_stride % 8)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "checksums need 8-byte aligned blocks");
    if (n == 0) return GOLLEK_OK;
    block_checksum_kernel<<<n, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(pool), blocks, num_blocks, block_stride, bytes_per_block,
        checksums);
    GK_CUDA(cudaGetLastError(), "block_checksum_kernel launch");
    return GOLLEK_OK;
}

int gollek_enable_peer_access(int device, int peer_device) {
    t_last_error.clear();
    if (device == peer_device) return GOLLEK_OK;
    int can = 0;
    GK_CUDA(cudaDeviceCanAccessPeer(&can, device, peer_device), "cudaDeviceCanAccessPeer");
    if (!can) return fail(GOLLEK_ERR_UNSUPPORTED, "device %d cannot access device %d", device, peer_device);
    DeviceGuard guard(device);
    cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return GOLLEK_OK;
    }
    GK_CUDA(e, "cudaDeviceEnablePeerAccess");
    return GOLLEK_OK;
}

int gollek_ipc_get_handle(const void *dev_ptr, void *handle_out_64, long long *offset_out) {
    t_last_error.clear();
    if (!dev_ptr || !handle_out_64 || !offset_out)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t h;
    GK_CUDA(cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)), "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(handle_out_64, &h, sizeof(h));
    auto range = address_range_fn();
    if (!range) return fail(GOLLEK_ERR_UNSUPPORTED, "cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(GOLLEK_ERR_INVALID_ARGUMENT, "cuMemGetAddressRange failed");
    *offset_out = static_cast<long long>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
    return GOLLEK_OK;
}

int gollek_ipc_open_handle(const void *handle_64, void **dev_ptr_out) {
    t_last_error.clear();
    if (!handle_64 || !dev_ptr_out) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle_64, sizeof(h));
    GK_CUDA(cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    return GOLLEK_OK;
}

int gollek_ipc_close_handle(void *dev_ptr) {
    t_last_error.clear();
    if (!dev_ptr) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null pointer");
    GK_CUDA(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
    return GOLLEK_OK;
}

int gollek_device_status(int device, int clear, unsigned int *status_out) {
    t_last_error.clear();
    if (!status_out) return fail(GOLLEK_ERR_INVALID_ARGUMENT, "null pointer");
    if (gollek_cuda_device_count() == 0) return fail(GOLLEK_ERR_NO_DEVICE, "no CUDA device");
    DeviceGuard guard(device);
    GK_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    unsigned v = 0;
    GK_CUDA(cudaMemcpyFromSymbol(&v, g_status, sizeof(v)), "read status");
    if (clear) {
        const unsigned zero = 0;
        GK_CUDA(cudaMemcpyToSymbol(g_status, &zero, sizeof(zero)), "clear status");
    }
    if (v & GOLLEK_STATUS_TIMEOUT) {
        const int rc = rezero_library_counters(device);
        if (rc) return rc;
    }
    *status_out = v;
    return GOLLEK_OK;
}

const char *gollek_last_error_string(void) { return t_last_error.c_str(); }

const char *gollek_version(void) { return "gollek-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
