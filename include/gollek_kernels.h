/*
 * gollek_kernels.h -- C ABI of libgollek_kernels.so, the sm_100a (B200) paged-KV
 * attention hot path for Gollek.
 *
 * Every entry point takes plain pointers and sizes, so that Gollek's Java side can
 * bind it through the FFM (Panama) linker exactly as it binds the original
 * symbols.  Paths in the comments are relative to the Gollek project root:
 *   PA/ = optimization/gollek-plugin-paged-attention/src/main/java/tech/kayys/gollek/kernel/paged/
 *   ST/ = runner/safetensor/gollek-safetensor-engine/src/main/java/tech/kayys/gollek/safetensor/engine/
 *   PD/ = optimization/gollek-plugin-prefill-decode/src/main/java/tech/kayys/gollek/prefilldecode/
 *   KV/ = optimization/gollek-plugin-kv-cache/src/main/java/tech/kayys/gollek/kvcache/
 *
 * Conventions
 *   - Return value: 0 on success; a positive value is a cudaError_t; a negative
 *     value is one of the GOLLEK_ERR_* codes below.  gollek_last_error_string()
 *     describes the last failure on the calling thread.
 *   - Tensor pointers are device pointers unless stated otherwise.  The caller owns
 *     every buffer; the library keeps only per-device, per-stream scratch.
 *   - Entry points that take a `stream` (a cudaStream_t; NULL = legacy default
 *     stream) are asynchronous.  Errors that only the device can see (a block id
 *     outside the pool, a wait that gave up) are recorded in a per-device status
 *     word: read it with gollek_device_status().
 *   - All entry points are reentrant: no call shares mutable host state with
 *     another call except through a mutex, and scratch is keyed by stream.
 */
#ifndef GOLLEK_KERNELS_H
#define GOLLEK_KERNELS_H

#include <stddef.h>

#if defined(__GNUC__)
#define GOLLEK_API __attribute__((visibility("default")))
#else
#define GOLLEK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (negative; positive values are cudaError_t) ---------------- */
#define GOLLEK_OK 0
#define GOLLEK_ERR_INVALID_ARGUMENT (-1)
#define GOLLEK_ERR_UNSUPPORTED (-2)
#define GOLLEK_ERR_BAD_BLOCK_ID (-3)      /* a block-table entry outside [0, num_blocks) */
#define GOLLEK_ERR_TIMEOUT (-4)           /* a device-side wait gave up */
#define GOLLEK_ERR_NO_DEVICE (-5)
#define GOLLEK_ERR_WORKSPACE (-6)         /* caller workspace too small */
#define GOLLEK_ERR_BAD_POSITION (-7)      /* context length / position beyond the table */

/* ---- device status bits (gollek_device_status) -------------------------------- */
#define GOLLEK_STATUS_BAD_BLOCK_ID 0x1u
#define GOLLEK_STATUS_TIMEOUT 0x2u
#define GOLLEK_STATUS_BAD_POSITION 0x4u

/* ---- element types ------------------------------------------------------------ */
#define GOLLEK_DTYPE_F32 0
#define GOLLEK_DTYPE_BF16 1
#define GOLLEK_DTYPE_F16 2
#define GOLLEK_DTYPE_I8 3   /* symmetric int8 with fp32 scales */
#define GOLLEK_DTYPE_I4 4   /* packed signed nibbles (value + 8), two per byte, fp32 scales */

/* ======================================================================== *
 * Symbols bound by PagedAttentionBinding (PA/PagedAttentionBinding.java:48-50)
 * ======================================================================== */

/*
 * Replaces `paged_attention_launch` as bound at PA/PagedAttentionBinding.java:200-217
 * and specified at :120-139 (CPU equivalent PA/PagedAttentionCpuFallback.java:37-124).
 *
 * fp32 decode attention, one query token per sequence, num_heads query heads that
 * equal the KV heads:
 *   out, q          [num_seqs, num_heads, head_dim]                     (device)
 *   k_cache,v_cache [total_blocks, num_heads, block_size, head_dim]     (device)
 *   block_tables    [num_seqs, max_blocks_per_seq] int32                (device)
 *   context_lens    [num_seqs] int32                                    (device)
 *   out[s,h,:] = softmax_t((q[s,h,:]*scale) . K[t]) @ V over t < context_lens[s].
 * Synchronous (the Java caller reads `out` right after the call,
 * PD/PrefillDecodeDisaggService.java:389-392): the call runs on the calling thread's
 * per-thread stream and waits for it.  Returns 0, a cudaError_t, or a GOLLEK_ERR_*.
 */
GOLLEK_API int paged_attention_launch(float *out, float *q, float *k_cache, float *v_cache,
                           int *block_tables, int *context_lens, int num_seqs, int num_heads,
                           int head_dim, int block_size, int max_blocks_per_seq, float scale);

/* Replaces `gollek_cuda_device_count` (PA/PagedAttentionBinding.java:219-220):
 * number of visible CUDA devices, 0 when there is none or the driver fails. */
GOLLEK_API int gollek_cuda_device_count(void);

/* Replaces `gollek_cuda_device_name` (PA/PagedAttentionBinding.java:222-227): writes the
 * NUL-terminated name of the calling thread's current device into buf (at most len
 * bytes).  Returns 0 or an error code. */
GOLLEK_API int gollek_cuda_device_name(char *buf, int len);

/* ======================================================================== *
 * Extended decode attention (the engine path)
 * ======================================================================== */

/*
 * Decode attention over a paged KV pool, with GQA, fp32/bf16/f16/int8/int4 storage,
 * sliding window and soft-cap.  Replaces, for one query token per sequence,
 * PagedAttentionVectorAPI.compute (ST/generation/attention/PagedAttentionVectorAPI.java:60-180)
 * as reached from FlashAttentionJavaDispatchAdapter.pagedAttention
 * (ST/generation/attention/FlashAttentionJavaDispatchAdapter.java:43-50), and, with
 * num_q_heads == num_kv_heads, the fp32 paged_attention_launch above.
 *
 *   q, out     [num_seqs, num_q_heads, head_dim] of q_dtype (F32 or BF16); out has q's type.
 *   k_cache, v_cache: element (page p, kv-head h, token t, dim d) sits at element index
 *              p*page_stride + h*block_size*head_dim + t*head_dim + d of kv_dtype
 *              (page_stride 0 means num_kv_heads*block_size*head_dim; for I4 the index
 *              counts nibbles).  This covers BlockManager's [maxBlocks][H][BS][D] slab
 *              (ST/generation/kv/BlockManager.java:75-84) and, per layer, the
 *              [block][layer][H*BS*D] PhysicalBlockPool (KV/PhysicalBlockPool.java:142-145:
 *              pass the layer's base pointer and page_stride = num_layers*H*BS*D).
 *   k_scales, v_scales (I8/I4 only, else NULL): the scale of (p, h, t) is
 *              scales[p*scale_page_stride + h*scale_head_stride + t*scale_token_stride];
 *              the reference's per-(block, head, token) scales are strides (H*BS, BS, 1),
 *              per-(block, head) scales are (H, 1, 0).
 *   block_tables [num_seqs, max_blocks_per_seq], context_lens [num_seqs]: the query of
 *              sequence s sits at position context_lens[s]-1 and attends to positions
 *              [max(0, len - sliding_window), len) (sliding_window <= 0: no window).
 *   num_blocks pool size in pages, for device-side bounds checks (0: unchecked).
 *   scale      softmax scale; soft_cap > 0 applies cap*tanh(score/cap).
 *   GQA group num_q_heads / num_kv_heads: up to 8 for every storage type; 16 for bf16 KV
 *              with head_dim 128; 32 and 64 (multi-query-attention models) for bf16 KV
 *              and bf16 q with head_dim 128, up to 6,879 sequences per call; otherwise
 *              GOLLEK_ERR_UNSUPPORTED.
 *   workspace  split-K scratch of at least gollek_paged_attention_workspace_size(...)
 *              bytes, zero-filled before its first use and left zeroed by every call
 *              that completes; NULL = library-owned scratch cached per (device, stream).
 *              After a call whose device wait gave up (GOLLEK_STATUS_TIMEOUT from
 *              gollek_device_status, GOLLEK_ERR_TIMEOUT from a synchronous call) the
 *              caller must zero its workspace again before reusing it; the library
 *              re-zeroes its own scratch when it reports the timeout.
 * Asynchronous on `stream`.  Numerics: fp32 scores, softmax and accumulation.
 */
GOLLEK_API int gollek_paged_attention_v2(void *out, const void *q, const void *k_cache, const void *v_cache,
                              const float *k_scales, const float *v_scales,
                              const int *block_tables, const int *context_lens, int num_seqs,
                              int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                              int max_blocks_per_seq, int num_blocks, long long page_stride,
                              int q_dtype, int kv_dtype, long long scale_page_stride,
                              long long scale_head_stride, long long scale_token_stride,
                              float scale, float soft_cap, int sliding_window, void *workspace,
                              size_t workspace_bytes, void *stream);

/* Bytes of split-K scratch gollek_paged_attention_v2 needs for these sizes. */
GOLLEK_API size_t gollek_paged_attention_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads,
                                             int head_dim);

/*
 * Multi-query paged attention (several new tokens per sequence: prefill chunks,
 * speculative verification).  Replaces PagedAttentionVectorAPI.compute with
 * seqLenQ = num_queries > 1 (ST/generation/attention/PagedAttentionVectorAPI.java:60-180;
 * query i at absolute position startPos + i = ctx[s] - num_queries + i, :77-78, and the
 * causal / window bounds of computePagedHeadQuery, :126-180), which the PD service reaches
 * through runPrefillAttention (PD/PrefillDecodeDisaggService.java:359-373).
 *   q, out        [num_seqs][num_queries][num_q_heads][head_dim] (q_dtype)
 *   context_lens  [num_seqs] total tokens including the num_queries new ones
 *   causal        1: query i attends positions <= its own; 0: all context_lens[s] tokens
 *   sliding_window  > 0: the last sliding_window positions up to the query (causal only
 *                 when num_queries > 1; otherwise GOLLEK_ERR_UNSUPPORTED)
 *   workspace     >= gollek_paged_attention_prefill_workspace_size(...), or NULL
 * Every other argument as gollek_paged_attention_v2.  Causal calls over bf16/f16/fp32 KV,
 * or int8 KV with head_dim 128, without a window read each page once per F queries: F (the
 * largest power of two that divides num_queries with F * num_q_heads / num_kv_heads <= 16
 * for bf16 KV with head_dim 128, <= 8 otherwise -- or 32 or 64 for bf16 KV and bf16 q with
 * head_dim 128, on the tcgen05 kernel) queries of a sequence share one pass over its pages
 * as extra rows, each row with its own causal bound.  Other calls read each query's
 * context once per query.  The environment variables GOLLEK_PREFILL_FOLD=0 (read per call)
 * select the per-query form everywhere, GOLLEK_PREFILL_TC=0 the <= 16-row passes only,
 * GOLLEK_PREFILL_TC_HALVES=0 one warp per 32 rows on the tcgen05 kernel (two by default).
 */
GOLLEK_API int gollek_paged_attention_prefill(void *out, const void *q, const void *k_cache,
                                   const void *v_cache, const float *k_scales, const float *v_scales,
                                   const int *block_tables, const int *context_lens, int num_seqs,
                                   int num_queries, int num_q_heads, int num_kv_heads, int head_dim,
                                   int block_size, int max_blocks_per_seq, int num_blocks,
                                   long long page_stride, int q_dtype, int kv_dtype,
                                   long long scale_page_stride, long long scale_head_stride,
                                   long long scale_token_stride, float scale, float soft_cap,
                                   int sliding_window, int causal, void *workspace,
                                   size_t workspace_bytes, void *stream);

/* Bytes of scratch gollek_paged_attention_prefill needs for these sizes. */
GOLLEK_API size_t gollek_paged_attention_prefill_workspace_size(int num_seqs, int num_queries,
                                                     int num_q_heads, int num_kv_heads, int head_dim);

/*
 * Decode attention that allocates nothing.  No counterpart in the reference: this entry
 * point exists for callers that cannot allocate device memory themselves -- a caller
 * running inside a CUDA graph being captured elsewhere, a real-time or embedded host that
 * forbids allocation after start-up, or an FFM/JNI host whose memory allocator is not
 * CUDA-aware -- and so can neither call cudaMalloc nor hand the library a workspace.
 *
 * Same arguments and results as gollek_paged_attention_v2, without the workspace pair.
 * The split-K scratch is a static device array of GOLLEK_NOALLOC_SCRATCH_BYTES built into
 * the library (every GPU that loads the library holds it until the process exits).
 *   - Calls whose gollek_paged_attention_workspace_size(...) exceeds that size are
 *     rejected with GOLLEK_ERR_WORKSPACE; nothing is launched.
 *   - The first call on a device looks up the array's device address (with that device
 *     current) and caches it; make that first call before any stream capture.  The
 *     cached address lives as long as the device's primary context: do not call this
 *     entry point on a device after cudaDeviceReset in the same process.
 *   - Each call clears the scratch's arrival counters on `stream` before the kernel and
 *     never calls cudaMalloc, cudaFree or any allocating routine.
 *   - All calls on a device share the one array: calls that overlap on the GPU (on
 *     different streams, or from different threads) race on it.  Serialise them on one
 *     stream.
 */
#define GOLLEK_NOALLOC_SCRATCH_BYTES (32u << 20)
GOLLEK_API int gollek_paged_attention_v2_noalloc(
    void *out, const void *q, const void *k_cache, const void *v_cache, const float *k_scales,
    const float *v_scales, const int *block_tables, const int *context_lens, int num_seqs,
    int num_q_heads, int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq,
    int num_blocks, long long page_stride, int q_dtype, int kv_dtype, long long scale_page_stride,
    long long scale_head_stride, long long scale_token_stride, float scale, float soft_cap,
    int sliding_window, void *stream);

/* ======================================================================== *
 * KV append (the write path)
 * ======================================================================== */

/*
 * Writes new key/value rows into their pages.  Replaces PagedKvCacheIO.updateCache
 * (ST/generation/attention/PagedKvCacheIO.java:23-62) with
 * PagedKvCacheQuantization.writeVector (ST/generation/attention/PagedKvCacheQuantization.java:17-30,66-106).
 *
 *   key, value [num_tokens, num_kv_heads, head_dim] of src_dtype (F32 or BF16).
 *   token i belongs to sequence token_seq[i] (token_seq NULL: sequence i) at absolute
 *   position token_pos[i]; its page is block_tables[seq*max_blocks_per_seq + pos/block_size]
 *   and its slot pos % block_size.
 *   Pool layout, scale strides and num_blocks as in gollek_paged_attention_v2.
 *   F32/BF16/F16 pools store the (converted) values.  I8 (I4) pools store
 *   clamp(Math.round(x/s), -127, 127) (clamp(.., -8, 7)) with s = absmax/127 (absmax/7)
 *   over the row, s = 1 for an all-zero row, and write s to the scale slot -- bit for
 *   bit what the reference's Java computes.  I4 needs an even head_dim.  I8/I4 pools
 *   need per-token scales (scale_token_stride != 0): with a scale shared by a page's
 *   rows (scale_token_stride == 0) each appended row would overwrite the shared scale
 *   and rescale the rows already in the page, so such calls return
 *   GOLLEK_ERR_UNSUPPORTED.  (Decode reads either granularity.)
 * Asynchronous on `stream`.
 */
GOLLEK_API int gollek_kv_append(const void *key, const void *value, int src_dtype, const int *token_seq,
                     const int *token_pos, const int *block_tables, int max_blocks_per_seq,
                     int num_blocks, void *k_cache, void *v_cache, float *k_scales,
                     float *v_scales, int kv_dtype, int num_tokens, int num_kv_heads,
                     int head_dim, int block_size, long long page_stride,
                     long long scale_page_stride, long long scale_head_stride,
                     long long scale_token_stride, void *stream);

/* ======================================================================== *
 * KV block migration (prefill -> decode)
 * ======================================================================== */

/*
 * Copies KV blocks with a block-id remap.  Replaces the copy loop of
 * PrefillDecodeDisaggService.transferKvToDecodePartition (PD/PrefillDecodeDisaggService.java:401-435),
 * whose per-(block, layer) slices are contiguous per block in PhysicalBlockPool's
 * [block][layer][bytesPerBlock] layout (KV/PhysicalBlockPool.java:142-145).
 *
 * For i < num_copies, bytes_per_block bytes move from
 *   src_k + src_blocks[i]*src_block_stride  ->  dst_k + dst_blocks[i]*dst_block_stride
 * and the same for V (src_v/dst_v may be NULL to copy K only).  src_blocks/dst_blocks
 * are device int32 arrays on the device the kernel runs on, `device`, which must also
 * hold the source pools.  src_num_blocks / dst_num_blocks are the pools' sizes in
 * blocks (0 = unchecked): a copy whose source or destination id lies outside
 * [0, num_blocks) -- or is negative, whatever the size -- is skipped and raises
 * GOLLEK_STATUS_BAD_BLOCK_ID (read it with gollek_device_status), as
 * PhysicalBlockPool.getKBlock rejects such ids (KV/PhysicalBlockPool.java:147-159).  A
 * bounded pool needs bytes_per_block <= its block stride.  The destination may be this device's memory (the reference's
 * two partitions of one pool; also the prompt cache's copy-on-write) or a peer's:
 * a peer pointer after gollek_enable_peer_access(device, peer) or one mapped with
 * gollek_ipc_open_handle().  The kernel reads locally and stores over NVLink with
 * 16-byte stores.  Asynchronous on `stream` (a stream of `device`).
 */
GOLLEK_API int gollek_kv_migrate(const void *src_k, const void *src_v, void *dst_k, void *dst_v,
                      const int *src_blocks, const int *dst_blocks, int num_copies,
                      int src_num_blocks, int dst_num_blocks, long long src_block_stride,
                      long long dst_block_stride, long long bytes_per_block, int device,
                      void *stream);

/*
 * Per-block 64-bit checksums, sum over the block's 8-byte words w_j of
 * (w_j XOR (j * 0x9E3779B97F4A7C15)) mod 2^64, of pool + blocks[i]*block_stride for
 * i < n (bytes_per_block a multiple of 8).  Lets a caller verify a migration of any
 * size without moving the blocks back to the host.  num_blocks is the pool's size in
 * blocks (0 = unchecked); an id outside [0, num_blocks), or negative, reads nothing,
 * gets checksum 0 and raises GOLLEK_STATUS_BAD_BLOCK_ID.  Asynchronous on `stream`.
 */
GOLLEK_API int gollek_kv_block_checksum(const void *pool, const int *blocks, int n, int num_blocks,
                             long long block_stride, long long bytes_per_block,
                             unsigned long long *checksums, void *stream);

/* Enables `device` to access `peer_device`'s memory (idempotent). */
GOLLEK_API int gollek_enable_peer_access(int device, int peer_device);

/* CUDA IPC for one-process-per-GPU deployments: export the device allocation holding
 * dev_ptr as a 64-byte handle plus dev_ptr's byte offset inside that allocation (the
 * importer adds it to the base that gollek_ipc_open_handle returns); map a peer
 * process's handle into this process; unmap it. */
GOLLEK_API int gollek_ipc_get_handle(const void *dev_ptr, void *handle_out_64,
                                     long long *offset_out);
GOLLEK_API int gollek_ipc_open_handle(const void *handle_64, void **dev_ptr_out);
GOLLEK_API int gollek_ipc_close_handle(void *dev_ptr);

/* ======================================================================== *
 * Diagnostics
 * ======================================================================== */

/* Reads (and with clear != 0, resets) the device status word of `device`; waits for
 * the device's outstanding work first.  Bits: GOLLEK_STATUS_*. */
GOLLEK_API int gollek_device_status(int device, int clear, unsigned int *status_out);

/* Message for the last failed call on this thread ("" when none). */
GOLLEK_API const char *gollek_last_error_string(void);

/* Library version string. */
GOLLEK_API const char *gollek_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GOLLEK_KERNELS_H */
