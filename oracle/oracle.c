/*
 * oracle.c -- CPU restatement of Gollek's paged-KV hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this file's
 * library, and only as the checker or the timed CPU baseline.  The product
 * (gollek_b200/, libgollek_kernels.so) never calls into it.
 *
 * The reference is Java 25 (Vector API, FFM); there is no JDK on either
 * machine, so it cannot be run.  This file restates the reference's
 * algorithms in C with Java float semantics:
 *   - every float operation rounds to float (compile with -ffp-contract=off,
 *     no -ffast-math: Java never fuses a*b+c);
 *   - (float) Math.exp(x) is a double exp of the float argument, then a cast;
 *   - Math.round(float) is "closest int, ties toward +infinity";
 *   - FloatVector reductions use L lanes (SPECIES_PREFERRED: 8 on AVX2,
 *     16 on AVX-512); lane partial sums are combined lane 0..L-1 in order.
 *     The Java spec leaves reduceLanes(ADD) order unspecified, so this is one
 *     admissible order; it moves results by a few float ulps at most.
 *
 * Pinning: the known-answer values in the reference's own unit tests
 * (PagedAttentionCpuFallbackTest, PagedAttentionVectorMathTest,
 * PagedKvCacheQuantizationTest, AttentionFp32VectorMathTest,
 * AttentionOnlineSoftmaxTest, PagedKvCacheLayoutTest) are re-checked against
 * these functions in tests/test_oracle_known_answers.py.
 *
 * Paths below are relative to the reference project root; abbreviations:
 *   PA/ = optimization/gollek-plugin-paged-attention/src/main/java/tech/kayys/gollek/kernel/paged/
 *   ST/ = runner/safetensor/gollek-safetensor-engine/src/main/java/tech/kayys/gollek/safetensor/engine/
 *   PD/ = optimization/gollek-plugin-prefill-decode/src/main/java/tech/kayys/gollek/prefilldecode/
 *   KV/ = optimization/gollek-plugin-kv-cache/src/main/java/tech/kayys/gollek/kvcache/
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_FP32 0
#define ORACLE_INT8 1
#define ORACLE_INT4 2

/* ---------------------------------------------------------------- helpers */

/* (float) Math.exp(x): double exp of the (float) argument, rounded to float. */
static float jexp(float x) { return (float)exp((double)x); }

/* Math.max(float, float) for the non-NaN values the paths produce. */
static float jmax(float a, float b) { return (a >= b) ? a : b; }

/* Math.round(float): closest int, ties toward +infinity; NaN -> 0.
 * (double)x + 0.5 is exact for every float below 2^29 in magnitude. */
static int jround(float x) {
    if (x != x) return 0;
    double r = floor((double)x + 0.5);
    if (r >= 2147483647.0) return 2147483647;
    if (r <= -2147483648.0) return (int)(-2147483647 - 1);
    return (int)r;
}

/* PagedKvCacheQuantization.readPackedSignedInt4, ST/generation/attention/PagedKvCacheQuantization.java:59-64 */
static int read_int4(const uint8_t *seg, long long elem) {
    int packed = seg[elem >> 1];
    int nib = (elem & 1LL) == 0 ? (packed & 0x0F) : ((packed >> 4) & 0x0F);
    return nib - 8;
}

/* PagedKvCacheQuantization.writePackedSignedInt4, :118-126 */
static void write_int4(uint8_t *seg, long long elem, int q) {
    long long byte = elem >> 1;
    int stored = q + 8;
    int existing = seg[byte];
    int packed = (elem & 1LL) == 0 ? ((existing & 0xF0) | (stored & 0x0F))
                                   : ((existing & 0x0F) | ((stored & 0x0F) << 4));
    seg[byte] = (uint8_t)packed;
}

/* ------------------------------------------------------------------- a1 */

/*
 * PagedAttentionCpuFallback.execute, PA/PagedAttentionCpuFallback.java:37-124.
 * fp32, MHA (one head count for Q and KV), three passes: scores, softmax
 * (max, exp, divide), weighted V sum.  Q/out [S,H,D]; K/V [NB,H,BS,D];
 * block tables [S,maxB]; context lengths [S].  Returns 0.
 */
static void a1_head(float *out, const float *q, const float *k, const float *v,
                    const int *bt, const int *ctx, int seq, int head, int H, int D,
                    int BS, int maxB, float scale, float *scores) {
    int contextLen = ctx[seq];
    int numBlocks = (contextLen + BS - 1) / BS;
    float maxScore = -INFINITY;
    for (int blockIdx = 0; blockIdx < numBlocks; blockIdx++) {          /* :59 */
        int physicalBlock = bt[(long long)seq * maxB + blockIdx];
        int tokensInBlock = BS < contextLen - blockIdx * BS ? BS : contextLen - blockIdx * BS;
        for (int tok = 0; tok < tokensInBlock; tok++) {
            int absPos = blockIdx * BS + tok;
            float dot = 0.0f;
            for (int d = 0; d < D; d++) {                                   /* :69-79 */
                long long qIdx = ((long long)seq * H + head) * D + d;
                float qVal = q[qIdx] * scale;
                long long kIdx = (((long long)physicalBlock * H + head) * BS + tok) * D + d;
                dot += qVal * k[kIdx];
            }
            scores[absPos] = dot;
            maxScore = jmax(maxScore, dot);
        }
    }
    float sumExp = 0.0f;                                                    /* :87-94 */
    for (int i = 0; i < contextLen; i++) {
        scores[i] = jexp(scores[i] - maxScore);
        sumExp += scores[i];
    }
    for (int i = 0; i < contextLen; i++) scores[i] /= sumExp;
    for (int d = 0; d < D; d++) {                                           /* :97-119 */
        float acc = 0.0f;
        for (int blockIdx = 0; blockIdx < numBlocks; blockIdx++) {
            int physicalBlock = bt[(long long)seq * maxB + blockIdx];
            int tokensInBlock = BS < contextLen - blockIdx * BS ? BS : contextLen - blockIdx * BS;
            for (int tok = 0; tok < tokensInBlock; tok++) {
                int absPos = blockIdx * BS + tok;
                long long vIdx = (((long long)physicalBlock * H + head) * BS + tok) * D + d;
                acc += scores[absPos] * v[vIdx];
            }
        }
        out[((long long)seq * H + head) * D + d] = acc;
    }
}

int oracle_a1_execute(float *out, const float *q, const float *k, const float *v,
                      const int *bt, const int *ctx, int S, int H, int D, int BS,
                      int maxB, float scale, int threads) {
    int maxCtx = 0;
    for (int s = 0; s < S; s++) maxCtx = ctx[s] > maxCtx ? ctx[s] : maxCtx;
    if (threads <= 1) {
        float *scores = (float *)malloc(sizeof(float) * (size_t)(maxCtx + 1));
        for (int seq = 0; seq < S; seq++)
            for (int head = 0; head < H; head++)
                a1_head(out, q, k, v, bt, ctx, seq, head, H, D, BS, maxB, scale, scores);
        free(scores);
        return 0;
    }
#ifdef _OPENMP
#pragma omp parallel num_threads(threads)
    {
        float *scores = (float *)malloc(sizeof(float) * (size_t)(maxCtx + 1));
#pragma omp for schedule(dynamic, 1)
        for (long long w = 0; w < (long long)S * H; w++)
            a1_head(out, q, k, v, bt, ctx, (int)(w / H), (int)(w % H), H, D, BS, maxB, scale, scores);
        free(scores);
    }
    return 0;
#else
    return -1;
#endif
}

/* ------------------------------------------------------------------- a2 */

/* AttentionFp32VectorMath.dotProduct, ST/generation/attention/AttentionFp32VectorMath.java:22-39 */
static float fp32_dot(const float *q, const float *k, int dim, int L) {
    float sum[64];
    int i = 0;
    for (int l = 0; l < L; l++) sum[l] = 0.0f;
    int upper = dim - dim % L;
    for (; i < upper; i += L)
        for (int l = 0; l < L; l++) {
            float prod = q[i + l] * k[i + l];
            sum[l] = sum[l] + prod;
        }
    float result = 0.0f;
    for (int l = 0; l < L; l++) result += sum[l];
    for (; i < dim; i++) result += q[i] * k[i];
    return result;
}

/* AttentionFp32VectorMath.updateAccumulator, :41-57 */
static void fp32_update(float *acc, const float *v, float prev, float cur, int dim) {
    for (int i = 0; i < dim; i++) {
        float a = acc[i] * prev;
        float b = v[i] * cur;
        acc[i] = a + b;
    }
}

/* PagedAttentionVectorMath.dotProductInt8 / Int4, ST/generation/attention/PagedAttentionVectorMath.java:46-74 */
static float quant_dot(int storage, const float *q, const uint8_t *blk, long long elem0,
                       float scale, int dim) {
    float result = 0.0f;
    for (int j = 0; j < dim; j++) {
        int kv = storage == ORACLE_INT8 ? (int)(int8_t)blk[elem0 + j] : read_int4(blk, elem0 + j);
        float kval = (float)kv * scale;
        result += q[j] * kval;
    }
    return result;
}

/* PagedAttentionVectorMath.updateAccumulatorInt8 / Int4, :57-84 */
static void quant_update(int storage, float *acc, const uint8_t *blk, long long elem0,
                         float scale, float prev, float cur, int dim) {
    for (int j = 0; j < dim; j++) {
        int vv = storage == ORACLE_INT8 ? (int)(int8_t)blk[elem0 + j] : read_int4(blk, elem0 + j);
        float a = acc[j] * prev;
        float b = ((float)vv * scale) * cur;
        acc[j] = a + b;
    }
}

typedef struct {
    const float *q;      /* [S][Tq][Hq][D] */
    float *out;          /* [S][Tq][Hq][D] */
    int S, Tq, Hq, Hkv, D, BS, maxB;
    const void *k_slab, *v_slab;        /* BlockManager slabs [maxBlocks][Hkv][BS][D] */
    const float *k_scale, *v_scale;     /* [maxBlocks][Hkv][BS] or NULL */
    int storage;
    const int *bt, *ctx;
    float scale, soft_cap;
    int causal, sliding_window, lanes;
} a2_args;

static long long block_bytes(int storage, int Hkv, int BS, int D) {
    long long elems = (long long)Hkv * BS * D;
    if (storage == ORACLE_FP32) return elems * 4;
    if (storage == ORACLE_INT8) return elems;
    return (elems + 1) / 2;
}

/*
 * computePagedHeadQuery, ST/generation/attention/PagedAttentionVectorAPI.java:126-180,
 * with AttentionOnlineSoftmax.observe / inverseNormalizer
 * (ST/generation/attention/AttentionOnlineSoftmax.java:38-56) and the GQA head map
 * and sliding-window minimum position of PagedAttentionVectorContext.queryAt
 * (ST/generation/attention/PagedAttentionVectorContext.java:59-88).
 * Sequence s owns block-table row bt[s*maxB..] and totalTokens = ctx[s]; its Tq
 * queries sit at absolute positions ctx[s]-Tq .. ctx[s]-1.
 */
static void a2_query(const a2_args *a, int s, int qh, int i, float *acc) {
    const int D = a->D, BS = a->BS;
    int totalTokens = a->ctx[s];
    int absolutePosition = totalTokens - a->Tq + i;
    int minPosition = a->sliding_window <= 0 ? 0
                      : (absolutePosition - a->sliding_window + 1 > 0 ? absolutePosition - a->sliding_window + 1 : 0);
    int gqaGroup = a->Hq / a->Hkv;
    int kvHead = qh / gqaGroup;
    long long qoff = (((long long)s * a->Tq + i) * a->Hq + qh) * D;
    const float *qv = a->q + qoff;
    long long bbytes = block_bytes(a->storage, a->Hkv, BS, D);

    float maxScore = -INFINITY, normalizer = 0.0f, prevW = 0.0f, curW = 0.0f;  /* reset() */
    for (int d = 0; d < D; d++) acc[d] = 0.0f;

    int currentTokCount = 0;
    for (int bi = 0; bi < a->maxB && totalTokens > 0; bi++) {
        int blockIdx = a->bt[(long long)s * a->maxB + bi];
        const uint8_t *kBlock = (const uint8_t *)a->k_slab + (long long)blockIdx * bbytes;
        const uint8_t *vBlock = (const uint8_t *)a->v_slab + (long long)blockIdx * bbytes;
        const float *kScale = a->k_scale ? a->k_scale + (long long)blockIdx * a->Hkv * BS : NULL;
        const float *vScale = a->v_scale ? a->v_scale + (long long)blockIdx * a->Hkv * BS : NULL;
        int tokensInThisBlock = BS < totalTokens - currentTokCount ? BS : totalTokens - currentTokCount;
        for (int tok = 0; tok < tokensInThisBlock; tok++) {
            int absPos = currentTokCount + tok;
            if (absPos < minPosition) continue;
            if (a->causal && absPos > absolutePosition) break;
            long long elem = (long long)kvHead * BS * D + (long long)tok * D;   /* PagedKvCacheLayout.sourceElement */
            long long sidx = (long long)kvHead * BS + tok;                      /* PagedKvCacheLayout.scaleIndex */
            float score;
            if (a->storage == ORACLE_FP32) {
                score = fp32_dot(qv, (const float *)kBlock + elem, D, a->lanes) * a->scale;
            } else {
                float sc = kScale ? kScale[sidx] : 1.0f;
                score = quant_dot(a->storage, qv, kBlock, elem, sc, D) * a->scale;
            }
            if (a->soft_cap > 0.0f)
                score = (float)(tanh((double)(score / a->soft_cap)) * (double)a->soft_cap);
            /* observe(score) */
            float prevMax = maxScore;
            maxScore = jmax(maxScore, score);
            prevW = jexp(prevMax - maxScore);
            curW = jexp(score - maxScore);
            normalizer = normalizer * prevW + curW;
            if (a->storage == ORACLE_FP32) {
                fp32_update(acc, (const float *)vBlock + elem, prevW, curW, D);
            } else {
                float sc = vScale ? vScale[sidx] : 1.0f;
                quant_update(a->storage, acc, vBlock, elem, sc, prevW, curW, D);
            }
        }
        currentTokCount += tokensInThisBlock;
        if (currentTokCount >= totalTokens) break;
    }
    float invL = 1.0f / (normalizer + 1e-9f);
    float *o = a->out + qoff;
    for (int d = 0; d < D; d++) o[d] = acc[d] * invL;
}

/*
 * PagedAttentionVectorAPI.compute, ST/generation/attention/PagedAttentionVectorAPI.java:60-124,
 * generalised to a batch of sequences each with its own block table and length.
 * storage: 0 FP32, 1 INT8, 2 INT4.  sliding_window <= 0 means no window.
 */
int oracle_a2_compute(float *out, const float *q, int S, int Tq, int Hq, int Hkv, int D, int BS,
                      const void *k_slab, const void *v_slab, const float *k_scale,
                      const float *v_scale, int storage, const int *bt, const int *ctx, int maxB,
                      float scale, int causal, float soft_cap, int sliding_window, int lanes,
                      int threads) {
    if (lanes < 1 || lanes > 64 || Hkv <= 0 || Hq % Hkv != 0) return -1;
    a2_args a = {q, out, S, Tq, Hq, Hkv, D, BS, maxB, k_slab, v_slab, k_scale, v_scale,
                 storage, bt, ctx, scale, soft_cap, causal, sliding_window, lanes};
    long long work = (long long)S * Hq * Tq;
    if (threads <= 1) {
        float *acc = (float *)malloc(sizeof(float) * (size_t)D);
        for (int b = 0; b < S; b++)
            for (int h = 0; h < Hq; h++)
                for (int i = 0; i < Tq; i++) a2_query(&a, b, h, i, acc);
        free(acc);
        return 0;
    }
#ifdef _OPENMP
#pragma omp parallel num_threads(threads)
    {
        float *acc = (float *)malloc(sizeof(float) * (size_t)D);
#pragma omp for schedule(dynamic, 1)
        for (long long w = 0; w < work; w++) {
            int i = (int)(w % Tq);
            int h = (int)((w / Tq) % Hq);
            int b = (int)(w / ((long long)Tq * Hq));
            a2_query(&a, b, h, i, acc);
        }
        free(acc);
    }
    return 0;
#else
    (void)work;
    return -1;
#endif
}

/* --------------------------------------------------------- math kernels */
/* Single-call restatements used by the known-answer tests. */

float oracle_fp32_dot(const float *q, const float *k, int dim, int lanes) {
    return fp32_dot(q, k, dim, lanes);
}

void oracle_fp32_update(float *acc, const float *v, float prev, float cur, int dim) {
    fp32_update(acc, v, prev, cur, dim);
}

/* PagedAttentionVectorMath.score, ST/generation/attention/PagedAttentionVectorMath.java:17-27 */
float oracle_score(int storage, const float *q, const void *k, long long elem0,
                   const float *scale_seg, long long scale_idx, int dim, float scale, int lanes) {
    if (storage == ORACLE_FP32) return fp32_dot(q, (const float *)k + elem0, dim, lanes) * scale;
    float sc = scale_seg ? scale_seg[scale_idx] : 1.0f;
    return quant_dot(storage, q, (const uint8_t *)k, elem0, sc, dim) * scale;
}

/* PagedAttentionVectorMath.updateAccumulator, :29-40 */
void oracle_update(int storage, float *acc, const void *v, long long elem0,
                   const float *scale_seg, long long scale_idx, float prev, float cur, int dim) {
    if (storage == ORACLE_FP32) { fp32_update(acc, (const float *)v + elem0, prev, cur, dim); return; }
    float sc = scale_seg ? scale_seg[scale_idx] : 1.0f;
    quant_update(storage, acc, (const uint8_t *)v, elem0, sc, prev, cur, dim);
}

/* AttentionOnlineSoftmax.observe over a score list; returns normalizer, writes
 * the last previous/current weights (ST/generation/attention/AttentionOnlineSoftmax.java:38-56). */
float oracle_softmax_observe(const float *scores, int n, float *prev_out, float *cur_out,
                             float *inv_out) {
    float maxScore = -INFINITY, normalizer = 0.0f, prevW = 0.0f, curW = 0.0f;
    for (int i = 0; i < n; i++) {
        float prevMax = maxScore;
        maxScore = jmax(maxScore, scores[i]);
        prevW = jexp(prevMax - maxScore);
        curW = jexp(scores[i] - maxScore);
        normalizer = normalizer * prevW + curW;
    }
    *prev_out = prevW;
    *cur_out = curW;
    *inv_out = 1.0f / (normalizer + 1e-9f);
    return normalizer;
}

int oracle_java_round(float x) { return jround(x); }

/* ------------------------------------------------------ quantise / append */

/* PagedKvCacheQuantization.vectorScale, ST/generation/attention/PagedKvCacheQuantization.java:96-106 */
static float vector_scale(const float *src, int dim, float maxq) {
    float absmax = 0.0f;
    for (int d = 0; d < dim; d++) {
        float a = fabsf(src[d]);
        if (a > absmax) absmax = a;
    }
    return absmax == 0.0f ? 1.0f : absmax / maxq;
}

/* PagedKvCacheQuantization.writeVector, :17-30 with quantizeVectorToInt8/Int4 :66-94. */
void oracle_write_vector(int storage, const float *src, void *dst, long long dst_elem,
                         float *scale_seg, long long scale_idx, int dim) {
    if (storage == ORACLE_FP32) {
        memcpy((float *)dst + dst_elem, src, sizeof(float) * (size_t)dim);
        return;
    }
    float maxq = storage == ORACLE_INT8 ? 127.0f : 7.0f;
    float sc = vector_scale(src, dim, maxq);
    if (scale_seg) scale_seg[scale_idx] = sc;
    for (int d = 0; d < dim; d++) {
        int qv = jround(src[d] / sc);
        if (storage == ORACLE_INT8) {
            qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
            ((int8_t *)dst)[dst_elem + d] = (int8_t)qv;
        } else {
            qv = qv < -8 ? -8 : (qv > 7 ? 7 : qv);
            write_int4((uint8_t *)dst, dst_elem + d, qv);
        }
    }
}

/* PagedKvCacheQuantization.writeVectorAsFloat, :32-57 (dequantise one vector). */
void oracle_read_vector(int storage, const void *src, const float *scale_seg, long long src_elem,
                        long long scale_idx, float *dst, int dim) {
    if (storage == ORACLE_FP32) {
        memcpy(dst, (const float *)src + src_elem, sizeof(float) * (size_t)dim);
        return;
    }
    float sc = scale_seg ? scale_seg[scale_idx] : 1.0f;
    for (int d = 0; d < dim; d++) {
        int v = storage == ORACLE_INT8 ? (int)((const int8_t *)src)[src_elem + d]
                                       : read_int4((const uint8_t *)src, src_elem + d);
        dst[d] = (float)v * sc;
    }
}

/*
 * PagedKvCacheIO.updateCache, ST/generation/attention/PagedKvCacheIO.java:23-62, for a
 * batch: token t (key/value rows src[t][Hkv][D]) belongs to sequence token_seq[t]
 * (or t when token_seq is NULL) at absolute position token_pos[t]; its block is
 * bt[seq*maxB + pos/BS] and its slot pos%BS.  Writes K and V through
 * oracle_write_vector.  Returns 0, or -1 for a missing (negative) block.
 */
int oracle_update_cache(const float *key, const float *value, int T, const int *token_seq,
                        const int *token_pos, const int *bt, int maxB, int Hkv, int D, int BS,
                        int storage, void *k_slab, void *v_slab, float *k_scale, float *v_scale) {
    long long bbytes = block_bytes(storage, Hkv, BS, D);
    for (int t = 0; t < T; t++) {
        int seq = token_seq ? token_seq[t] : t;
        int pos = token_pos[t];
        /* a position past the table has no block (the reference's lookup fails there too) */
        if (pos < 0 || pos / BS >= maxB) return -1;
        int blockIdx = bt[(long long)seq * maxB + pos / BS];
        if (blockIdx < 0) return -1;
        int tokIdx = pos % BS;
        uint8_t *kb = (uint8_t *)k_slab + (long long)blockIdx * bbytes;
        uint8_t *vb = (uint8_t *)v_slab + (long long)blockIdx * bbytes;
        float *ks = k_scale ? k_scale + (long long)blockIdx * Hkv * BS : NULL;
        float *vs = v_scale ? v_scale + (long long)blockIdx * Hkv * BS : NULL;
        for (int h = 0; h < Hkv; h++) {
            long long srcOff = ((long long)t * Hkv + h) * D;
            long long dstElem = (long long)h * BS * D + (long long)tokIdx * D;
            long long sidx = (long long)h * BS + tokIdx;
            if (storage == ORACLE_FP32) {
                memcpy((float *)kb + dstElem, key + srcOff, sizeof(float) * (size_t)D);
                memcpy((float *)vb + dstElem, value + srcOff, sizeof(float) * (size_t)D);
            } else {
                oracle_write_vector(storage, key + srcOff, kb, dstElem, ks, sidx, D);
                oracle_write_vector(storage, value + srcOff, vb, dstElem, vs, sidx, D);
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------- migration */

/*
 * PrefillDecodeDisaggService.transferKvToDecodePartition, PD/PrefillDecodeDisaggService.java:401-435,
 * over PhysicalBlockPool's [block][layer][bytesPerBlock] slabs (KV/PhysicalBlockPool.java:142-145):
 * for i, for layer: K and V slice of src_blocks[i] -> dst_blocks[i].  Source and
 * destination pools may be the same buffer (the reference's two partitions of one
 * pool) or different ones (two devices).  Returns bytes copied.
 */
long long oracle_migrate(const uint8_t *src_k, const uint8_t *src_v, uint8_t *dst_k, uint8_t *dst_v,
                         const int *src_blocks, const int *dst_blocks, int n, int num_layers,
                         long long bytes_per_block) {
    long long copied = 0;
    for (int i = 0; i < n; i++) {
        for (int layer = 0; layer < num_layers; layer++) {
            long long so = ((long long)src_blocks[i] * num_layers + layer) * bytes_per_block;
            long long dof = ((long long)dst_blocks[i] * num_layers + layer) * bytes_per_block;
            memcpy(dst_k + dof, src_k + so, (size_t)bytes_per_block);
            memcpy(dst_v + dof, src_v + so, (size_t)bytes_per_block);
            copied += 2 * bytes_per_block;
        }
    }
    return copied;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
