/*
 * ffm_harness.c -- calls libgollek_kernels.so the way Gollek's Java side binds it through the
 * FFM (Panama) linker: each entry point is looked up by name (dlsym, as
 * SymbolLookup.libraryLookup does, PagedAttentionBinding.java:69-86) and called through a
 * function-pointer type built from the FunctionDescriptor's value layouts only -- JAVA_INT as
 * int32_t, JAVA_LONG as int64_t, JAVA_FLOAT as float, ADDRESS as void* -- in the descriptors'
 * argument order (PagedAttentionBinding.java:200-227 for the original symbols; the
 * integration guide's descriptors for the new ones).  No header of the library is included,
 * so a mismatch between a descriptor and the library's real signature shows up here.
 *
 * Test infrastructure (tests/test_ffm_harness.py builds and runs it):
 *   ffm_harness abi <lib.so>            symbols and host-side argument checks, no device needed
 *   ffm_harness gpu <lib.so> <out.bin>  one call of each kind on device buffers; writes the
 *                                       inputs and outputs for the test to check with the oracle
 */
#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

typedef void *ADDRESS;

/* PagedAttentionBinding.java:200-217 -- ADDRESS x6, JAVA_INT x5, JAVA_FLOAT */
typedef int32_t (*paged_attention_launch_t)(ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, int32_t,
                                            int32_t, int32_t, int32_t, int32_t, float);
/* :219-220 and :222-227 */
typedef int32_t (*device_count_t)(void);
typedef int32_t (*device_name_t)(ADDRESS, int32_t);
/* gollek_paged_attention_v2: ADDRESS x8, JAVA_INT x7, JAVA_LONG, JAVA_INT x2, JAVA_LONG x3,
 * JAVA_FLOAT x2, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS */
typedef int32_t (*attention_v2_t)(ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS,
                                  int32_t, int32_t, int32_t, int32_t, int32_t, int32_t, int32_t, int64_t,
                                  int32_t, int32_t, int64_t, int64_t, int64_t, float, float, int32_t,
                                  ADDRESS, int64_t, ADDRESS);
/* gollek_kv_append: ADDRESS x2, JAVA_INT, ADDRESS x3, JAVA_INT x2, ADDRESS x4, JAVA_INT x5,
 * JAVA_LONG x4, ADDRESS */
typedef int32_t (*kv_append_t)(ADDRESS, ADDRESS, int32_t, ADDRESS, ADDRESS, ADDRESS, int32_t, int32_t,
                               ADDRESS, ADDRESS, ADDRESS, ADDRESS, int32_t, int32_t, int32_t, int32_t,
                               int32_t, int64_t, int64_t, int64_t, int64_t, ADDRESS);
/* gollek_kv_migrate: ADDRESS x6, JAVA_INT x3, JAVA_LONG x3, JAVA_INT, ADDRESS */
typedef int32_t (*kv_migrate_t)(ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, int32_t, int32_t,
                                int32_t, int64_t, int64_t, int64_t, int32_t, ADDRESS);
/* gollek_last_error_string: returns ADDRESS */
typedef ADDRESS (*last_error_t)(void);

static void *need(void *lib, const char *name) {
    void *f = dlsym(lib, name);
    if (!f) {
        fprintf(stderr, "missing symbol %s\n", name);
        exit(2);
    }
    return f;
}

static int check(int32_t rc, int32_t want, const char *what, last_error_t err) {
    if (rc != want) {
        fprintf(stderr, "%s: returned %d, expected %d (%s)\n", what, rc, want, (const char *)err());
        return 1;
    }
    return 0;
}

/* deterministic inputs: a 32-bit LCG mapped to [-1, 1) */
static uint32_t g_state = 12345u;
static float frand(void) {
    g_state = g_state * 1664525u + 1013904223u;
    return (float)((g_state >> 8) & 0xFFFFFF) / 8388608.0f - 1.0f;
}

#define DEV(call)                                                             \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess) {                                              \
            fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));      \
            return 3;                                                         \
        }                                                                     \
    } while (0)

int main(int argc, char **argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: %s abi|gpu <lib.so> [out.bin]\n", argv[0]);
        return 2;
    }
    void *lib = dlopen(argv[2], RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
        fprintf(stderr, "dlopen: %s\n", dlerror());
        return 2;
    }
    paged_attention_launch_t launch = (paged_attention_launch_t)need(lib, "paged_attention_launch");
    device_count_t count = (device_count_t)need(lib, "gollek_cuda_device_count");
    device_name_t name = (device_name_t)need(lib, "gollek_cuda_device_name");
    attention_v2_t v2 = (attention_v2_t)need(lib, "gollek_paged_attention_v2");
    kv_append_t append = (kv_append_t)need(lib, "gollek_kv_append");
    kv_migrate_t migrate = (kv_migrate_t)need(lib, "gollek_kv_migrate");
    last_error_t err = (last_error_t)need(lib, "gollek_last_error_string");
    int bad = 0;

    if (strcmp(argv[1], "abi") == 0) {
        /* host-side validation only: nothing here touches a device */
        char dummy[64];
        ADDRESS d = (ADDRESS)dummy;
        bad |= check(v2(d, d, d, d, NULL, NULL, d, d, 1, 6, 4, 64, 16, 4, 0, 0, 0, 0, 0, 0, 0, 1.0f, 0.0f, 0,
                        NULL, 0, NULL),
                     -1, "v2 with 6 q heads over 4 kv heads", err);
        bad |= check(append(d, d, 0, NULL, d, d, 4, 0, d, d, d, d, 3, 1, 1, 64, 16, 0, 8, 1, 0, NULL), -2,
                     "int8 append into per-page scales", err);
        bad |= check(migrate(d, NULL, d, d, d, d, 1, 0, 0, 16, 16, 16, 0, NULL), -1,
                     "migrate with src_v NULL and dst_v set", err);
        bad |= check(migrate(d, d, d, d, d, d, 1, -1, 4, 16, 16, 16, 0, NULL), -1,
                     "migrate with a negative pool size", err);
        printf("abi ok=%d devices=%d\n", !bad, count());
        return bad;
    }

    if (strcmp(argv[1], "gpu") != 0 || argc < 4) return 2;
    if (count() < 1) {
        fprintf(stderr, "no device\n");
        return 4;
    }
    char dev_name[128];
    bad |= check(name((ADDRESS)dev_name, (int32_t)sizeof dev_name), 0, "gollek_cuda_device_name", err);

    /* BASELINE config 1's shape: 4 sequences {37, 128, 301, 512}, 8 heads, head_dim 64,
     * block 16, pool 256 pages, pages assigned in a scrambled order */
    enum { S = 4, H = 8, D = 64, BS = 16, NB = 256, MAXB = 32 };
    static float q[S * H * D], k[NB * H * BS * D], v[NB * H * BS * D];
    static float out_legacy[S * H * D], out_v2[S * H * D];
    static int32_t bt[S * MAXB], ctx[S] = {37, 128, 301, 512};
    for (int i = 0; i < S * H * D; ++i) q[i] = frand();
    for (int i = 0; i < NB * H * BS * D; ++i) k[i] = frand();
    for (int i = 0; i < NB * H * BS * D; ++i) v[i] = frand();
    for (int i = 0; i < S * MAXB; ++i) bt[i] = (i * 97 + 13) % NB;  /* distinct, scrambled */
    void *dq, *dk, *dv, *dbt, *dctx, *dout;
    DEV(cudaMalloc(&dq, sizeof q));
    DEV(cudaMalloc(&dk, sizeof k));
    DEV(cudaMalloc(&dv, sizeof v));
    DEV(cudaMalloc(&dbt, sizeof bt));
    DEV(cudaMalloc(&dctx, sizeof ctx));
    DEV(cudaMalloc(&dout, sizeof out_legacy));
    DEV(cudaMemcpy(dq, q, sizeof q, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dk, k, sizeof k, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dv, v, sizeof v, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dbt, bt, sizeof bt, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dctx, ctx, sizeof ctx, cudaMemcpyHostToDevice));

    /* the plugin path: synchronous legacy symbol */
    bad |= check(launch(dout, dq, dk, dv, dbt, dctx, S, H, D, BS, MAXB, 0.125f), 0, "paged_attention_launch", err);
    DEV(cudaMemcpy(out_legacy, dout, sizeof out_legacy, cudaMemcpyDeviceToHost));

    /* the engine path: fp32 KV and q, GQA 1, library scratch, legacy default stream */
    bad |= check(v2(dout, dq, dk, dv, NULL, NULL, dbt, dctx, S, H, H, D, BS, MAXB, NB, 0, 0, 0, 0, 0, 0, 0.125f,
                    0.0f, 0, NULL, 0, NULL),
                 0, "gollek_paged_attention_v2", err);
    DEV(cudaDeviceSynchronize());
    DEV(cudaMemcpy(out_v2, dout, sizeof out_v2, cudaMemcpyDeviceToHost));

    /* append (overwrite) each sequence's last token, at position ctx - 1 of the pages the
     * tables name, then migrate three pages to free pages of the same pool */
    static float key[S * H * D], val[S * H * D];
    static int32_t pos[S];
    for (int i = 0; i < S * H * D; ++i) key[i] = frand();
    for (int i = 0; i < S * H * D; ++i) val[i] = frand();
    for (int s = 0; s < S; ++s) pos[s] = ctx[s] - 1;
    void *dkey, *dval, *dpos, *dsrc, *ddst;
    int32_t src[3] = {bt[0], bt[MAXB + 1], bt[3 * MAXB + 2]}, dst[3] = {250, 251, 252};
    DEV(cudaMalloc(&dkey, sizeof key));
    DEV(cudaMalloc(&dval, sizeof val));
    DEV(cudaMalloc(&dpos, sizeof pos));
    DEV(cudaMalloc(&dsrc, sizeof src));
    DEV(cudaMalloc(&ddst, sizeof dst));
    DEV(cudaMemcpy(dkey, key, sizeof key, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dval, val, sizeof val, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dpos, pos, sizeof pos, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(dsrc, src, sizeof src, cudaMemcpyHostToDevice));
    DEV(cudaMemcpy(ddst, dst, sizeof dst, cudaMemcpyHostToDevice));
    bad |= check(append(dkey, dval, 0, NULL, dpos, dbt, MAXB, NB, dk, dv, NULL, NULL, 0, S, H, D, BS, 0, 0, 0, 0,
                        NULL),
                 0, "gollek_kv_append", err);
    const int64_t page_bytes = (int64_t)H * BS * D * 4;
    bad |= check(migrate(dk, dv, dk, dv, dsrc, ddst, 3, NB, NB, page_bytes, page_bytes, page_bytes, 0, NULL), 0,
                 "gollek_kv_migrate", err);
    DEV(cudaDeviceSynchronize());
    static float k_after[NB * H * BS * D], v_after[NB * H * BS * D];
    DEV(cudaMemcpy(k_after, dk, sizeof k_after, cudaMemcpyDeviceToHost));
    DEV(cudaMemcpy(v_after, dv, sizeof v_after, cudaMemcpyDeviceToHost));

    FILE *f = fopen(argv[3], "wb");
    if (!f) return 2;
    fwrite(q, sizeof q, 1, f);
    fwrite(k, sizeof k, 1, f);
    fwrite(v, sizeof v, 1, f);
    fwrite(bt, sizeof bt, 1, f);
    fwrite(ctx, sizeof ctx, 1, f);
    fwrite(out_legacy, sizeof out_legacy, 1, f);
    fwrite(out_v2, sizeof out_v2, 1, f);
    fwrite(key, sizeof key, 1, f);
    fwrite(val, sizeof val, 1, f);
    fwrite(k_after, sizeof k_after, 1, f);
    fwrite(v_after, sizeof v_after, 1, f);
    fclose(f);
    printf("gpu ok=%d device=%s\n", !bad, dev_name);
    return bad;
}
