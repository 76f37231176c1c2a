"""Generates the golden fixtures in this directory (run from the repository root):

    python tests/golden/make_golden.py

The reference is Java and cannot run here, so the fixtures are the CPU oracle's outputs
(oracle/oracle.c, a restatement of the reference's CPU path pinned by the reference's own
known-answer tests) on seeded inputs.  Inputs are not stored: each case records its seed
and a checksum of the inputs numpy's PCG64 generator produces, so a test can regenerate
them and verify they are the same before comparing outputs.  Cases:

  config1   BASELINE config 1: fp32, 4 sequences, contexts {37,128,301,512}, 8 heads,
            head_dim 64, block 16, 256-block pool in a seeded permutation, scale 1/8
            (PagedAttentionCpuFallback.execute)
  gqa_bf16  bf16-rounded GQA 32/8, head_dim 128, 5 sequences (PagedAttentionVectorAPI.compute)
  int8_kv   int8 KV with per-(block, head, token) scales from the reference's quantiser
  append    KV append (updateCache) of 12 tokens into int8 pages: the bytes and scales
  migrate   transferKvToDecodePartition on a 4-layer pool: checksum of the decode pool
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def tables(ctx, bs, nb, rng, maxb):
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((len(ctx), maxb), np.int32)
    off = 0
    for s, c in enumerate(ctx):
        n = (int(c) + bs - 1) // bs
        bt[s, :n] = perm[off:off + n]
        off += n
    return bt


def case_config1(seed=1):
    rng = np.random.default_rng(seed)
    ctx = np.array([37, 128, 301, 512], np.int32)
    bt = tables(ctx, 16, 256, rng, 32)
    q = rng.standard_normal((4, 8, 64)).astype(np.float32)
    k = rng.standard_normal((256, 8, 16, 64)).astype(np.float32)
    v = rng.standard_normal((256, 8, 16, 64)).astype(np.float32)
    return dict(ctx=ctx, bt=bt, q=q, k=k, v=v, scale=np.float32(0.125))


def case_gqa_bf16(seed=2):
    rng = np.random.default_rng(seed)
    ctx = np.array([1, 33, 300, 1024, 2000], np.int32)
    nb = int(((ctx + 15) // 16).sum()) + 4
    bt = tables(ctx, 16, nb, rng, 125)
    q = O.round_bf16(rng.standard_normal((5, 32, 128)).astype(np.float32))
    k = O.round_bf16((rng.standard_normal((nb, 8, 16, 128)) * 0.5).astype(np.float32))
    v = O.round_bf16((rng.standard_normal((nb, 8, 16, 128)) * 0.5).astype(np.float32))
    return dict(ctx=ctx, bt=bt, q=q, k=k, v=v, scale=np.float32(1 / np.sqrt(128)))


def quant_rows(x):
    nb, h, bs, d = x.shape
    qb = np.zeros(x.size, np.int8)
    sc = np.zeros(nb * h * bs, np.float32)
    xf = x.reshape(-1, d)
    for r in range(xf.shape[0]):
        O.write_vector(O.INT8, xf[r], qb, r * d, sc, r)
    return qb.reshape(x.shape), sc.reshape(nb, h, bs)


def case_int8(seed=3):
    c = case_gqa_bf16(seed)
    kq, ks = quant_rows(c["k"])
    vq, vs = quant_rows(c["v"])
    c.update(kq=kq, ks=ks, vq=vq, vs=vs)
    return c


def case_append(seed=4):
    rng = np.random.default_rng(seed)
    key = (rng.standard_normal((12, 4, 64)) * 2).astype(np.float32)
    val = (rng.standard_normal((12, 4, 64)) * 2).astype(np.float32)
    pos = np.array([0, 1, 15, 16, 17, 31, 40, 2, 5, 60, 63, 20], np.int32)
    seq = np.array([0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1], np.int32)
    bt = np.array([[3, 0, 7, 1], [5, 2, 6, 4]], np.int32)
    return dict(key=key, val=val, pos=pos, seq=seq, bt=bt)


def case_migrate(seed=5):
    rng = np.random.default_rng(seed)
    L, bpb, nb = 4, 256, 40
    pool_k = rng.integers(0, 256, nb * L * bpb, dtype=np.uint8)
    pool_v = rng.integers(0, 256, nb * L * bpb, dtype=np.uint8)
    src = rng.permutation(20)[:9].astype(np.int32)
    dst = (20 + rng.permutation(20)[:9]).astype(np.int32)
    return dict(pool_k=pool_k, pool_v=pool_v, src=src, dst=dst, L=L, bpb=bpb)


def outputs():
    res = {}
    c = case_config1()
    res["config1_in"] = digest(c["q"], c["k"], c["v"], c["bt"], c["ctx"])
    res["config1_out"] = O.a1_execute(c["q"], c["k"], c["v"], c["bt"], c["ctx"], c["scale"])
    c = case_gqa_bf16()
    res["gqa_bf16_in"] = digest(c["q"], c["k"], c["v"], c["bt"], c["ctx"])
    res["gqa_bf16_out"] = O.a2_compute(c["q"][:, None], c["k"], c["v"], c["bt"], c["ctx"], c["scale"],
                                       num_kv_heads=8, block_size=16)[:, 0]
    c = case_int8()
    res["int8_kv_in"] = digest(c["q"], c["kq"], c["vq"], c["ks"], c["vs"], c["bt"], c["ctx"])
    res["int8_kv_out"] = O.a2_compute(c["q"][:, None], c["kq"], c["vq"], c["bt"], c["ctx"],
                                      c["scale"], storage=O.INT8, num_kv_heads=8, block_size=16,
                                      k_scale=c["ks"], v_scale=c["vs"])[:, 0]
    c = case_append()
    res["append_in"] = digest(c["key"], c["val"], c["pos"], c["seq"], c["bt"])
    kb = np.zeros(8 * 4 * 16 * 64, np.int8)
    vb = np.zeros_like(kb)
    ks = np.zeros(8 * 4 * 16, np.float32)
    vs = np.zeros_like(ks)
    assert O.update_cache(c["key"], c["val"], c["pos"], c["bt"], storage=O.INT8, k_slab=kb,
                          v_slab=vb, k_scale=ks, v_scale=vs, token_seq=c["seq"], block_size=16) == 0
    res["append_k"], res["append_v"], res["append_ks"], res["append_vs"] = kb, vb, ks, vs
    c = case_migrate()
    res["migrate_in"] = digest(c["pool_k"], c["pool_v"], c["src"], c["dst"])
    k2, v2 = c["pool_k"].copy(), c["pool_v"].copy()
    O.migrate(k2, v2, k2, v2, c["src"], c["dst"], c["L"], c["bpb"])
    res["migrate_out"] = digest(k2, v2)
    return res


if __name__ == "__main__":
    res = outputs()
    np.savez_compressed(os.path.join(HERE, "golden.npz"),
                        **{k: (np.array(v) if isinstance(v, str) else v) for k, v in res.items()})
    print("wrote", os.path.join(HERE, "golden.npz"))
