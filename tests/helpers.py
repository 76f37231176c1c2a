"""Seeded paged-KV cases shared by the tests (numpy, CPU)."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O


def make_tables(ctx, block_size, num_blocks, rng, max_blocks=None):
    """Block tables whose pages are a seeded random permutation of the pool."""
    ctx = np.asarray(ctx, np.int32)
    need = [(int(c) + block_size - 1) // block_size for c in ctx]
    if max_blocks is None:
        max_blocks = max(1, max(need) if need else 1)
    assert sum(need) <= num_blocks
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.full((len(ctx), max_blocks), -1, np.int32)
    off = 0
    for s, n in enumerate(need):
        bt[s, :n] = perm[off:off + n]
        off += n
    return bt


def decode_case(ctx, *, hq, hkv, d, bs, seed=0, kv_std=1.0, spare_pages=3, max_blocks=None):
    """q [S,Hq,D], K/V pools [NB,Hkv,BS,D] (fp32), tables, context lengths."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, np.int32)
    need = sum((int(c) + bs - 1) // bs for c in ctx)
    nb = need + spare_pages
    bt = make_tables(ctx, bs, nb, rng, max_blocks)
    q = rng.standard_normal((len(ctx), hq, d)).astype(np.float32)
    k = (rng.standard_normal((nb, hkv, bs, d)) * kv_std).astype(np.float32)
    v = (rng.standard_normal((nb, hkv, bs, d)) * kv_std).astype(np.float32)
    return q, k, v, bt, ctx


def oracle_decode(q, k, v, bt, ctx, scale, *, hkv, bs, storage=O.FP32, k_scale=None,
                  v_scale=None, soft_cap=0.0, window=0, lanes=8):
    out = O.a2_compute(q[:, None], k, v, bt, ctx, scale, storage=storage, num_kv_heads=hkv,
                       block_size=bs, k_scale=k_scale, v_scale=v_scale, soft_cap=soft_cap,
                       sliding_window=window, lanes=lanes, threads=O.num_threads())
    return out[:, 0]


def quantize_rows_int8(x):
    """The reference's per-row (per block, head, token) int8 quantisation, via the oracle.

    x: [NB, H, BS, D] fp32 -> (int8 [NB,H,BS,D], scales [NB,H,BS])."""
    nb, h, bs, d = x.shape
    q = np.zeros((nb, h, bs, d), np.int8)
    s = np.zeros((nb, h, bs), np.float32)
    qf = q.reshape(-1)
    sf = s.reshape(-1)
    xf = x.reshape(-1, d)
    for r in range(xf.shape[0]):
        O.write_vector(O.INT8, xf[r], qf, r * d, sf, r)
    return q, s


def quantize_pages_int8(x):
    """Per-(page, head) symmetric int8: scale = max|x|/127 over the page's BS x D values."""
    absmax = np.abs(x).max(axis=(2, 3))
    scale = np.where(absmax == 0, np.float32(1.0), (absmax / np.float32(127.0)).astype(np.float32))
    q = np.clip(np.floor(x / scale[:, :, None, None] + 0.5), -127, 127).astype(np.int8)
    return q, scale.astype(np.float32)
