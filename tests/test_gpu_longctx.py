"""BASELINE config 5 lengths on the device: Llama-3-70B-shaped long-context decode.

64 query heads over 8 KV heads (GQA 8), head_dim 128, block size 16, bf16 KV ~ N(0, 0.5^2),
q ~ N(0, 1), contexts of 32k, 64k and 131,072 tokens -- the lengths config 5 draws from
log-uniform[4096, 131072].  At these lengths a (sequence, kv-head) is cut into many split-K
pieces (up to the schedule's cap of 64: a lone 131,072-token unit is 8,192 16-token groups
over ~62 CTAs), so this is where the merge of the pieces' log-sum-exp states is exercised.
Each case runs the full 8 KV heads and, as one rank of the KV-head sharding sees it, a
slice of the heads with its own [pages, heads/N, 16, 128] pool and the matching q heads.

Reference: PagedAttentionVectorAPI.computePagedHeadQuery
(ST/generation/attention/PagedAttentionVectorAPI.java:126-180), restated in oracle/oracle.c.
Tolerance: 2e-2 absolute against the fp32 oracle on the same bf16-rounded inputs.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HQ, HKV, D, BS = 64, 8, 128, 16
G = HQ // HKV


def _case(ctx, seed):
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, np.int32)
    need = (ctx + BS - 1) // BS
    nb = int(need.sum()) + 5
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((len(ctx), int(need.max())), -1, np.int32)
    off = 0
    for s, n in enumerate(need):
        bt[s, :n] = perm[off:off + n]
        off += n
    q = O.round_bf16(rng.standard_normal((len(ctx), HQ, D), dtype=np.float32))
    k = O.round_bf16((rng.standard_normal((nb, HKV, BS, D), dtype=np.float32) * 0.5))
    v = O.round_bf16((rng.standard_normal((nb, HKV, BS, D), dtype=np.float32) * 0.5))
    return q, k, v, bt, ctx


def _run(dev, q, k, v, bt, ctx, hkv):
    from gollek_b200 import ops
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    out = ops.paged_attention(T(q).to(torch.bfloat16), T(k).to(torch.bfloat16),
                              T(v).to(torch.bfloat16), T(bt), T(ctx), num_kv_heads=hkv,
                              block_size=BS, num_blocks=k.shape[0], scale=1.0 / math.sqrt(D))
    torch.cuda.synchronize()
    assert ops.device_status(dev.index, clear=True) == 0
    return out.float().cpu().numpy()


def _oracle(q, k, v, bt, ctx, hkv):
    return O.a2_compute(q[:, None], k, v, bt, ctx, 1.0 / math.sqrt(D), num_kv_heads=hkv,
                        block_size=BS, threads=O.num_threads())[:, 0]


@pytest.mark.parametrize("ctx,shards,seed", [
    ([32768, 65536, 131072], [1, 8], 51),   # full heads, and the 1-head shard of N = 8
    ([131072], [1, 8], 52),                 # a lone unit: ~62 split-K pieces per kv-head
    (None, [2, 4], 53),                     # config 5's own draw (first sequences), N = 2 / 4 shards
])
def test_config5_lengths_match_oracle(cuda_device, ctx, shards, seed):
    if ctx is None:
        r = np.random.default_rng(2024)
        u = r.uniform(math.log(4096), math.log(131072), 256)
        ctx = np.exp(u).astype(np.int32)[:6]
    q, k, v, bt, ctx = _case(ctx, seed)
    for n in shards:
        per = HKV // n
        # rank n - 1 of n (the last shard): kv-heads [lo, hi) and their q heads
        lo, hi = HKV - per, HKV
        ks = np.ascontiguousarray(k[:, lo:hi])
        vs = np.ascontiguousarray(v[:, lo:hi])
        qs = np.ascontiguousarray(q[:, lo * G:hi * G])
        got = _run(cuda_device, qs, ks, vs, bt, ctx, per)
        want = _oracle(qs, ks, vs, bt, ctx, per)
        assert np.isfinite(got).all()
        err = np.abs(got - want).max()
        assert err <= 2e-2, (n, err)
