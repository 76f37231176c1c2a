"""The engine path on the device: KVCacheSession + update_cache + paged_attention_compute
against the oracle, and the PD service's migration through the pool."""
import math

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

STORAGE = {"fp32": O.FP32, "int8": O.INT8, "int4": O.INT4}


@pytest.mark.parametrize("storage", ["fp32", "int8", "int4", "bf16"])
def test_engine_prefill_then_decode(cuda_device, storage):
    from gollek_b200.engine import (BlockManager, KVCacheSession, KvStorageType,
                                    paged_attention_compute, update_cache)
    rng = np.random.default_rng(5)
    L, Hq, Hkv, D = 2, 8, 2, 64
    T = 45
    sess = KVCacheSession(256, BlockManager(device=cuda_device))
    sess.allocate(L, Hkv, D, KvStorageType(storage))
    layer = 1
    key = rng.standard_normal((T, Hkv, D)).astype(np.float32)
    val = rng.standard_normal((T, Hkv, D)).astype(np.float32)
    update_cache(torch.from_numpy(key).to(cuda_device), torch.from_numpy(val).to(cuda_device),
                 sess, layer, 0, T)
    q = rng.standard_normal((1, 1, Hq, D)).astype(np.float32)
    scale = 1 / math.sqrt(D)
    out = paged_attention_compute(torch.from_numpy(q).to(cuda_device), sess, layer, T, Hq, Hkv, D,
                                  scale).cpu().numpy()
    # oracle: the reference's updateCache into host slabs, then compute
    bm = sess.block_manager
    table = np.array([sess.get_block_table(layer)], np.int32)
    nb = bm.max_blocks
    if storage in ("fp32", "bf16"):
        ks = np.zeros((nb, Hkv, 16, D), np.float32)
        vs = np.zeros_like(ks)
        O.update_cache(key, val, np.arange(T, dtype=np.int32), table, storage=O.FP32, k_slab=ks,
                       v_slab=vs, token_seq=np.zeros(T, np.int32), block_size=16)
        if storage == "bf16":
            ks, vs = O.round_bf16(ks), O.round_bf16(vs)
        want = O.a2_compute(q, ks, vs, table, np.array([T], np.int32), scale, num_kv_heads=Hkv,
                            block_size=16)
        got_k = bm.k_slab.float().cpu().numpy()
        assert np.array_equal(got_k, ks)
        tol = 1e-4 * np.abs(want).max() if storage == "fp32" else 2e-2
    else:
        st = STORAGE[storage]
        bb = O.block_bytes(st, Hkv, 16, D)
        ks = np.zeros(nb * bb, np.uint8)
        vs = np.zeros_like(ks)
        ksc = np.zeros(nb * Hkv * 16, np.float32)
        vsc = np.zeros_like(ksc)
        O.update_cache(key, val, np.arange(T, dtype=np.int32), table, storage=st, k_slab=ks,
                       v_slab=vs, k_scale=ksc, v_scale=vsc, token_seq=np.zeros(T, np.int32),
                       block_size=16)
        assert np.array_equal(bm.k_slab.cpu().numpy().view(np.uint8).reshape(-1), ks)
        assert np.array_equal(bm.k_scale.cpu().numpy().reshape(-1), ksc)
        want = O.a2_compute(q, ks, vs, table, np.array([T], np.int32), scale, storage=st,
                            num_kv_heads=Hkv, block_size=16, k_scale=ksc, v_scale=vsc)
        tol = 1e-4 * np.abs(want).max()
    assert np.abs(out - want).max() <= tol


def test_pd_transfer_moves_every_layer(cuda_device):
    from gollek_b200.kv_cache import KVCacheConfig, PagedKVCacheManager
    from gollek_b200.prefill_decode import PrefillDecodeDisaggService
    cfg = KVCacheConfig(block_size=16, total_blocks=40, num_layers=4, num_heads=2, head_dim=32,
                        use_gpu=True)
    m = PagedKVCacheManager(cfg, device=cuda_device)
    svc = PrefillDecodeDisaggService(m, prefill_block_fraction=0.5)
    svc.init_partitions()
    pool = m.get_block_pool()
    g = torch.Generator(device=cuda_device).manual_seed(1)
    pool.k_pool.copy_(torch.randn(pool.k_pool.shape, generator=g, device=cuda_device))
    pool.v_pool.copy_(torch.randn(pool.v_pool.shape, generator=g, device=cuda_device))
    before_k, before_v = pool.k_pool.clone(), pool.v_pool.clone()
    prefill = m.allocate_for_prefill("req", 70)       # 5 blocks from the prefill side
    dst = svc.transfer_kv_to_decode_partition("req", prefill, "xfer-1")
    torch.cuda.synchronize()
    assert len(dst) == 5 and all(20 <= d < 40 for d in dst)
    for s, d in zip(prefill, dst):
        assert torch.equal(pool.k_pool[d], before_k[s]) and torch.equal(pool.v_pool[d], before_v[s])
    assert svc.status()["kv_transfer_bytes"] == 2 * 5 * cfg.num_layers * cfg.bytes_per_block()
    untouched = [b for b in range(40) if b not in dst]
    assert torch.equal(pool.k_pool[untouched], before_k[untouched])


def test_binding_launch_through_native(cuda_device):
    from gollek_b200.binding import PagedAttentionBinding
    PagedAttentionBinding.reset()
    assert PagedAttentionBinding.initialize()
    b = PagedAttentionBinding.get_instance()
    assert b.get_cuda_device_count() >= 1 and "B200" in b.get_cuda_device_name()
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 4, 64)).astype(np.float32)
    k = rng.standard_normal((6, 4, 16, 64)).astype(np.float32)
    v = rng.standard_normal((6, 4, 16, 64)).astype(np.float32)
    bt = np.array([[5, 0, 3], [1, 2, 4]], np.int32)
    ctx = np.array([40, 33], np.int32)
    T = lambda x: torch.from_numpy(x).to(cuda_device)
    out = torch.empty((2, 4, 64), device=cuda_device)
    rc = b.paged_attention_launch(out, T(q), T(k), T(v), T(bt), T(ctx), 2, 4, 64, 16, 3, 0.125)
    assert rc == 0
    want = O.a1_execute(q, k, v, bt, ctx, 0.125)
    assert np.abs(out.cpu().numpy() - want).max() <= 1e-4 * np.abs(want).max()
    PagedAttentionBinding.reset()
