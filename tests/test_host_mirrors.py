"""Host-side mirrors of the reference's Java classes (CPU only).

Ports of the reference's own tests:
  KVT/PagedKVCacheManagerTest.java  (optimization/gollek-plugin-kv-cache/src/test/java/tech/kayys/gollek/kvcache/)
  PDT/PrefillDecodeDisaggServiceTest.java (optimization/gollek-plugin-prefill-decode/src/test/...)
  PAT/PagedAttentionCpuFallbackTest.java:150-161 (binding in fallback mode)
  STT/generation/kv/KVCacheAllocationTest.java:20-71
"""
import threading

import pytest

from gollek_b200.binding import PagedAttentionBinding
from gollek_b200.engine import BlockManager, KVCacheSession, KvStorageType
from gollek_b200.kv_cache import (IllegalStateError, KVCacheConfig, KVCacheExhaustedException,
                                  PagedKVCacheManager)
from gollek_b200.prefill_decode import PrefillDecodeDisaggService


def _cfg(**kw):
    b = KVCacheConfig.builder().block_size(4).total_blocks(8).num_layers(2).num_heads(2).head_dim(4)
    for k, v in kw.items():
        getattr(b, k)(v)
    return b.use_gpu(False).build()


@pytest.fixture
def manager():
    m = PagedKVCacheManager(_cfg())
    yield m
    m.close()


# ---------------------------------------------------- PagedKVCacheManagerTest.java

def test_allocate_for_prefill_basic(manager):       # :44-55
    blocks = manager.allocate_for_prefill("req-1", 10)
    assert len(blocks) == 3
    assert manager.get_free_block_count() == 5
    assert manager.get_allocated_block_count() == 3
    assert manager.get_active_request_count() == 1
    assert manager.get_token_count("req-1") == 10


def test_allocate_exact_fit(manager):                # :57-64
    assert len(manager.allocate_for_prefill("req-1", 4)) == 1
    assert manager.get_free_block_count() == 7


def test_allocate_multiple_requests(manager):        # :66-76
    manager.allocate_for_prefill("req-1", 4)
    manager.allocate_for_prefill("req-2", 8)
    manager.allocate_for_prefill("req-3", 3)
    assert manager.get_active_request_count() == 3
    assert manager.get_allocated_block_count() == 4
    assert manager.get_free_block_count() == 4


def test_exhausted(manager):                         # :78-87
    manager.allocate_for_prefill("req-1", 32)
    with pytest.raises(KVCacheExhaustedException, match="exhausted"):
        manager.allocate_for_prefill("req-2", 1)


def test_duplicate_request(manager):                 # :89-97
    manager.allocate_for_prefill("req-1", 4)
    with pytest.raises(IllegalStateError, match="already has allocated blocks"):
        manager.allocate_for_prefill("req-1", 4)


def test_invalid_tokens(manager):                    # :99-106
    with pytest.raises(ValueError):
        manager.allocate_for_prefill("req-1", 0)
    with pytest.raises(ValueError):
        manager.allocate_for_prefill("req-1", -5)


def test_extend_within_block(manager):               # :110-119
    manager.allocate_for_prefill("req-1", 2)
    assert manager.extend_for_decode("req-1") >= 0
    assert manager.get_allocated_block_count() == 1


def test_extend_new_block(manager):                  # :121-131
    manager.allocate_for_prefill("req-1", 4)
    assert manager.extend_for_decode("req-1") >= 0
    assert manager.get_allocated_block_count() == 2
    assert len(manager.get_block_table("req-1")) == 2


def test_append_token_tracking(manager):             # :133-141
    manager.allocate_for_prefill("req-1", 3)
    assert manager.append_token("req-1") is False
    assert manager.append_token("req-1") is True
    assert manager.get_allocated_block_count() == 2


def test_free_request(manager):                      # :145-155
    manager.allocate_for_prefill("req-1", 12)
    assert manager.get_free_block_count() == 5
    assert manager.free_request("req-1") == 3
    assert manager.get_free_block_count() == 8
    assert manager.get_active_request_count() == 0


def test_free_then_reallocate(manager):              # :157-169
    manager.allocate_for_prefill("req-1", 32)
    assert manager.get_free_block_count() == 0
    manager.free_request("req-1")
    assert manager.get_free_block_count() == 8
    manager.allocate_for_prefill("req-2", 16)
    assert manager.get_free_block_count() == 4


def test_free_unknown(manager):                      # :171-176
    assert manager.free_request("nonexistent") == 0


def test_block_table_order_and_growth(manager):      # :180-204
    blocks = manager.allocate_for_prefill("req-1", 12)
    assert manager.get_block_table("req-1") == blocks
    manager.allocate_for_prefill("req-2", 4)
    assert len(manager.get_block_table("req-2")) == 1
    manager.extend_for_decode("req-2")
    assert len(manager.get_block_table("req-2")) == 2
    with pytest.raises(ValueError):
        manager.get_block_table("nonexistent")


def test_utilization_stats_capacity(manager):        # :208-245
    assert manager.get_utilization() == 0.0
    manager.allocate_for_prefill("req-1", 16)
    assert manager.get_utilization() == 0.5
    assert manager.has_capacity(4) and not manager.has_capacity(5)
    manager.allocate_for_prefill("req-2", 16)
    assert manager.get_utilization() == 1.0
    m = PagedKVCacheManager(_cfg())
    m.allocate_for_prefill("req-1", 8)
    m.free_request("req-1")
    m.allocate_for_prefill("req-2", 4)
    st = m.get_stats()
    assert (st.total_blocks, st.free_blocks, st.allocated_blocks, st.active_requests) == (8, 7, 1, 1)
    assert (st.total_allocations, st.total_deallocations) == (3, 2)


def test_max_blocks_per_request():                   # :249-268
    m = PagedKVCacheManager(_cfg(max_blocks_per_request=2))
    with pytest.raises(IllegalStateError, match="max blocks per request"):
        m.allocate_for_prefill("req-1", 9)


def test_concurrent_alloc_and_free():                # :272-321
    m = PagedKVCacheManager(_cfg(total_blocks=100))
    errors = []

    def worker(tid):
        try:
            for op in range(20):
                rid = f"thread-{tid}-op-{op}"
                try:
                    m.allocate_for_prefill(rid, 2)
                    m.free_request(rid)
                except KVCacheExhaustedException:
                    pass
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(t,)) for t in range(10)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(10)
    assert not errors
    assert m.get_free_block_count() == 100
    assert m.get_active_request_count() == 0


def test_block_table_native_is_int32(manager):
    manager.allocate_for_prefill("r", 9)
    t = manager.get_block_table_native("r")
    assert str(t.dtype) == "torch.int32" and t.tolist() == manager.get_block_table("r")


def test_pool_layout_and_bounds():
    m = PagedKVCacheManager(_cfg())
    pool = m.get_block_pool()
    assert pool.bytes_per_block == 4 * 2 * 4 * 2
    assert pool.get_total_allocated_bytes() == pool.bytes_per_block * 8 * 2 * 2
    assert tuple(pool.get_k_block(7, 1).shape) == (2, 4, 4)
    with pytest.raises(IndexError):
        pool.get_k_block(8, 0)
    with pytest.raises(IndexError):
        pool.get_v_block(0, 2)


# ---------------------------------------------- PrefillDecodeDisaggServiceTest.java

def _pd(total=10):
    m = PagedKVCacheManager(KVCacheConfig(block_size=4, total_blocks=total, num_layers=1,
                                          num_heads=1, head_dim=1))
    svc = PrefillDecodeDisaggService(m, prefill_block_fraction=0.5)
    svc.init_partitions()
    return svc


def test_pd_allocates_and_releases_decode_blocks():  # :16-37
    svc = _pd()
    blocks = svc.allocate_decode_blocks(3)
    assert len(blocks) == 3 and len(set(blocks)) == 3
    assert all(5 <= b < 10 for b in blocks)
    svc.release_decode_blocks(blocks)
    assert len(svc.allocate_decode_blocks(5)) == 5


def test_pd_exhausts_decode_blocks():                # :39-57
    svc = _pd()
    with pytest.raises(IllegalStateError):
        svc.allocate_decode_blocks(6)
    assert len(svc.allocate_decode_blocks(5)) == 5   # rollback restored the free list


def test_pd_status_counters():
    svc = _pd()
    st = svc.status()
    assert st["decode_blocks"] == [5, 10] and st["decode_free_blocks"] == 5
    assert st["kv_transfer_bytes"] == 0


# ------------------------------------------------ binding / engine allocation

def test_binding_fallback_mode():                    # PagedAttentionCpuFallbackTest.java:150-161
    PagedAttentionBinding.reset()
    PagedAttentionBinding.initialize_fallback()
    b = PagedAttentionBinding.get_instance()
    assert not b.is_native_available()
    assert b.get_cuda_device_count() == 0
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        b.paged_attention_launch(0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1.0)
    PagedAttentionBinding.reset()
    with pytest.raises(RuntimeError):
        PagedAttentionBinding.get_instance()


def test_binding_loads_native_library():
    PagedAttentionBinding.reset()
    assert PagedAttentionBinding.initialize() is True
    assert PagedAttentionBinding.get_instance().is_native_available()
    PagedAttentionBinding.reset()
    assert PagedAttentionBinding.initialize("/nonexistent/libgollek_kernels.so") is False
    PagedAttentionBinding.reset()


def test_session_ensure_capacity():                  # KVCacheAllocationTest.java:20-42
    s = KVCacheSession(128, BlockManager(device="cpu"))
    s.allocate(num_layers=2, num_kv_heads=1, head_dim=64)
    assert len(s.get_block_table(0)) == 1
    s.ensure_capacity(35)
    assert len(s.get_block_table(0)) == 3
    s.ensure_capacity(16)
    assert len(s.get_block_table(0)) == 3
    s.ensure_capacity(49)
    assert len(s.get_block_table(0)) == 4


def test_int4_blocks_are_packed():                   # KVCacheAllocationTest.java:44-71
    s = KVCacheSession(128, BlockManager(device="cpu"))
    s.allocate(num_layers=1, num_kv_heads=1, head_dim=64, storage=KvStorageType.INT4)
    bm = s.block_manager
    assert bm.storage_type == KvStorageType.INT4
    assert bm.get_block_size_bytes() == 512
    assert bm.k_scale is not None and tuple(bm.k_scale.shape[1:]) == (1, 16)
