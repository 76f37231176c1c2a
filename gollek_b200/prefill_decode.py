"""Prefill -> decode KV migration: the transfer half of Gollek's PD disaggregation.

Mirrors optimization/gollek-plugin-prefill-decode/src/main/java/tech/kayys/gollek/prefilldecode/
PrefillDecodeDisaggService.java: initPartitions (:446-455), allocateDecodeBlocks (:464-481),
releaseDecodeBlocks, transferKvToDecodePartition (:401-435) and the transfer counters behind
/v1/pd/status (:202-220).  The REST layer, the batcher and the simulated decode loop are
not part of the hot path and are not mirrored.

The copy itself is gollek_kv_migrate: one kernel moves every (block, layer) K and V slice
of a request -- within one pool (the reference's two partitions of one pool) or into
another device's pool over NVLink.
"""
from __future__ import annotations

import collections
import threading

from .kv_cache import IllegalStateError, PagedKVCacheManager


class PrefillDecodeDisaggService:
    def __init__(self, kv_cache_manager: PagedKVCacheManager, prefill_block_fraction: float = 0.3,
                 kv_transfer_backend: str = "ipc"):
        self.kv_cache_manager = kv_cache_manager
        self.prefill_block_fraction = prefill_block_fraction
        self.kv_backend = kv_transfer_backend
        self.prefill_block_start = self.prefill_block_end = 0
        self.decode_block_start = self.decode_block_end = 0
        self._decode_free: collections.deque[int] = collections.deque()
        self._decode_lock = threading.Lock()
        self.total_kv_transfers = 0
        self.kv_transfer_bytes_total = 0

    # ---- partitions (:446-481)
    def init_partitions(self) -> None:
        total = self.kv_cache_manager.get_config().total_blocks
        self.prefill_block_start = 0
        self.prefill_block_end = int(total * self.prefill_block_fraction)
        self.decode_block_start = self.prefill_block_end
        self.decode_block_end = total
        self._decode_free = collections.deque(range(self.decode_block_start, self.decode_block_end))

    def allocate_decode_blocks(self, count: int) -> list[int]:
        if count <= 0:
            return []
        with self._decode_lock:
            got = []
            for _ in range(count):
                if not self._decode_free:
                    self._decode_free.extend(got)  # roll back (:471-476)
                    raise IllegalStateError(
                        f"Decode partition exhausted: need {count} blocks, have {len(got)}")
                got.append(self._decode_free.popleft())
            return got

    def release_decode_blocks(self, blocks) -> None:
        if not blocks:
            return
        with self._decode_lock:
            self._decode_free.extend(blocks)

    # ---- transfer (:401-435)
    def transfer_kv_to_decode_partition(self, request_id: str, prefill_blocks, kv_transfer_id: str,
                                        dst_pool=None, decode_blocks=None,
                                        stream=None) -> list[int]:
        """Copy every layer's K and V of prefill_blocks[i] to decode_blocks[i].

        dst_pool: (k, v) device tensors of another device's pool with this pool's layout;
        None copies within this manager's pool.  decode_blocks defaults to a fresh
        allocation from the decode partition.  Returns the destination block ids."""
        import torch

        from . import ops

        pool = self.kv_cache_manager.get_block_pool()
        if decode_blocks is None:
            decode_blocks = self.allocate_decode_blocks(len(prefill_blocks))
        if len(decode_blocks) != len(prefill_blocks):
            raise ValueError("decode_blocks and prefill_blocks differ in length")
        if not prefill_blocks:
            return list(decode_blocks)
        src_k, src_v = pool.raw_k_pool(), pool.raw_v_pool()
        dk, dv = (src_k, src_v) if dst_pool is None else dst_pool
        dev = src_k.device
        per_block = pool.bytes_per_block * self.kv_cache_manager.get_config().num_layers
        s = torch.tensor(list(prefill_blocks), dtype=torch.int32, device=dev)
        d = torch.tensor(list(decode_blocks), dtype=torch.int32, device=dev)
        ops.kv_migrate(src_k, src_v, dk, dv, s, d, src_block_stride=per_block,
                       dst_block_stride=per_block, bytes_per_block=per_block, device=dev.index,
                       stream=stream)
        copied = 2 * per_block * len(prefill_blocks)
        self.total_kv_transfers += 1
        self.kv_transfer_bytes_total += copied
        return list(decode_blocks)

    def status(self) -> dict:
        """The transfer fields of GET /v1/pd/status (:202-220)."""
        return {"kv_backend": self.kv_backend,
                "prefill_blocks": [self.prefill_block_start, self.prefill_block_end],
                "decode_blocks": [self.decode_block_start, self.decode_block_end],
                "decode_free_blocks": len(self._decode_free),
                "total_kv_transfers": self.total_kv_transfers,
                "kv_transfer_bytes": self.kv_transfer_bytes_total}
