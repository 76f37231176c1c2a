"""Paged KV-cache bookkeeping and the device-resident block pool.

Mirrors optimization/gollek-plugin-kv-cache/src/main/java/tech/kayys/gollek/kvcache/:
  KVCacheConfig.java          -> KVCacheConfig
  KVCacheExhaustedException   -> KVCacheExhaustedException
  PhysicalBlockPool.java      -> PhysicalBlockPool (slabs in HBM instead of an off-heap Arena)
  PagedKVCacheManager.java    -> PagedKVCacheManager (host allocator, same semantics)

The allocator stays on the host, as in the reference (it is a free list, not a
kernel); the pool it hands out lives in device memory so that the C ABI's device
pointers are real, which the reference's useGpu flag (KVCacheConfig.java:33) only
promised.
"""
from __future__ import annotations

import collections
import math
import threading
from dataclasses import dataclass


class KVCacheExhaustedException(RuntimeError):
    """The block pool cannot satisfy an allocation (KVCacheExhaustedException.java)."""


class IllegalStateError(RuntimeError):
    """Java's IllegalStateException (an operation not allowed in the current state).
    IllegalArgumentException maps to ValueError."""


@dataclass
class KVCacheConfig:
    """KVCacheConfig.java:12-210 (defaults :15-40)."""
    block_size: int = 16
    total_blocks: int = 1024
    num_layers: int = 32
    num_heads: int = 32
    head_dim: int = 128
    use_gpu: bool = False
    max_blocks_per_request: int = 0
    dtype_bytes: int = 2  # the reference sizes blocks as 16-bit values (PhysicalBlockPool.java:46-49)

    def bytes_per_block(self) -> int:
        """One (block, layer) slice of K (or V)."""
        return self.block_size * self.num_heads * self.head_dim * self.dtype_bytes

    def total_pool_bytes(self) -> int:
        return self.bytes_per_block() * self.total_blocks * self.num_layers * 2

    def max_context_length(self) -> int:
        return self.total_blocks * self.block_size

    @staticmethod
    def builder() -> "KVCacheConfigBuilder":
        return KVCacheConfigBuilder()


class KVCacheConfigBuilder:
    """KVCacheConfig.Builder (KVCacheConfig.java:163-210)."""

    def __init__(self):
        self._c = KVCacheConfig()

    def __getattr__(self, name):
        if name.startswith("_") or not hasattr(self._c, name):
            raise AttributeError(name)

        def setter(value):
            setattr(self._c, name, value)
            return self
        return setter

    def build(self) -> KVCacheConfig:
        return self._c


class PhysicalBlockPool:
    """K and V slabs laid out [block][layer][block_size*num_heads*head_dim] (16-bit), the
    layout of PhysicalBlockPool.java:38-60,142-145.  On a GPU config the slabs are device
    memory; within a (block, layer) slice the order is [head][token][dim], which is what the
    decode kernels read (PagedAttentionCpuFallback.java:15-22).

    get_k_block/get_v_block validate ids like the reference (IndexError for
    IndexOutOfBoundsException, :147-159).
    """

    def __init__(self, config: KVCacheConfig, device=None, dtype=None):
        import torch
        self.config = config
        self.bytes_per_block = config.bytes_per_block()
        dev = device if device is not None else ("cuda" if config.use_gpu else "cpu")
        dt = dtype if dtype is not None else torch.bfloat16
        shape = (config.total_blocks, config.num_layers, config.num_heads, config.block_size,
                 config.head_dim)
        self.k_pool = torch.zeros(shape, dtype=dt, device=dev)
        self.v_pool = torch.zeros(shape, dtype=dt, device=dev)

    def _validate(self, block_id: int, layer: int) -> None:
        if block_id < 0 or block_id >= self.config.total_blocks:
            raise IndexError(f"Block ID {block_id} out of range [0, {self.config.total_blocks})")
        if layer < 0 or layer >= self.config.num_layers:
            raise IndexError(f"Layer {layer} out of range [0, {self.config.num_layers})")

    def get_k_block(self, block_id: int, layer: int):
        self._validate(block_id, layer)
        return self.k_pool[block_id, layer]

    def get_v_block(self, block_id: int, layer: int):
        self._validate(block_id, layer)
        return self.v_pool[block_id, layer]

    def raw_k_pool(self):
        return self.k_pool

    def raw_v_pool(self):
        return self.v_pool

    def layer_view(self, layer: int):
        """(k, v, page_stride_elems) for the decode kernel on one layer."""
        c = self.config
        return (self.k_pool[:, layer], self.v_pool[:, layer],
                c.num_layers * c.num_heads * c.block_size * c.head_dim)

    def pack_block_table(self, block_ids, device=None):
        import torch
        return torch.tensor(list(block_ids), dtype=torch.int32,
                            device=device if device is not None else self.k_pool.device)

    def get_total_allocated_bytes(self) -> int:
        return self.bytes_per_block * self.config.total_blocks * self.config.num_layers * 2


CacheStats = collections.namedtuple(
    "CacheStats", "total_blocks free_blocks allocated_blocks active_requests utilization "
                  "total_allocations total_deallocations")


class PagedKVCacheManager:
    """PagedKVCacheManager.java:32-372: a FIFO free list of block ids and per-request
    block tables.  Thread-safe (one lock; the reference uses concurrent collections)."""

    def __init__(self, config: KVCacheConfig, allocate_pool: bool = True, device=None):
        self.config = config
        self.block_pool = PhysicalBlockPool(config, device=device) if allocate_pool else None
        self._free = collections.deque(range(config.total_blocks))
        self._blocks: dict[str, list[int]] = {}
        self._tokens: dict[str, int] = {}
        self._allocs = 0
        self._deallocs = 0
        self._lock = threading.RLock()

    # ---- allocation (:79-165)
    def allocate_for_prefill(self, request_id: str, num_tokens: int) -> list[int]:
        if num_tokens <= 0:
            raise ValueError(f"numTokens must be > 0, got: {num_tokens}")
        with self._lock:
            if request_id in self._blocks:
                raise IllegalStateError(f"Request already has allocated blocks: {request_id}")
            need = self.blocks_required(num_tokens)
            self._enforce_max_blocks(need)
            got = self._allocate_blocks(need)
            self._blocks[request_id] = list(got)
            self._tokens[request_id] = num_tokens
            self._allocs += need
            return list(got)

    def extend_for_decode(self, request_id: str) -> int:
        with self._lock:
            blocks = self._blocks.get(request_id)
            if blocks is None:
                raise ValueError(f"Unknown request: {request_id}")
            cur = self._tokens.get(request_id, 0)
            if cur < len(blocks) * self.config.block_size:
                self._tokens[request_id] = cur + 1
                return blocks[-1]
            self._enforce_max_blocks(len(blocks) + 1)
            if not self._free:
                raise KVCacheExhaustedException(
                    "KV-Cache pool exhausted. Free: 0, Requested: 1. "
                    "Consider increasing totalBlocks or evicting idle requests.")
            b = self._free.popleft()
            blocks.append(b)
            self._tokens[request_id] = cur + 1
            self._allocs += 1
            return b

    def append_token(self, request_id: str) -> bool:
        with self._lock:
            blocks = self._blocks.get(request_id)
            if blocks is None:
                raise ValueError(f"Unknown request: {request_id}")
            cur = self._tokens.get(request_id, 0)
            if cur < len(blocks) * self.config.block_size:
                self._tokens[request_id] = cur + 1
                return False
            self.extend_for_decode(request_id)
            return True

    # ---- deallocation (:176-191)
    def free_request(self, request_id: str) -> int:
        with self._lock:
            blocks = self._blocks.pop(request_id, None)
            self._tokens.pop(request_id, None)
            if not blocks:
                return 0
            self._free.extend(blocks)
            self._deallocs += len(blocks)
            return len(blocks)

    # ---- block tables (:202-222)
    def get_block_table(self, request_id: str) -> list[int]:
        with self._lock:
            blocks = self._blocks.get(request_id)
            if blocks is None:
                raise ValueError(f"Unknown request: {request_id}")
            return list(blocks)

    def get_block_table_native(self, request_id: str, device=None):
        """The table as an int32 tensor (device memory when the pool is on a GPU)."""
        import torch
        dev = device if device is not None else (
            self.block_pool.k_pool.device if self.block_pool is not None else "cpu")
        return torch.tensor(self.get_block_table(request_id), dtype=torch.int32, device=dev)

    # ---- queries (:229-299)
    def get_free_block_count(self) -> int:
        return len(self._free)

    def get_allocated_block_count(self) -> int:
        return self.config.total_blocks - len(self._free)

    def get_active_request_count(self) -> int:
        return len(self._blocks)

    def get_token_count(self, request_id: str) -> int:
        return self._tokens.get(request_id, -1)

    def get_utilization(self) -> float:
        return self.get_allocated_block_count() / self.config.total_blocks

    def has_capacity(self, blocks_needed: int) -> bool:
        return len(self._free) >= blocks_needed

    def get_block_pool(self) -> PhysicalBlockPool:
        return self.block_pool

    def get_config(self) -> KVCacheConfig:
        return self.config

    def get_stats(self) -> CacheStats:
        with self._lock:
            return CacheStats(self.config.total_blocks, self.get_free_block_count(),
                              self.get_allocated_block_count(), self.get_active_request_count(),
                              self.get_utilization(), self._allocs, self._deallocs)

    def blocks_required(self, num_tokens: int) -> int:
        return int(math.ceil(num_tokens / self.config.block_size))

    # ---- internal (:307-337)
    def _allocate_blocks(self, count: int) -> list[int]:
        if len(self._free) < count:
            raise KVCacheExhaustedException(
                f"KV-Cache pool exhausted. Free: {len(self._free)}, Requested: {count}. "
                "Consider increasing totalBlocks or evicting idle requests.")
        return [self._free.popleft() for _ in range(count)]

    def _enforce_max_blocks(self, total: int) -> None:
        m = self.config.max_blocks_per_request
        if m > 0 and total > m:
            raise IllegalStateError(f"Request exceeds max blocks per request limit: {total} > {m}")

    def close(self) -> None:
        with self._lock:
            self._blocks.clear()
            self._tokens.clear()
            self._free.clear()
            self.block_pool = None
