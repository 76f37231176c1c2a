"""The safetensor engine's paged KV cache and its attention call, on the device.

Mirrors runner/safetensor/gollek-safetensor-engine/src/main/java/tech/kayys/gollek/safetensor/
engine/generation/:
  kv/BlockManager.java                   -> BlockManager (slabs [maxBlocks][H][BS][D] in HBM)
  kv/KVCacheManager.KVCacheSession       -> KVCacheSession (one block table per layer)
  attention/PagedKvCacheIO.updateCache   -> update_cache (gollek_kv_append)
  attention/PagedAttentionVectorAPI.compute -> paged_attention_compute (gollek_paged_attention_v2)

FP32, INT8 and INT4 storage follow the reference bit for bit on the write side (per
(block, head, token) symmetric scales); BF16 storage is an extension.  A call with one
query token per sequence runs decode attention (gollek_paged_attention_v2); with Tq > 1 new
tokens (a prefill chunk, speculative verification) it runs multi-query attention
(gollek_paged_attention_prefill), causal by default, like compute with seqLenQ > 1.
"""
from __future__ import annotations

import collections
import enum
import math

from .kv_cache import IllegalStateError


class KvStorageType(enum.Enum):
    FP32 = "fp32"
    INT8 = "int8"
    INT4 = "int4"
    BF16 = "bf16"  # not in the reference (BlockManager.java:18-22 has FP32/INT8/INT4)


class BlockManager:
    """BlockManager.java:17-222: contiguous K/V slabs, per-block-head-token fp32 scales for
    the quantised types, a FIFO free list."""

    def __init__(self, device="cuda"):
        self.device = device
        self.initialized = False
        self.max_blocks = 0
        self.tokens_per_block = 0
        self.num_heads = 0
        self.head_dim = 0
        self.storage_type = KvStorageType.FP32
        self._free: collections.deque[int] = collections.deque()

    def initialize(self, tokens_per_block: int, num_heads: int, head_dim: int, max_blocks: int,
                   storage_type: KvStorageType = KvStorageType.FP32) -> None:
        import torch
        same = (self.initialized and self.tokens_per_block == tokens_per_block and
                self.num_heads == num_heads and self.head_dim == head_dim and
                self.storage_type == storage_type and self.max_blocks >= max_blocks)
        if same:
            self._reset_free()
            return
        if storage_type == KvStorageType.INT4 and head_dim % 2:
            raise ValueError("INT4 storage needs an even head_dim")
        self.tokens_per_block, self.num_heads, self.head_dim = tokens_per_block, num_heads, head_dim
        self.max_blocks, self.storage_type = max_blocks, storage_type
        shape = (max_blocks, num_heads, tokens_per_block, head_dim)
        if storage_type == KvStorageType.FP32:
            mk = lambda: torch.zeros(shape, dtype=torch.float32, device=self.device)
        elif storage_type == KvStorageType.BF16:
            mk = lambda: torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        elif storage_type == KvStorageType.INT8:
            mk = lambda: torch.zeros(shape, dtype=torch.int8, device=self.device)
        else:  # INT4: packed, (blockElements + 1) / 2 bytes per block (:80-84)
            elems = num_heads * tokens_per_block * head_dim
            mk = lambda: torch.zeros((max_blocks, (elems + 1) // 2), dtype=torch.uint8,
                                     device=self.device)
        self.k_slab, self.v_slab = mk(), mk()
        if storage_type in (KvStorageType.INT8, KvStorageType.INT4):
            self.k_scale = torch.zeros((max_blocks, num_heads, tokens_per_block), dtype=torch.float32,
                                       device=self.device)
            self.v_scale = torch.zeros_like(self.k_scale)
        else:
            self.k_scale = self.v_scale = None
        self._reset_free()
        self.initialized = True

    def _reset_free(self):
        self._free = collections.deque(range(self.max_blocks))

    def allocate_block(self):
        return self._free.popleft() if self._free else None

    def free_block(self, index: int) -> None:
        self._free.append(index)

    def get_block_size_bytes(self) -> int:
        elems = self.num_heads * self.tokens_per_block * self.head_dim
        return {KvStorageType.FP32: elems * 4, KvStorageType.BF16: elems * 2,
                KvStorageType.INT8: elems, KvStorageType.INT4: (elems + 1) // 2}[self.storage_type]

    def scale_strides(self):
        """(page, head, token) strides of the per-token scale slabs."""
        return (self.num_heads * self.tokens_per_block, self.tokens_per_block, 1)

    def close(self):
        self.k_slab = self.v_slab = self.k_scale = self.v_scale = None
        self._free.clear()
        self.initialized = False
        self.max_blocks = 0


class KVCacheSession:
    """KVCacheManager.KVCacheSession (kv/KVCacheManager.java:30-233): one block table per
    layer, all drawing on one BlockManager; tokensPerBlock 16 (:57)."""

    def __init__(self, max_seq_len: int, block_manager: BlockManager):
        self.max_seq_len = max_seq_len
        self.block_manager = block_manager
        self.block_tables: dict[int, list[int]] = {}
        self.current_pos = 0
        self.tokens_per_block = 16

    def allocate(self, num_layers: int, num_kv_heads: int, head_dim: int,
                 storage: KvStorageType = KvStorageType.FP32) -> None:
        """KVCacheSession.allocate (:51-81): pool sized for min(maxSeqLen, 4096) tokens."""
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        safe = min(self.max_seq_len, 4096)
        initial = (safe // self.tokens_per_block) * num_layers + 64
        self.block_manager.initialize(self.tokens_per_block, num_kv_heads, head_dim, initial, storage)
        for i in range(num_layers):
            self.block_tables[i] = []
            self._append_block(i)

    def _append_block(self, layer: int) -> None:
        b = self.block_manager.allocate_block()
        if b is None:
            raise IllegalStateError("KVCache: Out of physical blocks!")
        self.block_tables[layer].append(b)

    def ensure_capacity(self, total_tokens_needed: int) -> None:
        if total_tokens_needed <= 0:
            return
        need = (total_tokens_needed + self.tokens_per_block - 1) // self.tokens_per_block
        for i in range(self.num_layers):
            while len(self.block_tables[i]) < need:
                self._append_block(i)

    def advance(self, seq_len: int) -> None:
        prev = 0 if self.current_pos == 0 else (self.current_pos + self.tokens_per_block - 1) // self.tokens_per_block
        self.current_pos += seq_len
        new = (self.current_pos + self.tokens_per_block - 1) // self.tokens_per_block
        for i in range(self.num_layers):
            while len(self.block_tables[i]) < new:
                self._append_block(i)

    def get_block_for_token(self, layer: int, token: int) -> int:
        table = self.block_tables.get(layer)
        if table is None or token < 0:
            return -1
        idx = token // self.tokens_per_block
        while idx >= len(table):
            self._append_block(layer)
        return table[idx]

    def get_block_table(self, layer: int) -> list[int]:
        return self.block_tables[layer]

    def block_table_tensor(self, layer: int, width: int | None = None):
        import torch
        t = self.block_tables[layer]
        w = width or max(1, len(t))
        row = t + [-1] * (w - len(t))
        return torch.tensor([row], dtype=torch.int32, device=self.block_manager.device)

    def close(self):
        for t in self.block_tables.values():
            for b in t:
                self.block_manager.free_block(b)
        self.block_tables.clear()
        self.block_manager.close()


def _kv_args(bm: BlockManager):
    return dict(k_scales=bm.k_scale, v_scales=bm.v_scale,
                scale_strides=bm.scale_strides() if bm.k_scale is not None else (0, 0, 0),
                int4=bm.storage_type == KvStorageType.INT4)


def update_cache(key, value, session: KVCacheSession, layer_idx: int, start_pos: int,
                 seq_len: int) -> None:
    """PagedKvCacheIO.updateCache (attention/PagedKvCacheIO.java:23-62): key/value
    [seq_len, num_kv_heads, head_dim] written at positions start_pos .. start_pos+seq_len-1."""
    import torch

    from . import ops
    bm = session.block_manager
    session.ensure_capacity(start_pos + seq_len)
    for p in range(start_pos, start_pos + seq_len):
        if session.get_block_for_token(layer_idx, p) < 0:
            raise IllegalStateError(f"Missing KV block for layer {layer_idx} token {p}")
    dev = key.device
    table = session.block_table_tensor(layer_idx)
    pos = torch.arange(start_pos, start_pos + seq_len, dtype=torch.int32, device=dev)
    seq = torch.zeros(seq_len, dtype=torch.int32, device=dev)
    ops.kv_append(key.reshape(seq_len, session.num_kv_heads, session.head_dim).contiguous(),
                  value.reshape(seq_len, session.num_kv_heads, session.head_dim).contiguous(),
                  pos, table, bm.k_slab, bm.v_slab, block_size=session.tokens_per_block,
                  num_blocks=bm.max_blocks, token_seq=seq, **_kv_args(bm))


def paged_attention_compute(q, session: KVCacheSession, layer_idx: int, total_tokens: int,
                            num_q_heads: int, num_kv_heads: int, head_dim: int, scale: float,
                            soft_cap: float = 0.0, sliding_window: int = 0, out=None,
                            causal: bool = True):
    """PagedAttentionVectorAPI.compute (attention/PagedAttentionVectorAPI.java:60-180):
    q [1, Tq, num_q_heads, head_dim] (fp32 or bf16), query i at position
    total_tokens - Tq + i, attending to the layer's first total_tokens positions (up to its
    own position when causal).  Returns [1, Tq, num_q_heads, head_dim]."""
    import torch

    from . import ops
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("q must be [1, Tq, num_q_heads, head_dim]")
    bm = session.block_manager
    table = session.block_table_tensor(layer_idx)
    ctx = torch.tensor([total_tokens], dtype=torch.int32, device=q.device)
    if q.shape[1] == 1:
        res = ops.paged_attention(q.reshape(1, num_q_heads, head_dim).contiguous(), bm.k_slab,
                                  bm.v_slab, table, ctx, num_kv_heads=num_kv_heads,
                                  block_size=session.tokens_per_block, scale=scale,
                                  num_blocks=bm.max_blocks, soft_cap=soft_cap,
                                  sliding_window=sliding_window, **_kv_args(bm))
    else:
        res = ops.paged_attention_prefill(q.contiguous(), bm.k_slab, bm.v_slab, table, ctx,
                                          num_kv_heads=num_kv_heads,
                                          block_size=session.tokens_per_block, scale=scale,
                                          causal=causal, num_blocks=bm.max_blocks,
                                          soft_cap=soft_cap, sliding_window=sliding_window,
                                          **_kv_args(bm))
    res = res.reshape(q.shape)
    if out is not None:
        out.copy_(res)
        return out
    return res
