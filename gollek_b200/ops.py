"""Tensor-level wrappers over the C ABI (torch CUDA tensors in, status checked).

Every function here is a thin call into libgollek_kernels.so on the tensors' device
and the current torch stream; none has a CPU path.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import BF16, F16, F32, I4, I8, check

_TORCH_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.int8: I8}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor, stream=None):
    if stream is not None:
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("gollek_b200 ops take CUDA tensors only (no CPU path)")


def kv_dtype_code(t: torch.Tensor, int4: bool = False) -> int:
    if int4:
        return I4
    if t.dtype not in _TORCH_DTYPE:
        raise ValueError(f"unsupported KV dtype {t.dtype}")
    return _TORCH_DTYPE[t.dtype]


def workspace_size(num_seqs: int, num_q_heads: int, num_kv_heads: int, head_dim: int) -> int:
    return int(_lib.load().gollek_paged_attention_workspace_size(num_seqs, num_q_heads,
                                                                 num_kv_heads, head_dim))


def new_workspace(num_seqs, num_q_heads, num_kv_heads, head_dim, device) -> torch.Tensor:
    """Caller-owned split-K scratch, zero-filled (the kernels leave it zeroed)."""
    n = workspace_size(num_seqs, num_q_heads, num_kv_heads, head_dim)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def paged_attention(q, k_cache, v_cache, block_tables, context_lens, *, num_kv_heads,
                    block_size, scale=None, num_blocks=0, page_stride=0, k_scales=None,
                    v_scales=None, scale_strides=(0, 0, 0), soft_cap=0.0, sliding_window=0,
                    int4=False, out=None, workspace=None, stream=None):
    """Decode attention (gollek_paged_attention_v2).

    q: [S, Hq, D] fp32/bf16.  k_cache/v_cache: pool tensors (any shape) whose element
    (page p, head h, token t, dim d) sits at p*page_stride + (h*BS + t)*D + d.
    """
    _require_cuda(q, k_cache, v_cache, block_tables, context_lens, k_scales, v_scales, out)
    S, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    sps, shs, sts = scale_strides
    lib = _lib.load()
    rc = lib.gollek_paged_attention_v2(
        _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k_scales), _ptr(v_scales),
        _ptr(block_tables), _ptr(context_lens), S, Hq, int(num_kv_heads), D, int(block_size),
        block_tables.shape[1], int(num_blocks), int(page_stride), _TORCH_DTYPE[q.dtype],
        kv_dtype_code(k_cache, int4), int(sps), int(shs), int(sts), float(scale),
        float(soft_cap), int(sliding_window), _ptr(workspace),
        0 if workspace is None else workspace.numel() * workspace.element_size(),
        _stream(q, stream))
    check(rc)
    return out


def paged_attention_prefill(q, k_cache, v_cache, block_tables, context_lens, *, num_kv_heads,
                            block_size, scale=None, causal=True, num_blocks=0, page_stride=0,
                            k_scales=None, v_scales=None, scale_strides=(0, 0, 0), soft_cap=0.0,
                            sliding_window=0, int4=False, out=None, workspace=None, stream=None):
    """Multi-query attention (gollek_paged_attention_prefill): q [S, Tq, Hq, D]; the Tq
    queries of sequence s sit at positions context_lens[s] - Tq .. context_lens[s] - 1."""
    _require_cuda(q, k_cache, v_cache, block_tables, context_lens, k_scales, v_scales, out)
    S, Tq, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    sps, shs, sts = scale_strides
    rc = _lib.load().gollek_paged_attention_prefill(
        _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k_scales), _ptr(v_scales),
        _ptr(block_tables), _ptr(context_lens), S, Tq, Hq, int(num_kv_heads), D, int(block_size),
        block_tables.shape[1], int(num_blocks), int(page_stride), _TORCH_DTYPE[q.dtype],
        kv_dtype_code(k_cache, int4), int(sps), int(shs), int(sts), float(scale),
        float(soft_cap), int(sliding_window), int(bool(causal)), _ptr(workspace),
        0 if workspace is None else workspace.numel() * workspace.element_size(),
        _stream(q, stream))
    check(rc)
    return out


def paged_attention_launch(out, q, k_cache, v_cache, block_tables, context_lens, scale):
    """The legacy fp32 entry point (synchronous): q/out [S,H,D], K/V [NB,H,BS,D]."""
    _require_cuda(out, q, k_cache, v_cache, block_tables, context_lens)
    S, H, D = q.shape
    rc = _lib.load().paged_attention_launch(
        _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_tables), _ptr(context_lens),
        S, H, D, k_cache.shape[2], block_tables.shape[1], float(scale))
    check(rc)
    return out


def kv_append(key, value, token_pos, block_tables, k_cache, v_cache, *, block_size,
              num_blocks=0, token_seq=None, page_stride=0, k_scales=None, v_scales=None,
              scale_strides=(0, 0, 0), int4=False, stream=None):
    """Write [T, Hkv, D] key/value rows into their pages (gollek_kv_append)."""
    _require_cuda(key, value, token_pos, block_tables, k_cache, v_cache, token_seq, k_scales,
                  v_scales)
    T, Hkv, D = key.shape
    sps, shs, sts = scale_strides
    rc = _lib.load().gollek_kv_append(
        _ptr(key), _ptr(value), _TORCH_DTYPE[key.dtype], _ptr(token_seq), _ptr(token_pos),
        _ptr(block_tables), block_tables.shape[1], int(num_blocks), _ptr(k_cache), _ptr(v_cache),
        _ptr(k_scales), _ptr(v_scales), kv_dtype_code(k_cache, int4), T, Hkv, D, int(block_size),
        int(page_stride), int(sps), int(shs), int(sts), _stream(key, stream))
    check(rc)


def pool_blocks(pool, block_stride, bytes_per_block) -> int:
    """Whole blocks of `bytes_per_block` bytes, `block_stride` bytes apart, that fit in
    the tensor `pool` (the bound the migration and checksum kernels check ids against)."""
    nbytes = pool.numel() * pool.element_size()
    if nbytes < bytes_per_block or block_stride <= 0:
        return 0 if block_stride <= 0 else -1
    return (nbytes - bytes_per_block) // block_stride + 1


def kv_migrate(src_k, src_v, dst_k, dst_v, src_blocks, dst_blocks, *, src_block_stride,
               dst_block_stride, bytes_per_block, device=None, stream=None, dst_k_ptr=None,
               dst_v_ptr=None, src_num_blocks=None, dst_num_blocks=None):
    """Block-remapped copy (gollek_kv_migrate).  Strides/sizes in bytes.

    dst_k_ptr/dst_v_ptr override the destination with raw device addresses (a peer
    pointer mapped through CUDA IPC); give dst_num_blocks with them.  Pool sizes default
    to what the tensors hold, so ids outside a pool are skipped on the device and
    reported by device_status() (GOLLEK_STATUS_BAD_BLOCK_ID)."""
    dev = src_k.device.index if device is None else device
    dk = dst_k_ptr if dst_k_ptr is not None else _ptr(dst_k)
    dv = dst_v_ptr if dst_v_ptr is not None else _ptr(dst_v)
    if src_num_blocks is None:
        src_num_blocks = pool_blocks(src_k, src_block_stride, bytes_per_block)
    if dst_num_blocks is None:
        dst_num_blocks = (pool_blocks(dst_k, dst_block_stride, bytes_per_block)
                          if dst_k_ptr is None else 0)
    if src_num_blocks < 0 or dst_num_blocks < 0:
        raise ValueError("a pool tensor is smaller than one block")
    rc = _lib.load().gollek_kv_migrate(
        _ptr(src_k), _ptr(src_v), dk, dv, _ptr(src_blocks), _ptr(dst_blocks), src_blocks.numel(),
        int(src_num_blocks), int(dst_num_blocks), int(src_block_stride), int(dst_block_stride),
        int(bytes_per_block), int(dev), _stream(src_k, stream))
    check(rc)


def block_checksums(pool, blocks, *, block_stride, bytes_per_block, num_blocks=None, stream=None):
    """Per-block 64-bit checksums (gollek_kv_block_checksum) as an int64 tensor."""
    if num_blocks is None:
        num_blocks = pool_blocks(pool, block_stride, bytes_per_block)
    if num_blocks < 0:
        raise ValueError("the pool tensor is smaller than one block")
    out = torch.empty(blocks.numel(), dtype=torch.int64, device=pool.device)
    rc = _lib.load().gollek_kv_block_checksum(_ptr(pool), _ptr(blocks), blocks.numel(),
                                              int(num_blocks), int(block_stride),
                                              int(bytes_per_block), _ptr(out), _stream(pool, stream))
    check(rc)
    return out


def device_status(device: int = 0, clear: bool = True) -> int:
    import ctypes
    v = ctypes.c_uint(0)
    check(_lib.load().gollek_device_status(int(device), int(clear), ctypes.byref(v)))
    return int(v.value)


def enable_peer_access(device: int, peer: int) -> None:
    check(_lib.load().gollek_enable_peer_access(int(device), int(peer)))
