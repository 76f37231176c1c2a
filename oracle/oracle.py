"""ctypes wrapper around the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker or the timed CPU baseline.  The
product package ``gollek_b200`` never imports it.

Every function restates one reference routine; the C file names the reference
file:line each one follows.  Arrays are numpy, C-contiguous.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

FP32, INT8, INT4 = 0, 1, 2
STORAGE = {"fp32": FP32, "int8": INT8, "int4": INT4}

_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p


def build() -> str:
    """Compile the oracle with its Makefile (system gcc, Java float semantics)."""
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        c_int, c_float, c_ll = ctypes.c_int, ctypes.c_float, ctypes.c_longlong
        L.oracle_a1_execute.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, _i32p, c_int, c_int,
                                        c_int, c_int, c_int, c_float, c_int]
        L.oracle_a1_execute.restype = c_int
        L.oracle_a2_compute.argtypes = [_f32p, _f32p, c_int, c_int, c_int, c_int, c_int, c_int,
                                        _vp, _vp, _vp, _vp, c_int, _i32p, _i32p, c_int, c_float,
                                        c_int, c_float, c_int, c_int, c_int]
        L.oracle_a2_compute.restype = c_int
        L.oracle_fp32_dot.argtypes = [_f32p, _f32p, c_int, c_int]
        L.oracle_fp32_dot.restype = c_float
        L.oracle_fp32_update.argtypes = [_f32p, _f32p, c_float, c_float, c_int]
        L.oracle_fp32_update.restype = None
        L.oracle_score.argtypes = [c_int, _f32p, _vp, c_ll, _vp, c_ll, c_int, c_float, c_int]
        L.oracle_score.restype = c_float
        L.oracle_update.argtypes = [c_int, _f32p, _vp, c_ll, _vp, c_ll, c_float, c_float, c_int]
        L.oracle_update.restype = None
        L.oracle_softmax_observe.argtypes = [_f32p, c_int, ctypes.POINTER(c_float),
                                             ctypes.POINTER(c_float), ctypes.POINTER(c_float)]
        L.oracle_softmax_observe.restype = c_float
        L.oracle_java_round.argtypes = [c_float]
        L.oracle_java_round.restype = c_int
        L.oracle_write_vector.argtypes = [c_int, _f32p, _vp, c_ll, _vp, c_ll, c_int]
        L.oracle_write_vector.restype = None
        L.oracle_read_vector.argtypes = [c_int, _vp, _vp, c_ll, c_ll, _f32p, c_int]
        L.oracle_read_vector.restype = None
        L.oracle_update_cache.argtypes = [_f32p, _f32p, c_int, _vp, _i32p, _i32p, c_int, c_int,
                                          c_int, c_int, c_int, _vp, _vp, _vp, _vp]
        L.oracle_update_cache.restype = c_int
        L.oracle_migrate.argtypes = [_vp, _vp, _vp, _vp, _i32p, _i32p, c_int, c_int, c_ll]
        L.oracle_migrate.restype = c_ll
        L.oracle_num_threads.argtypes = []
        L.oracle_num_threads.restype = c_int
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def num_threads() -> int:
    return lib().oracle_num_threads()


# --------------------------------------------------------------------- a1

def a1_execute(q, k_cache, v_cache, block_tables, context_lens, scale, threads=1):
    """PagedAttentionCpuFallback.execute: q [S,H,D], K/V [NB,H,BS,D] fp32."""
    q = _f32(q)
    k_cache, v_cache = _f32(k_cache), _f32(v_cache)
    bt, ctx = _i32(block_tables), _i32(context_lens)
    S, H, D = q.shape
    BS = k_cache.shape[2]
    out = np.zeros_like(q)
    rc = lib().oracle_a1_execute(out, q, k_cache, v_cache, bt, ctx, S, H, D, BS, bt.shape[1],
                                 float(scale), int(threads))
    assert rc == 0
    return out


# --------------------------------------------------------------------- a2

def block_bytes(storage: int, hkv: int, bs: int, d: int) -> int:
    elems = hkv * bs * d
    return elems * 4 if storage == FP32 else (elems if storage == INT8 else (elems + 1) // 2)


def a2_compute(q, k_slab, v_slab, block_tables, context_lens, scale, *, storage=FP32,
               num_kv_heads, block_size, k_scale=None, v_scale=None, causal=True,
               soft_cap=0.0, sliding_window=0, lanes=8, threads=1):
    """PagedAttentionVectorAPI.compute for a batch of sequences.

    q: [S, Tq, Hq, D] fp32.  k_slab/v_slab: BlockManager slabs, fp32 [NB,Hkv,BS,D]
    or raw bytes (int8 / packed int4) of NB blocks.  k_scale/v_scale: fp32
    [NB, Hkv, BS] per-token scales (INT8/INT4), or None (scale 1.0).
    """
    q = _f32(q)
    if q.ndim == 3:
        q = q[:, None]
    S, Tq, Hq, D = q.shape
    out = np.zeros_like(q)
    bt, ctx = _i32(block_tables), _i32(context_lens)
    k_slab = np.ascontiguousarray(k_slab)
    v_slab = np.ascontiguousarray(v_slab)
    ks = None if k_scale is None else _f32(k_scale)
    vs = None if v_scale is None else _f32(v_scale)
    rc = lib().oracle_a2_compute(out, q, S, Tq, Hq, int(num_kv_heads), D, int(block_size),
                                 _ptr(k_slab), _ptr(v_slab), _ptr(ks), _ptr(vs), int(storage), bt,
                                 ctx, bt.shape[1], float(scale), int(bool(causal)), float(soft_cap),
                                 int(sliding_window), int(lanes), int(threads))
    assert rc == 0, rc
    return out


# ------------------------------------------------------- single-call kernels

def fp32_dot(q, k, lanes=8):
    q, k = _f32(q), _f32(k)
    return float(lib().oracle_fp32_dot(q, k, q.size, lanes))


def fp32_update(acc, v, prev, cur):
    acc = _f32(acc).copy()
    lib().oracle_fp32_update(acc, _f32(v), prev, cur, acc.size)
    return acc


def score(storage, q, k, elem0=0, scale_seg=None, scale_idx=0, dim=None, scale=1.0, lanes=8):
    q = _f32(q)
    k = np.ascontiguousarray(k)
    ss = None if scale_seg is None else _f32(scale_seg)
    dim = q.size if dim is None else dim
    return float(lib().oracle_score(storage, q, _ptr(k), elem0, _ptr(ss), scale_idx, dim,
                                    float(scale), lanes))


def update(storage, acc, v, elem0=0, scale_seg=None, scale_idx=0, prev=0.0, cur=0.0, dim=None):
    acc = _f32(acc).copy()
    v = np.ascontiguousarray(v)
    ss = None if scale_seg is None else _f32(scale_seg)
    dim = acc.size if dim is None else dim
    lib().oracle_update(storage, acc, _ptr(v), elem0, _ptr(ss), scale_idx, prev, cur, dim)
    return acc


def softmax_observe(scores):
    s = _f32(scores)
    p, c, inv = ctypes.c_float(), ctypes.c_float(), ctypes.c_float()
    norm = lib().oracle_softmax_observe(s, s.size, ctypes.byref(p), ctypes.byref(c),
                                        ctypes.byref(inv))
    return norm, p.value, c.value, inv.value


def java_round(x: float) -> int:
    return int(lib().oracle_java_round(float(x)))


def write_vector(storage, src, dst, dst_elem=0, scale_seg=None, scale_idx=0):
    """Quantise/copy one vector into ``dst`` (modified in place)."""
    src = _f32(src)
    lib().oracle_write_vector(storage, src, _ptr(dst), dst_elem, _ptr(scale_seg), scale_idx,
                              src.size)


def read_vector(storage, src, scale_seg, src_elem, scale_idx, dim):
    out = np.zeros(dim, np.float32)
    lib().oracle_read_vector(storage, _ptr(np.ascontiguousarray(src)),
                             _ptr(None if scale_seg is None else _f32(scale_seg)), src_elem,
                             scale_idx, out, dim)
    return out


def update_cache(key, value, token_pos, block_tables, *, storage, k_slab, v_slab,
                 k_scale=None, v_scale=None, token_seq=None, block_size):
    """PagedKvCacheIO.updateCache for a batch of tokens; slabs modified in place.

    key/value: [T, Hkv, D] fp32.  Returns the C status (0, or -1 for a missing block).
    """
    key, value = _f32(key), _f32(value)
    T, Hkv, D = key.shape
    ts = None if token_seq is None else _i32(token_seq)
    bt = _i32(block_tables)
    return lib().oracle_update_cache(key, value, T, _ptr(ts), _i32(token_pos), bt, bt.shape[1],
                                     Hkv, D, int(block_size), int(storage), _ptr(k_slab),
                                     _ptr(v_slab), _ptr(k_scale), _ptr(v_scale))


def migrate(src_k, src_v, dst_k, dst_v, src_blocks, dst_blocks, num_layers, bytes_per_block):
    """transferKvToDecodePartition's copy loop over [block][layer][bytes] pools (in place)."""
    sb, db = _i32(src_blocks), _i32(dst_blocks)
    return int(lib().oracle_migrate(_ptr(src_k), _ptr(src_v), _ptr(dst_k), _ptr(dst_v), sb, db,
                                    sb.size, int(num_layers), int(bytes_per_block)))


# ------------------------------------------------------------ bf16 helpers

def f32_to_bf16_bits(x) -> np.ndarray:
    """Round fp32 to bf16 (round-to-nearest-even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))
