"""Multi-query paged attention (gollek_paged_attention_prefill) against the oracle's
restatement of PagedAttentionVectorAPI.compute with seqLenQ > 1 (causal / non-causal,
sliding window, soft-cap; fp32, bf16 and int8 KV), through the C ABI.

Tolerances as for decode: fp32 <= 1e-4 relative to the output scale; bf16 / int8 KV
<= 2e-2 absolute against the fp32 oracle on the same rounded inputs.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import decode_case, quantize_rows_int8

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _t(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dtype is None else t.to(dtype)


def _case(ctx, tq, hq, hkv, seed, bs=16):
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=hkv, d=128, bs=bs, seed=seed, kv_std=0.5)
    rng = np.random.default_rng(seed + 1)
    qm = rng.standard_normal((len(ctx), tq, hq, 128)).astype(np.float32)
    return qm, k, v, bt, ctx


def _oracle(q, k, v, bt, ctx, scale, *, hkv, bs, causal, window=0, soft_cap=0.0, storage=O.FP32,
            ks=None, vs=None):
    return O.a2_compute(q, k, v, bt, ctx, scale, storage=storage, num_kv_heads=hkv, block_size=bs,
                        k_scale=ks, v_scale=vs, causal=causal, soft_cap=soft_cap,
                        sliding_window=window, threads=O.num_threads())


@pytest.mark.parametrize("tq,causal,window,soft_cap", [(1, 1, 0, 0.0), (4, 1, 0, 0.0), (8, 1, 0, 0.0),
                                                       (5, 0, 0, 0.0), (6, 1, 64, 0.0), (3, 1, 0, 30.0)])
def test_prefill_bf16(cuda_device, tq, causal, window, soft_cap):
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([3, 17, 300, 2100, 6000], tq, 32, 8, seed=50 + tq)
    qb, kb, vb = O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)
    scale = 1 / math.sqrt(128)
    want = _oracle(qb, kb, vb, bt, ctx, scale, hkv=8, bs=16, causal=causal, window=window,
                   soft_cap=soft_cap)
    for _ in range(2):
        out = ops.paged_attention_prefill(_t(qb, cuda_device, torch.bfloat16),
                                          _t(kb, cuda_device, torch.bfloat16),
                                          _t(vb, cuda_device, torch.bfloat16), _t(bt, cuda_device),
                                          _t(ctx, cuda_device), num_kv_heads=8, block_size=16,
                                          scale=scale, causal=bool(causal), num_blocks=k.shape[0],
                                          sliding_window=window, soft_cap=soft_cap)
        np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)
    assert ops.device_status(cuda_device.index or 0) == 0


def test_prefill_fp32_gqa8(cuda_device):
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([40, 129, 777], 4, 64, 8, seed=61)
    scale = 1 / math.sqrt(128)
    want = _oracle(q, k, v, bt, ctx, scale, hkv=8, bs=16, causal=1)
    out = ops.paged_attention_prefill(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                                      _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8,
                                      block_size=16, scale=scale, num_blocks=k.shape[0])
    got = out.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_prefill_int8_reference_scales(cuda_device):
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([9, 250, 1500], 3, 32, 8, seed=62)
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    qb = O.round_bf16(q)
    scale = 1 / math.sqrt(128)
    want = _oracle(qb, kq, vq, bt, ctx, scale, hkv=8, bs=16, causal=1, storage=O.INT8, ks=ks, vs=vs)
    out = ops.paged_attention_prefill(_t(qb, cuda_device, torch.bfloat16), _t(kq, cuda_device),
                                      _t(vq, cuda_device), _t(bt, cuda_device), _t(ctx, cuda_device),
                                      num_kv_heads=8, block_size=16, scale=scale,
                                      num_blocks=k.shape[0], k_scales=_t(ks, cuda_device),
                                      v_scales=_t(vs, cuda_device), scale_strides=(8 * 16, 16, 1))
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)


def test_prefill_more_queries_than_context(cuda_device):
    """Sequences shorter than the query count: queries before the first position see
    nothing and come out as zeros, as in the reference (no token passes the causal bound)."""
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([2, 5, 40], 6, 16, 8, seed=63)
    scale = 1 / math.sqrt(128)
    want = _oracle(q, k, v, bt, ctx, scale, hkv=8, bs=16, causal=1)
    out = ops.paged_attention_prefill(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                                      _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8,
                                      block_size=16, scale=scale, num_blocks=k.shape[0])
    got = out.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-4 * max(np.abs(want).max(), 1e-6)
    assert not got[0, :4].any() and not got[1, :1].any()


def test_prefill_refuses_window_without_causal(cuda_device):
    from gollek_b200 import _lib, ops
    q, k, v, bt, ctx = _case([40], 2, 8, 8, seed=64)
    with pytest.raises(_lib.GollekError) as e:
        ops.paged_attention_prefill(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                                    _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8,
                                    block_size=16, causal=False, sliding_window=16,
                                    num_blocks=k.shape[0])
    assert e.value.code == _lib.ERR_UNSUPPORTED


def _prefill(q, k, v, bt, ctx, dev, *, hkv, q_dtype, kv_dtype, scale):
    from gollek_b200 import ops
    return ops.paged_attention_prefill(_t(q, dev, q_dtype), _t(k, dev, kv_dtype), _t(v, dev, kv_dtype),
                                       _t(bt, dev), _t(ctx, dev), num_kv_heads=hkv, block_size=16,
                                       scale=scale, causal=True, num_blocks=k.shape[0])


@pytest.mark.parametrize("hq,hkv,tq", [(32, 8, 2), (32, 8, 4), (32, 8, 8), (8, 8, 8), (16, 8, 4),
                                       (16, 8, 6), (64, 8, 2), (8, 8, 16), (16, 8, 8), (64, 8, 6)])
def test_prefill_page_once_chunks(cuda_device, monkeypatch, hq, hkv, tq):
    """Causal bf16 multi-query calls whose queries fold into the decode kernel's rows
    (F queries x G heads <= 16 per page read with head_dim 128, F the largest power of two
    dividing Tq; 16 rows use the kernel's second value MMA):
    against the oracle, and against the same call with folding turned off
    (GOLLEK_PREFILL_FOLD=0: one decode sequence per query).  Lengths below Tq give queries
    that see nothing (zeros); 6000 tokens split across CTAs (split-K merge per row)."""
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([2, 5, 17, 300, 2100, 6000], tq, hq, hkv, seed=70 + tq + hq)
    qb, kb, vb = O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)
    scale = 1 / math.sqrt(128)
    want = _oracle(qb, kb, vb, bt, ctx, scale, hkv=hkv, bs=16, causal=1)
    folded = [_prefill(qb, kb, vb, bt, ctx, cuda_device, hkv=hkv, q_dtype=torch.bfloat16,
                       kv_dtype=torch.bfloat16, scale=scale).float().cpu().numpy() for _ in range(2)]
    monkeypatch.setenv("GOLLEK_PREFILL_FOLD", "0")
    per_query = _prefill(qb, kb, vb, bt, ctx, cuda_device, hkv=hkv, q_dtype=torch.bfloat16,
                         kv_dtype=torch.bfloat16, scale=scale).float().cpu().numpy()
    for got in folded + [per_query]:
        np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    np.testing.assert_allclose(folded[0], per_query, atol=1e-2, rtol=0)
    # queries before a sequence's first position see nothing
    assert not folded[0][0, :max(0, tq - 2)].any()
    assert ops.device_status(cuda_device.index or 0) == 0


@pytest.mark.parametrize("kv", ["f16", "bf16_fp32q"])
def test_prefill_page_once_other_types(cuda_device, kv):
    """Folded queries on the f16-KV kernel (q split into f16 hi + lo, power-of-two
    prescale) and with fp32 q over bf16 KV (hi + lo bf16 halves)."""
    q, k, v, bt, ctx = _case([31, 700, 3000], 4, 32, 8, seed=81)
    scale = 1 / math.sqrt(128)
    if kv == "f16":
        kr = k.astype(np.float16).astype(np.float32)
        vr = v.astype(np.float16).astype(np.float32)
        qr, q_dt, kv_dt = O.round_bf16(q), torch.bfloat16, torch.float16
    else:
        kr, vr = O.round_bf16(k), O.round_bf16(v)
        qr, q_dt, kv_dt = q, torch.float32, torch.bfloat16
    want = _oracle(qr, kr, vr, bt, ctx, scale, hkv=8, bs=16, causal=1)
    got = _prefill(qr, kr, vr, bt, ctx, cuda_device, hkv=8, q_dtype=q_dt, kv_dtype=kv_dt,
                   scale=scale).float().cpu().numpy()
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("hq,tq,scales,qf32", [(32, 2, "token", False), (32, 4, "page", False),
                                               (16, 4, "token", False), (8, 8, "page", False),
                                               (32, 2, "token", True)])
def test_prefill_page_once_int8(cuda_device, monkeypatch, hq, tq, scales, qf32):
    """Causal multi-query calls over int8 KV fold F queries x G heads <= 8 rows into one
    page pass of the int8 tensor-pipe kernel, with the reference's per-token scales or
    one scale per (page, kv-head): against the oracle's INT8 restatement and against the
    per-query form (GOLLEK_PREFILL_FOLD=0)."""
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([3, 20, 333, 1900, 5000], tq, hq, 8, seed=90 + tq + hq)
    if scales == "token":
        kq, ks = quantize_rows_int8(k)
        vq, vs = quantize_rows_int8(v)
        strides, ks_t, vs_t = (8 * 16, 16, 1), ks, vs
    else:  # one scale per (page, kv-head): absmax over the page's rows / 127
        def per_page(x):
            amax = np.abs(x).max(axis=(2, 3))
            sc = np.where(amax == 0, 1.0, amax / 127.0).astype(np.float32)
            qq = np.clip(np.floor(x / sc[:, :, None, None] + 0.5), -127, 127).astype(np.int8)
            return qq, sc
        kq, ks_t = per_page(k)
        vq, vs_t = per_page(v)
        ks = np.repeat(ks_t[:, :, None], 16, axis=2)
        vs = np.repeat(vs_t[:, :, None], 16, axis=2)
        strides = (8, 1, 0)
    qr = q if qf32 else O.round_bf16(q)
    scale = 1 / math.sqrt(128)
    want = _oracle(qr, kq, vq, bt, ctx, scale, hkv=8, bs=16, causal=1, storage=O.INT8, ks=ks, vs=vs)

    def call():
        return ops.paged_attention_prefill(
            _t(qr, cuda_device, torch.float32 if qf32 else torch.bfloat16), _t(kq, cuda_device),
            _t(vq, cuda_device), _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8,
            block_size=16, scale=scale, num_blocks=k.shape[0], k_scales=_t(ks_t, cuda_device),
            v_scales=_t(vs_t, cuda_device), scale_strides=strides).float().cpu().numpy()

    folded = [call(), call()]
    monkeypatch.setenv("GOLLEK_PREFILL_FOLD", "0")
    per_query = call()
    for got in folded + [per_query]:
        np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    np.testing.assert_allclose(folded[0], per_query, atol=1e-2, rtol=0)
    assert not folded[0][0, :max(0, tq - 3)].any()
    assert ops.device_status(cuda_device.index or 0) == 0


@pytest.mark.parametrize("hq,hkv,d,tq", [(8, 8, 64, 8), (32, 8, 128, 2), (16, 8, 128, 4)])
def test_prefill_page_once_fp32(cuda_device, monkeypatch, hq, hkv, d, tq):
    """Causal multi-query calls over the reference's own fp32 KV storage fold F queries x
    G heads <= 8 rows into one page pass of the CUDA-core fp32 kernel: within 1e-4 of the
    output scale against the oracle, with folding and without (GOLLEK_PREFILL_FOLD=0)."""
    from gollek_b200 import ops
    qd, k, v, bt, ctx = decode_case([4, 37, 301, 512, 3000], hq=hq, hkv=hkv, d=d, bs=16,
                                    seed=110 + tq + hq, kv_std=1.0)
    q = np.random.default_rng(111 + tq).standard_normal((len(ctx), tq, hq, d)).astype(np.float32)
    scale = 1 / math.sqrt(d)
    want = _oracle(q, k, v, bt, ctx, scale, hkv=hkv, bs=16, causal=1)

    def call():
        return ops.paged_attention_prefill(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                                           _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=hkv,
                                           block_size=16, scale=scale,
                                           num_blocks=k.shape[0]).cpu().numpy()

    folded = [call(), call()]
    monkeypatch.setenv("GOLLEK_PREFILL_FOLD", "0")
    per_query = call()
    tol = 1e-4 * max(1.0, float(np.abs(want).max()))
    for got in folded + [per_query]:
        assert np.abs(got - want).max() <= tol
    assert not folded[0][0, :max(0, tq - 4)].any()
    assert ops.device_status(cuda_device.index or 0) == 0


def _nan_past_context(k, v, bt, ctx, bs=16):
    """NaN in every pool row no query may read: past each context in its last page."""
    k, v = k.copy(), v.copy()
    for s, n in enumerate(ctx):
        if n > 0 and n % bs:
            page = bt[s, (n - 1) // bs]
            k[page, :, n % bs:] = np.nan
            v[page, :, n % bs:] = np.nan
    return k, v


@pytest.mark.parametrize("hq,hkv,tq,soft_cap,bs", [(32, 8, 16, 0.0, 16), (64, 8, 8, 0.0, 16),
                                                   (64, 8, 16, 0.0, 16), (16, 8, 32, 0.0, 16),
                                                   (8, 8, 64, 0.0, 16), (32, 8, 48, 0.0, 16),
                                                   (32, 8, 16, 30.0, 16), (32, 8, 8, 0.0, 16),
                                                   (32, 8, 16, 0.0, 8), (32, 8, 8, 0.0, 32)])
def test_prefill_tc_rows(cuda_device, monkeypatch, hq, hkv, tq, soft_cap, bs):
    """Folded calls of 32 or 64 rows (F queries x G heads) per (chunk, kv-head): the
    tensor-memory kernel (prefill_tc.cuh) in both forms -- two warps per 32 rows, one per
    half of a tile's tokens (the default), and one warp (GOLLEK_PREFILL_TC_HALVES=0) --
    against the oracle and against the same call on the 16-row mma.sync fold
    (GOLLEK_PREFILL_TC=0).  Lengths below Tq give rows that see
    nothing or part of a tile; NaN fills the page rows past every context; the 6000-token
    sequence splits across CTAs (merged by the last piece); Tq = 48 gives three 16-query
    chunks per sequence."""
    from gollek_b200 import ops
    q, k, v, bt, ctx = _case([2, 5, 17, 300, 2100, 6000], tq, hq, hkv, seed=130 + tq + hq + bs, bs=bs)
    qb, kb, vb = O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)
    scale = 1 / math.sqrt(128)
    want = _oracle(qb, kb, vb, bt, ctx, scale, hkv=hkv, bs=bs, causal=1, soft_cap=soft_cap)
    kn, vn = _nan_past_context(kb, vb, bt, ctx, bs=bs)

    def run():
        return ops.paged_attention_prefill(_t(qb, cuda_device, torch.bfloat16),
                                           _t(kn, cuda_device, torch.bfloat16),
                                           _t(vn, cuda_device, torch.bfloat16), _t(bt, cuda_device),
                                           _t(ctx, cuda_device), num_kv_heads=hkv, block_size=bs,
                                           scale=scale, causal=True, num_blocks=k.shape[0],
                                           soft_cap=soft_cap).float().cpu().numpy()

    tc = [run() for _ in range(2)]
    monkeypatch.setenv("GOLLEK_PREFILL_TC_HALVES", "0")
    one = run()
    monkeypatch.delenv("GOLLEK_PREFILL_TC_HALVES")
    monkeypatch.setenv("GOLLEK_PREFILL_TC", "0")
    mma = run()
    for got in tc + [one, mma]:
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    np.testing.assert_allclose(tc[0], mma, atol=1e-2, rtol=0)
    np.testing.assert_allclose(tc[0], one, atol=1e-2, rtol=0)
    assert not tc[0][0, :max(0, tq - 2)].any()
    assert ops.device_status(cuda_device.index or 0) == 0
