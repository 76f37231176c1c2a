"""Parity of the CUDA decode-attention paths with the CPU oracle (through the C ABI).

Tolerances: fp32 <= 1e-4 relative; bf16 / int8 KV <= 2e-2
absolute against the fp32 oracle on the same rounded inputs.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import decode_case, oracle_decode, quantize_pages_int8, quantize_rows_int8

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _t(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dtype is None else t.to(dtype)


def _fp32_close(got, want):
    # <= 1e-4 relative, measured against the output's scale
    err = np.abs(got - want).max()
    ref = max(np.abs(want).max(), 1e-6)
    assert err <= 1e-4 * ref, f"max err {err} vs scale {ref}"


# ------------------------------------------------------------------ legacy ABI

def test_legacy_config1_fp32(cuda_device):
    """BASELINE config 1 through paged_attention_launch (fp32, MHA)."""
    from gollek_b200 import ops
    rng = np.random.default_rng(1)
    ctx = np.array([37, 128, 301, 512], np.int32)
    H, D, BS, NB = 8, 64, 16, 256
    perm = rng.permutation(NB).astype(np.int32)
    bt = np.zeros((4, 32), np.int32)
    off = 0
    for s, c in enumerate(ctx):
        n = (c + BS - 1) // BS
        bt[s, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((4, H, D)).astype(np.float32)
    k = rng.standard_normal((NB, H, BS, D)).astype(np.float32)
    v = rng.standard_normal((NB, H, BS, D)).astype(np.float32)
    scale = 1.0 / math.sqrt(D)
    want = O.a1_execute(q, k, v, bt, ctx, scale)
    out = torch.empty((4, H, D), dtype=torch.float32, device=cuda_device)
    ops.paged_attention_launch(out, _t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                               _t(bt, cuda_device), _t(ctx, cuda_device), scale)
    _fp32_close(out.cpu().numpy(), want)


def test_legacy_reference_known_answers(cuda_device):
    """PagedAttentionCpuFallbackTest.java:35-148 cases on the device (generic kernel)."""
    from gollek_b200 import ops
    q = np.array([[[1.0, 0.0]]], np.float32)
    k = np.zeros((1, 1, 4, 2), np.float32)
    k[0, 0, 0] = [1, 0]
    k[0, 0, 1] = [0, 1]
    out = torch.empty((1, 1, 2), device=cuda_device)
    ops.paged_attention_launch(out, _t(q, cuda_device), _t(k, cuda_device), _t(k, cuda_device),
                               _t(np.zeros((1, 1), np.int32), cuda_device),
                               _t(np.array([2], np.int32), cuda_device), 1 / math.sqrt(2))
    o = out.cpu().numpy()[0, 0]
    assert o[0] > 0.5 and o[1] < 0.5 and abs(o.sum() - 1) < 1e-3

    k2 = np.array([1, 1, 1, 0], np.float32).reshape(2, 1, 2, 1)
    v2 = np.array([2, 4, 6, 0], np.float32).reshape(2, 1, 2, 1)
    out = torch.empty((1, 1, 1), device=cuda_device)
    ops.paged_attention_launch(out, _t(np.ones((1, 1, 1), np.float32), cuda_device),
                               _t(k2, cuda_device), _t(v2, cuda_device),
                               _t(np.array([[0, 1]], np.int32), cuda_device),
                               _t(np.array([3], np.int32), cuda_device), 1.0)
    assert abs(out.item() - 4.0) < 1e-3


# ------------------------------------------------------------------ v2: bf16 GQA

@pytest.mark.parametrize("hq,hkv,d,bs", [(32, 8, 128, 16), (8, 8, 128, 16), (16, 8, 128, 16),
                                         (64, 8, 128, 16), (32, 8, 64, 16), (32, 8, 128, 8),
                                         (32, 8, 128, 32), (32, 8, 128, 64)])
def test_bf16_gqa_parity(cuda_device, hq, hkv, d, bs):
    from gollek_b200 import ops
    ctx = [1, 31, 32, 33, 200, 517, 1024, 2049, 0, 77]
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=hkv, d=d, bs=bs, seed=hq + d + bs, kv_std=0.5)
    qb, kb, vb = O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)
    scale = 1.0 / math.sqrt(d)
    want = oracle_decode(qb, kb, vb, bt, ctx, scale, hkv=hkv, bs=bs)
    out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kb, cuda_device, torch.bfloat16),
                              _t(vb, cuda_device, torch.bfloat16), _t(bt, cuda_device),
                              _t(ctx, cuda_device), num_kv_heads=hkv, block_size=bs, scale=scale,
                              num_blocks=k.shape[0])
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    assert not got[8].any()  # empty context -> zeros


@pytest.mark.parametrize("window,soft_cap", [(100, 0.0), (0, 30.0), (40, 5.0)])
def test_window_and_softcap(cuda_device, window, soft_cap):
    from gollek_b200 import ops
    ctx = [1, 50, 129, 640, 1000]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=5)
    scale = 1.0 / math.sqrt(128)
    want = oracle_decode(q, k, v, bt, ctx, scale, hkv=8, bs=16, soft_cap=soft_cap, window=window)
    out = ops.paged_attention(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                              _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8,
                              block_size=16, scale=scale, soft_cap=soft_cap, sliding_window=window,
                              num_blocks=k.shape[0])
    _fp32_close(out.cpu().numpy(), want)


@pytest.mark.parametrize("hq,hkv,window,soft_cap,bs", [(32, 1, 0, 0.0, 16), (64, 1, 0, 0.0, 16),
                                                       (256, 8, 0, 0.0, 16), (64, 2, 100, 0.0, 16),
                                                       (32, 1, 0, 30.0, 16), (64, 1, 40, 5.0, 16),
                                                       (32, 1, 0, 0.0, 8), (64, 2, 0, 0.0, 64)])
def test_bf16_large_groups(cuda_device, monkeypatch, hq, hkv, window, soft_cap, bs):
    """Decode with 32 or 64 q heads per kv head (multi-query-attention models): the
    tensor-memory kernel of prefill_tc.cuh with the heads as its rows, against the oracle,
    twice (bit-identical); windows and soft-cap; pages of 8, 16 and 64 tokens; an empty
    context gives zeros; the 9000-token context splits across CTAs.  Both forms of the kernel:
    two warps per 32 heads, one per half of a tile's tokens (the default), and one warp
    (GOLLEK_PREFILL_TC_HALVES=0).  No other kernel serves these groups: with
    GOLLEK_PREFILL_TC=0 the call is refused as unsupported."""
    from gollek_b200 import ops
    ctx = [1, 31, 32, 33, 200, 517, 1024, 2049, 0, 77, 9000]
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=hkv, d=128, bs=bs, seed=hq + hkv + window + bs, kv_std=0.5)
    qb, kb, vb = O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)
    scale = 1.0 / math.sqrt(128)
    want = oracle_decode(qb, kb, vb, bt, ctx, scale, hkv=hkv, bs=bs, window=window, soft_cap=soft_cap)

    def run():
        out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kb, cuda_device, torch.bfloat16),
                                  _t(vb, cuda_device, torch.bfloat16), _t(bt, cuda_device),
                                  _t(ctx, cuda_device), num_kv_heads=hkv, block_size=bs, scale=scale,
                                  soft_cap=soft_cap, sliding_window=window, num_blocks=k.shape[0])
        return out.float().cpu().numpy()

    tc = [run(), run()]
    monkeypatch.setenv("GOLLEK_PREFILL_TC_HALVES", "0")
    one = run()
    monkeypatch.delenv("GOLLEK_PREFILL_TC_HALVES")
    for got in tc + [one]:
        np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    np.testing.assert_array_equal(tc[0], tc[1])
    assert not one[8].any()
    monkeypatch.setenv("GOLLEK_PREFILL_TC", "0")
    from gollek_b200 import _lib
    with pytest.raises(_lib.GollekError) as err:
        run()
    assert err.value.code == _lib.ERR_UNSUPPORTED
    assert not tc[0][8].any()  # empty context -> zeros
    assert ops.device_status(cuda_device.index or 0) == 0


@pytest.mark.parametrize("hq,hkv,d,bs", [(32, 8, 128, 16), (8, 2, 64, 16), (4, 4, 64, 32)])
def test_fp32_gqa_parity(cuda_device, hq, hkv, d, bs):
    from gollek_b200 import ops
    ctx = [3, 64, 300, 1500, 4100]
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=hkv, d=d, bs=bs, seed=11)
    scale = 1.0 / math.sqrt(d)
    want = oracle_decode(q, k, v, bt, ctx, scale, hkv=hkv, bs=bs)
    out = ops.paged_attention(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                              _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=hkv,
                              block_size=bs, scale=scale, num_blocks=k.shape[0])
    _fp32_close(out.cpu().numpy(), want)


@pytest.mark.parametrize("d,bs", [(5, 8), (2, 4), (96, 16), (128, 4)])
def test_generic_shapes(cuda_device, d, bs):
    """Shapes outside the TMA path go through the generic kernel."""
    from gollek_b200 import ops
    ctx = [1, 7, 40, 130]
    q, k, v, bt, ctx = decode_case(ctx, hq=4, hkv=2, d=d, bs=bs, seed=d)
    scale = 0.3
    want = oracle_decode(q, k, v, bt, ctx, scale, hkv=2, bs=bs)
    out = ops.paged_attention(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                              _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=2,
                              block_size=bs, scale=scale, num_blocks=k.shape[0])
    _fp32_close(out.cpu().numpy(), want)


# ------------------------------------------------------------------ v2: int8 / int4

def test_int8_reference_granularity(cuda_device):
    """Per-(block, head, token) scales, the reference's BlockManager layout."""
    from gollek_b200 import ops
    ctx = [5, 100, 333, 1200, 2047]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=21, kv_std=0.5)
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    qb = O.round_bf16(q)
    scale = 1.0 / math.sqrt(128)
    want = oracle_decode(qb, kq, vq, bt, ctx, scale, hkv=8, bs=16, storage=O.INT8, k_scale=ks,
                         v_scale=vs)
    out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kq, cuda_device),
                              _t(vq, cuda_device), _t(bt, cuda_device), _t(ctx, cuda_device),
                              num_kv_heads=8, block_size=16, scale=scale, num_blocks=k.shape[0],
                              k_scales=_t(ks, cuda_device), v_scales=_t(vs, cuda_device),
                              scale_strides=(8 * 16, 16, 1))
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)


def test_int8_page_granularity(cuda_device):
    """one scale per (block, kv-head) from bf16 N(0, 0.5^2) values."""
    from gollek_b200 import ops
    ctx = [17, 512, 900, 3000]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=22, kv_std=0.5)
    k, v = O.round_bf16(k), O.round_bf16(v)
    kq, ks = quantize_pages_int8(k)
    vq, vs = quantize_pages_int8(v)
    qb = O.round_bf16(q)
    scale = 1.0 / math.sqrt(128)
    ks_tok = np.repeat(ks[:, :, None], 16, axis=2)
    vs_tok = np.repeat(vs[:, :, None], 16, axis=2)
    want = oracle_decode(qb, kq, vq, bt, ctx, scale, hkv=8, bs=16, storage=O.INT8,
                         k_scale=ks_tok, v_scale=vs_tok)
    out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kq, cuda_device),
                              _t(vq, cuda_device), _t(bt, cuda_device), _t(ctx, cuda_device),
                              num_kv_heads=8, block_size=16, scale=scale, num_blocks=k.shape[0],
                              k_scales=_t(ks, cuda_device), v_scales=_t(vs, cuda_device),
                              scale_strides=(8, 1, 0))
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    # and against the fp32 oracle on the unquantised bf16 values (quantisation error)
    want_f = oracle_decode(qb, k, v, bt, ctx, scale, hkv=8, bs=16)
    assert np.abs(got - want_f).max() < 5e-2


def test_int4_generic(cuda_device):
    from gollek_b200 import ops
    ctx = [3, 40, 200]
    Hkv, D, BS = 2, 64, 16
    q, k, v, bt, ctx = decode_case(ctx, hq=4, hkv=Hkv, d=D, bs=BS, seed=31)
    nb = k.shape[0]
    kq = np.zeros(nb * Hkv * BS * D // 2, np.uint8)
    vq = np.zeros_like(kq)
    ks = np.zeros(nb * Hkv * BS, np.float32)
    vs = np.zeros_like(ks)
    for r in range(nb * Hkv * BS):
        O.write_vector(O.INT4, k.reshape(-1, D)[r], kq, r * D, ks, r)
        O.write_vector(O.INT4, v.reshape(-1, D)[r], vq, r * D, vs, r)
    scale = 0.125
    want = oracle_decode(q, kq, vq, bt, ctx, scale, hkv=Hkv, bs=BS, storage=O.INT4, k_scale=ks,
                         v_scale=vs)
    out = ops.paged_attention(_t(q, cuda_device), _t(kq, cuda_device), _t(vq, cuda_device),
                              _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=Hkv,
                              block_size=BS, scale=scale, num_blocks=nb, k_scales=_t(ks, cuda_device),
                              v_scales=_t(vs, cuda_device), scale_strides=(Hkv * BS, BS, 1),
                              int4=True)
    _fp32_close(out.cpu().numpy(), want)


# ------------------------------------------------------------------ layouts, scratch, errors

def test_physical_block_pool_layer_view(cuda_device):
    """Attention on one layer of a [block][layer][H*BS*D] pool via base + page_stride."""
    from gollek_b200 import ops
    L, layer = 4, 2
    ctx = [20, 300, 64]
    q, k, v, bt, ctx = decode_case(ctx, hq=16, hkv=8, d=128, bs=16, seed=41)
    nb = k.shape[0]
    kp = np.random.default_rng(0).standard_normal((nb, L, 8, 16, 128)).astype(np.float32)
    vp = np.random.default_rng(1).standard_normal((nb, L, 8, 16, 128)).astype(np.float32)
    kp[:, layer], vp[:, layer] = k, v
    kt, vt = _t(kp, cuda_device, torch.bfloat16), _t(vp, cuda_device, torch.bfloat16)
    want = oracle_decode(O.round_bf16(q), O.round_bf16(k), O.round_bf16(v), bt, ctx,
                         1 / math.sqrt(128), hkv=8, bs=16)
    out = ops.paged_attention(_t(q, cuda_device, torch.bfloat16), kt[:, layer], vt[:, layer],
                              _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8,
                              block_size=16, num_blocks=nb, page_stride=L * 8 * 16 * 128)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)


def test_workspace_stays_zeroed_and_results_repeat(cuda_device):
    from gollek_b200 import ops
    ctx = [4000, 8000, 100, 5000]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=51)
    args = [_t(q, cuda_device, torch.bfloat16), _t(k, cuda_device, torch.bfloat16),
            _t(v, cuda_device, torch.bfloat16), _t(bt, cuda_device), _t(ctx, cuda_device)]
    ws = ops.new_workspace(4, 32, 8, 128, cuda_device)
    outs = [ops.paged_attention(*args, num_kv_heads=8, block_size=16, num_blocks=k.shape[0],
                                workspace=ws) for _ in range(3)]
    lib_out = ops.paged_attention(*args, num_kv_heads=8, block_size=16, num_blocks=k.shape[0])
    torch.cuda.synchronize()
    nctr = 4 * 8
    assert int(ws[: nctr * 4].view(torch.int32).abs().sum()) == 0
    for o in outs[1:] + [lib_out]:
        assert torch.equal(o, outs[0])


def test_page_relocation_is_bit_exact(cuda_device):
    """Moving pages in the pool (and remapping the table) leaves outputs bit-identical."""
    from gollek_b200 import ops
    ctx = [700, 3000, 9]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=61, spare_pages=40)
    nb = k.shape[0]
    perm = np.random.default_rng(7).permutation(nb)
    inv = np.argsort(perm)
    k2, v2 = k[perm], v[perm]                       # new page i holds old page perm[i]
    bt2 = np.where(bt >= 0, inv[np.maximum(bt, 0)], -1).astype(np.int32)
    run = lambda kk, vv, tt: ops.paged_attention(
        _t(q, cuda_device, torch.bfloat16), _t(kk, cuda_device, torch.bfloat16),
        _t(vv, cuda_device, torch.bfloat16), _t(tt, cuda_device), _t(ctx, cuda_device),
        num_kv_heads=8, block_size=16, num_blocks=nb)
    assert torch.equal(run(k, v, bt), run(k2, v2, bt2))


def test_bad_block_id_reports_status(cuda_device):
    from gollek_b200 import ops
    from gollek_b200._lib import STATUS_BAD_BLOCK_ID
    ctx = [40]
    q, k, v, bt, ctx = decode_case(ctx, hq=8, hkv=8, d=128, bs=16, seed=71)
    bt[0, 1] = k.shape[0] + 5  # outside the pool; the kernel must not read it
    ops.device_status(cuda_device.index or 0, clear=True)
    ops.paged_attention(_t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device),
                        _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=8, block_size=16,
                        num_blocks=k.shape[0])
    st = ops.device_status(cuda_device.index or 0, clear=True)
    assert st & STATUS_BAD_BLOCK_ID
    assert ops.device_status(cuda_device.index or 0) == 0


def test_full_config2_sample_parity(cuda_device):
    """BASELINE config 2 at full size; a seeded sample of sequences checked on the oracle."""
    from gollek_b200 import ops
    rng = np.random.default_rng(2024)
    B, Hq, Hkv, D, BS = 64, 32, 8, 128, 16
    ctx = rng.integers(512, 8193, B).astype(np.int32)
    need = (ctx + BS - 1) // BS
    nb = int(need.sum())
    perm = rng.permutation(nb).astype(np.int32)
    maxb = int(need.max())
    bt = np.zeros((B, maxb), np.int32)
    off = 0
    for s in range(B):
        bt[s, :need[s]] = perm[off:off + need[s]]
        off += need[s]
    g = torch.Generator(device=cuda_device).manual_seed(5)
    k = (torch.randn((nb, Hkv, BS, D), generator=g, device=cuda_device) * 0.5).to(torch.bfloat16)
    v = (torch.randn((nb, Hkv, BS, D), generator=g, device=cuda_device) * 0.5).to(torch.bfloat16)
    q = torch.randn((B, Hq, D), generator=g, device=cuda_device).to(torch.bfloat16)
    out = ops.paged_attention(q, k, v, _t(bt, cuda_device), _t(ctx, cuda_device),
                              num_kv_heads=Hkv, block_size=BS, num_blocks=nb)
    sample = [0, int(np.argmax(ctx)), int(np.argmin(ctx)), 33]
    kf, vf = k.float().cpu().numpy(), v.float().cpu().numpy()
    want = oracle_decode(q.float().cpu().numpy()[sample], kf, vf, bt[sample], ctx[sample],
                         1 / math.sqrt(D), hkv=Hkv, bs=BS)
    np.testing.assert_allclose(out.float().cpu().numpy()[sample], want, atol=2e-2, rtol=0)


def test_int8_interleaved_scales_general_path(cuda_device):
    """Scales stored as one [NB][H][BS][2] array (K at even, V at odd slots): strided,
    unaligned scale reads take the per-token copy path."""
    from gollek_b200 import ops
    ctx = [9, 130, 700]
    q, k, v, bt, ctx = decode_case(ctx, hq=16, hkv=8, d=128, bs=16, seed=23, kv_std=0.5)
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    both = np.stack([ks, vs], axis=-1)  # [NB, H, BS, 2]
    scale = 1.0 / math.sqrt(128)
    qb = O.round_bf16(q)
    want = oracle_decode(qb, kq, vq, bt, ctx, scale, hkv=8, bs=16, storage=O.INT8, k_scale=ks,
                         v_scale=vs)
    bt_d = _t(both, cuda_device).reshape(-1)
    out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kq, cuda_device),
                              _t(vq, cuda_device), _t(bt, cuda_device), _t(ctx, cuda_device),
                              num_kv_heads=8, block_size=16, scale=scale, num_blocks=k.shape[0],
                              k_scales=bt_d, v_scales=bt_d[1:],
                              scale_strides=(8 * 16 * 2, 16 * 2, 2))
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)


# ------------------------------------------------------------------ int8 on the tensor pipe

def _int8_call(dev, q, kq, vq, bt, ctx, ks, vs, strides, *, bs=16, hkv=8, window=0, soft_cap=0.0,
               q_dtype=None):
    from gollek_b200 import ops
    scale = 1.0 / math.sqrt(q.shape[-1])
    qd = _t(q, dev) if q_dtype is None else _t(q, dev, q_dtype)
    return ops.paged_attention(qd, _t(kq, dev), _t(vq, dev), _t(bt, dev), _t(ctx, dev),
                               num_kv_heads=hkv, block_size=bs, scale=scale, num_blocks=kq.shape[0],
                               k_scales=_t(ks, dev), v_scales=_t(vs, dev), scale_strides=strides,
                               sliding_window=window, soft_cap=soft_cap)


def test_int8_fp32_query(cuda_device):
    """fp32 q with int8 KV: q enters the f16 MMAs as hi + lo halves."""
    ctx = [7, 260, 1500]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=24, kv_std=0.5)
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    want = oracle_decode(q, kq, vq, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16, storage=O.INT8,
                         k_scale=ks, v_scale=vs)
    out = _int8_call(cuda_device, q, kq, vq, bt, ctx, ks, vs, (8 * 16, 16, 1))
    np.testing.assert_allclose(out.cpu().numpy(), want, atol=2e-2, rtol=0)


def test_int8_large_query_magnitude(cuda_device):
    """|q| far above the f16 range: a power of two is taken out of q and put back on the
    scores."""
    ctx = [50, 300]
    q, k, v, bt, ctx = decode_case(ctx, hq=16, hkv=8, d=128, bs=16, seed=25, kv_std=0.5)
    q = O.round_bf16(q * np.float32(3e5))
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    scale = 1.0 / math.sqrt(128)
    want = oracle_decode(q, kq, vq, bt, ctx, scale, hkv=8, bs=16, storage=O.INT8, k_scale=ks,
                         v_scale=vs)
    out = _int8_call(cuda_device, q, kq, vq, bt, ctx, ks, vs, (8 * 16, 16, 1), q_dtype=torch.bfloat16)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)


def test_int8_scales_spanning_decades(cuda_device):
    """Page scales from 1e-4 to 1e3 in one sequence: the power of two carried by the value
    accumulators moves with them."""
    rng = np.random.default_rng(26)
    ctx = [40, 700, 2100]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=26, kv_std=0.5)
    f = (10.0 ** rng.uniform(-4, 3, size=(k.shape[0], 1, 1, 1))).astype(np.float32)
    k = k * np.float32(0.05)  # keep scores moderate; V carries the wide range
    v = v * f
    for per_token in (True, False):
        if per_token:
            kq, ks = quantize_rows_int8(k)
            vq, vs = quantize_rows_int8(v)
            strides, ks_t, vs_t = (8 * 16, 16, 1), ks, vs
        else:
            kq, ks = quantize_pages_int8(k)
            vq, vs = quantize_pages_int8(v)
            strides = (8, 1, 0)
            ks_t = np.repeat(ks[:, :, None], 16, axis=2)
            vs_t = np.repeat(vs[:, :, None], 16, axis=2)
        qb = O.round_bf16(q)
        want = oracle_decode(qb, kq, vq, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16, storage=O.INT8,
                             k_scale=ks_t, v_scale=vs_t)
        got = _int8_call(cuda_device, qb, kq, vq, bt, ctx, ks, vs, strides,
                         q_dtype=torch.bfloat16).float().cpu().numpy()
        # outputs span decades too: 2e-2 absolute, or 1e-2 of the row's own scale
        err = np.abs(got - want)
        bound = np.maximum(2e-2 * np.minimum(1.0, np.abs(want).max(axis=-1, keepdims=True)),
                           1e-2 * np.abs(want).max(axis=-1, keepdims=True))
        assert (err <= bound).all(), (per_token, float((err / bound).max()))


@pytest.mark.parametrize("bs", [8, 16, 32, 64])
def test_int8_block_sizes(cuda_device, bs):
    ctx = [3, 77, 640]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=bs, seed=27, kv_std=0.5)
    qb = O.round_bf16(q)
    for per_token in (True, False):
        if per_token:
            kq, ks = quantize_rows_int8(k)
            vq, vs = quantize_rows_int8(v)
            strides, ks_t, vs_t = (8 * bs, bs, 1), ks, vs
        else:
            kq, ks = quantize_pages_int8(k)
            vq, vs = quantize_pages_int8(v)
            strides = (8, 1, 0)
            ks_t = np.repeat(ks[:, :, None], bs, axis=2)
            vs_t = np.repeat(vs[:, :, None], bs, axis=2)
        want = oracle_decode(qb, kq, vq, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=bs, storage=O.INT8,
                             k_scale=ks_t, v_scale=vs_t)
        got = _int8_call(cuda_device, qb, kq, vq, bt, ctx, ks, vs, strides, bs=bs,
                         q_dtype=torch.bfloat16)
        np.testing.assert_allclose(got.float().cpu().numpy(), want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("window,soft_cap", [(100, 0.0), (0, 30.0), (40, 5.0)])
def test_int8_window_and_softcap(cuda_device, window, soft_cap):
    ctx = [10, 150, 1000]
    q, k, v, bt, ctx = decode_case(ctx, hq=16, hkv=8, d=128, bs=16, seed=28, kv_std=0.5)
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    qb = O.round_bf16(q)
    want = oracle_decode(qb, kq, vq, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16, storage=O.INT8,
                         k_scale=ks, v_scale=vs, window=window, soft_cap=soft_cap)
    got = _int8_call(cuda_device, qb, kq, vq, bt, ctx, ks, vs, (8 * 16, 16, 1), window=window,
                     soft_cap=soft_cap, q_dtype=torch.bfloat16)
    np.testing.assert_allclose(got.float().cpu().numpy(), want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("hq", [8, 16, 32, 64])
@pytest.mark.parametrize("per_token", [True, False])
def test_int8_long_contexts_split_k(cuda_device, hq, per_token):
    """GQA 1/2/4/8 over contexts long enough that (sequence, kv-head) pairs are cut into
    split-K pieces, a few sequences only (many pieces each), both scale granularities."""
    ctx = [9000, 31, 4097, 12000]
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=8, d=128, bs=16, seed=29 + hq, kv_std=0.5)
    qb = O.round_bf16(q)
    if per_token:
        kq, ks = quantize_rows_int8(k)
        vq, vs = quantize_rows_int8(v)
        strides, ks_t, vs_t = (8 * 16, 16, 1), ks, vs
    else:
        kq, ks = quantize_pages_int8(O.round_bf16(k))
        vq, vs = quantize_pages_int8(O.round_bf16(v))
        strides = (8, 1, 0)
        ks_t = np.repeat(ks[:, :, None], 16, axis=2)
        vs_t = np.repeat(vs[:, :, None], 16, axis=2)
    want = oracle_decode(qb, kq, vq, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16, storage=O.INT8,
                         k_scale=ks_t, v_scale=vs_t)
    got = _int8_call(cuda_device, qb, kq, vq, bt, ctx, ks, vs, strides, q_dtype=torch.bfloat16)
    from gollek_b200 import ops
    assert ops.device_status(cuda_device.index, clear=True) == 0
    np.testing.assert_allclose(got.float().cpu().numpy(), want, atol=2e-2, rtol=0)


def test_int8_stale_table_entries_outside_the_window(cuda_device):
    """Pages wholly before a sliding window, and the page after a context's last token, may
    hold stale table entries (-1 here): they must be neither read nor reported."""
    from gollek_b200 import ops
    ctx = [200, 333, 1000]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=41, kv_std=0.5)
    kq, ks = quantize_rows_int8(k)
    vq, vs = quantize_rows_int8(v)
    qb = O.round_bf16(q)
    window = 100
    bt2 = bt.copy()
    for s_, c in enumerate(ctx):
        first = (int(c) - window) // 16  # first page holding a token of the window
        bt2[s_, :max(0, first)] = -1
        bt2[s_, (int(c) + 15) // 16:] = -1
    want = oracle_decode(qb, kq, vq, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16, storage=O.INT8,
                         k_scale=ks, v_scale=vs, window=window)
    ops.device_status(cuda_device.index, clear=True)
    got = _int8_call(cuda_device, qb, kq, vq, bt2, ctx, ks, vs, (8 * 16, 16, 1), window=window,
                     q_dtype=torch.bfloat16)
    assert ops.device_status(cuda_device.index, clear=True) == 0
    np.testing.assert_allclose(got.float().cpu().numpy(), want, atol=2e-2, rtol=0)


# ------------------------------------------------------------------ both 16-bit kernels

_PATH_CASES = [
    # hq, hkv, bs, q_f32, window, soft_cap
    (32, 8, 16, False, 0, 0.0),
    (64, 8, 16, True, 0, 0.0),
    (128, 8, 16, False, 0, 0.0),
    (8, 8, 16, False, 0, 0.0),
    (16, 8, 16, True, 0, 0.0),
    (32, 8, 8, False, 0, 0.0),
    (32, 8, 32, False, 0, 0.0),
    (32, 8, 16, False, 100, 0.0),
    (32, 8, 16, False, 0, 30.0),
]


@pytest.mark.parametrize("path", ["tc", "mma"])
@pytest.mark.parametrize("hq,hkv,bs,q_f32,window,soft_cap", _PATH_CASES)
def test_bf16_kernel_paths(cuda_device, monkeypatch, path, hq, hkv, bs, q_f32, window, soft_cap):
    """bf16 KV through the tcgen05 kernel and through the mma.sync kernel (selected with
    GOLLEK_DECODE_PATH): contexts that split across CTAs, tiles with 1..8 groups, GQA
    groups 1-16, fp32 q (hi + lo), block sizes 8/16/32, window and soft-cap."""
    from gollek_b200 import ops
    if path == "mma" and hq // hkv > 8:
        pytest.skip("the mma.sync kernel serves GQA groups up to 8")
    monkeypatch.setenv("GOLLEK_DECODE_PATH", path)
    ctx = [9000, 5000, 1, 16, 17, 128, 129, 250, 0, 3000]
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=hkv, d=128, bs=bs, seed=hq + bs + window, kv_std=0.5)
    kb, vb = O.round_bf16(k), O.round_bf16(v)
    qq = q if q_f32 else O.round_bf16(q)
    scale = 1.0 / math.sqrt(128)
    want = oracle_decode(qq, kb, vb, bt, ctx, scale, hkv=hkv, bs=bs, window=window, soft_cap=soft_cap)
    for _ in range(2):  # the split-K scratch must be left zeroed by the first call
        out = ops.paged_attention(_t(qq, cuda_device) if q_f32 else _t(qq, cuda_device, torch.bfloat16),
                                  _t(kb, cuda_device, torch.bfloat16), _t(vb, cuda_device, torch.bfloat16),
                                  _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=hkv,
                                  block_size=bs, scale=scale, num_blocks=k.shape[0],
                                  sliding_window=window, soft_cap=soft_cap)
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
        assert not got[8].any()
    assert ops.device_status(cuda_device.index or 0) == 0


@pytest.mark.parametrize("path", ["tc", "mma"])
def test_bf16_nan_outside_the_context(cuda_device, monkeypatch, path):
    """Pool rows past a sequence's length and before its window hold NaN: they must not
    reach the output (a zero probability does not cancel a NaN on the tensor pipe)."""
    from gollek_b200 import ops
    monkeypatch.setenv("GOLLEK_DECODE_PATH", path)
    ctx = [37, 300, 1000]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=41, kv_std=0.5)
    kb, vb = O.round_bf16(k), O.round_bf16(v)
    qb = O.round_bf16(q)
    window = 200
    want = oracle_decode(qb, kb, vb, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16, window=window)
    kn, vn = kb.copy(), vb.copy()
    for s, c in enumerate(ctx):
        ws = max(0, int(c) - window)
        for t in list(range(ws)) + list(range(int(c), ((int(c) + 15) // 16) * 16)):
            kn[bt[s, t // 16], :, t % 16, :] = np.nan
            vn[bt[s, t // 16], :, t % 16, :] = np.nan
    out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kn, cuda_device, torch.bfloat16),
                              _t(vn, cuda_device, torch.bfloat16), _t(bt, cuda_device),
                              _t(ctx, cuda_device), num_kv_heads=8, block_size=16,
                              scale=1 / math.sqrt(128), num_blocks=k.shape[0], sliding_window=window)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("own_workspace", [True, False])
def test_workspace_reuse_across_batch_sizes(cuda_device, own_workspace):
    """One split-K workspace serving calls of different batch sizes in turn: the arrival
    counters of a larger batch must not land on partials a smaller batch left behind."""
    from gollek_b200 import _lib, ops
    lib = _lib.load()
    big = lib.gollek_paged_attention_workspace_size(24, 32, 8, 128)
    ws = torch.zeros(big, dtype=torch.uint8, device=cuda_device) if own_workspace else None
    rng = np.random.default_rng(71)
    for S in (3, 24, 3, 17, 5, 24):
        ctx = rng.integers(3000, 9000, S).tolist()  # few long sequences: split across CTAs
        q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=S, kv_std=0.5)
        qb, kb, vb = O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)
        want = oracle_decode(qb, kb, vb, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16)
        out = ops.paged_attention(_t(qb, cuda_device, torch.bfloat16), _t(kb, cuda_device, torch.bfloat16),
                                  _t(vb, cuda_device, torch.bfloat16), _t(bt, cuda_device),
                                  _t(ctx, cuda_device), num_kv_heads=8, block_size=16,
                                  num_blocks=k.shape[0], workspace=ws)
        np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0, err_msg=f"S={S}")


def test_decode_and_append_capture_in_a_cuda_graph(cuda_device):
    """With a caller workspace, gollek_kv_append + gollek_paged_attention_v2 capture into a
    CUDA graph (no allocation or synchronisation inside) and replays match eager calls."""
    from gollek_b200 import _lib, ops
    ctx = [100, 2000, 5000]
    q, k, v, bt, ctx = decode_case(ctx, hq=32, hkv=8, d=128, bs=16, seed=81, kv_std=0.5)
    dev = cuda_device
    qd = _t(O.round_bf16(q), dev, torch.bfloat16)
    kd, vd = _t(O.round_bf16(k), dev, torch.bfloat16), _t(O.round_bf16(v), dev, torch.bfloat16)
    btd, ctxd = _t(bt, dev), _t(ctx, dev)
    new_k = torch.randn((3, 8, 128), device=dev).to(torch.bfloat16)
    new_v = torch.randn((3, 8, 128), device=dev).to(torch.bfloat16)
    pos = (ctxd - 1).to(torch.int32)
    ws = torch.zeros(_lib.load().gollek_paged_attention_workspace_size(3, 32, 8, 128), dtype=torch.uint8,
                     device=dev)
    out = torch.empty_like(qd)

    def step():
        ops.kv_append(new_k, new_v, pos, btd, kd, vd, block_size=16, num_blocks=k.shape[0])
        ops.paged_attention(qd, kd, vd, btd, ctxd, num_kv_heads=8, block_size=16, num_blocks=k.shape[0],
                            out=out, workspace=ws)

    step()
    torch.cuda.synchronize()
    eager = out.clone()
    out.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


def test_concurrent_callers_on_their_own_streams(cuda_device):
    """The binding is a process-wide singleton called from many threads: concurrent calls
    on separate streams (library-owned scratch per stream) and through the legacy
    synchronous symbol (per-thread stream) all return the oracle's results."""
    import threading

    from gollek_b200 import ops
    cases = []
    for i in range(6):
        ctx = [300 + 500 * i, 4000 + 700 * i, 33]
        q, k, v, bt, ctx = decode_case(ctx, hq=8, hkv=8, d=64, bs=16, seed=90 + i)
        want = oracle_decode(q, k, v, bt, ctx, 0.125, hkv=8, bs=16, lanes=8)
        a1 = O.a1_execute(q, k, v, bt, ctx, 0.125)
        cases.append((q, k, v, bt, ctx, want, a1))
    errors = []

    def worker(i):
        try:
            torch.cuda.set_device(cuda_device)
            q, k, v, bt, ctx, want, a1 = cases[i]
            dq, dk, dv = _t(q, cuda_device), _t(k, cuda_device), _t(v, cuda_device)
            dbt, dctx = _t(bt, cuda_device), _t(ctx, cuda_device)
            st = torch.cuda.Stream(cuda_device)
            for _ in range(5):
                with torch.cuda.stream(st):
                    out = ops.paged_attention(dq, dk, dv, dbt, dctx, num_kv_heads=8, block_size=16,
                                              scale=0.125, num_blocks=k.shape[0], stream=st)
                st.synchronize()
                _fp32_close(out.cpu().numpy(), want)
                leg = torch.empty_like(dq)
                ops.paged_attention_launch(leg, dq, dk, dv, dbt, dctx, 0.125)
                _fp32_close(leg.cpu().numpy(), a1)
        except Exception as e:  # reported below
            errors.append((i, repr(e)))

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(len(cases))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors


def _round_f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("hq,hkv,d,q_f32,qmag", [(32, 8, 128, False, 1.0), (64, 8, 128, True, 1.0),
                                                 (16, 4, 64, False, 1.0), (32, 8, 128, False, 3e5),
                                                 (32, 8, 128, True, 3e5)])
def test_f16_kv_parity(cuda_device, hq, hkv, d, q_f32, qmag):
    """f16 KV on the tensor pipe (q enters as f16 hi + lo; |q| above the f16 range is
    brought in by a power of two put back on the scores)."""
    from gollek_b200 import ops
    ctx = [1, 70, 900, 4100, 0]
    q, k, v, bt, ctx = decode_case(ctx, hq=hq, hkv=hkv, d=d, bs=16, seed=hq + d + int(qmag) % 7, kv_std=0.5)
    kh, vh = _round_f16(k), _round_f16(v)
    qq = q * np.float32(qmag)
    if not q_f32:
        qq = O.round_bf16(qq)
    scale = 1.0 / math.sqrt(d)
    want = oracle_decode(qq, kh, vh, bt, ctx, scale, hkv=hkv, bs=16)
    out = ops.paged_attention(_t(qq, cuda_device) if q_f32 else _t(qq, cuda_device, torch.bfloat16),
                              _t(kh, cuda_device, torch.float16), _t(vh, cuda_device, torch.float16),
                              _t(bt, cuda_device), _t(ctx, cuda_device), num_kv_heads=hkv, block_size=16,
                              scale=scale, num_blocks=k.shape[0])
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    assert not got[4].any()
