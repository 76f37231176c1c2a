"""Seeded random sweep of the decode / multi-query entry points against the oracle.

Each case draws: KV dtype (fp32, bf16, int8 with per-token or per-page scales), q dtype,
kv heads and GQA group, head_dim, block size, batch, context lengths (some empty, some
longer than a CTA's share so split-K runs), sliding window, soft-cap and query count.
Tolerances as everywhere: fp32 KV and q <= 1e-4 relative to the output scale; otherwise
<= 2e-2 absolute against the fp32 oracle on the same rounded inputs.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import decode_case, quantize_pages_int8, quantize_rows_int8

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _t(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dtype is None else t.to(dtype)


def _draw(seed):
    r = np.random.default_rng(seed)
    kv = r.choice(["f32", "bf16", "bf16", "i8tok", "i8page"])
    q_f32 = bool(r.integers(0, 2)) or kv == "f32"
    hkv = int(r.choice([1, 2, 4, 8]))
    g = int(r.choice([1, 2, 4, 8]))
    d = 128 if kv.startswith("i8") else int(r.choice([64, 128]))
    bs = int(r.choice([8, 16, 32]))
    S = int(r.integers(1, 24))
    ctx = r.integers(0, 3000, S)
    ctx[r.random(S) < 0.15] = 0
    if S > 2:
        ctx[0] = int(r.integers(6000, 12000))  # long enough to split across CTAs
    window = int(r.choice([0, 0, 0, int(r.integers(1, 700))]))
    cap = float(r.choice([0.0, 0.0, 25.0]))
    tq = int(r.choice([1, 1, 1, 2, 4]))
    return dict(kv=kv, q_f32=q_f32, hkv=hkv, g=g, d=d, bs=bs, ctx=ctx.astype(np.int32), window=window,
                cap=cap, tq=tq)


@pytest.mark.parametrize("seed", range(24))
def test_random_case_matches_oracle(cuda_device, seed):
    from gollek_b200 import ops
    c = _draw(1000 + seed)
    hq = c["hkv"] * c["g"]
    q, k, v, bt, ctx = decode_case(c["ctx"], hq=hq, hkv=c["hkv"], d=c["d"], bs=c["bs"], seed=seed,
                                   kv_std=0.5)
    tq = c["tq"]
    rng = np.random.default_rng(seed + 7)
    qm = rng.standard_normal((len(ctx), tq, hq, c["d"])).astype(np.float32)
    if not c["q_f32"]:
        qm = O.round_bf16(qm)
    scale = 1 / math.sqrt(c["d"])
    kw = {}
    if c["kv"] == "f32":
        kd, vd, storage, ks_o, vs_o = k, v, O.FP32, None, None
    elif c["kv"] == "bf16":
        kd, vd = O.round_bf16(k), O.round_bf16(v)
        storage, ks_o, vs_o = O.FP32, None, None
    elif c["kv"] == "i8tok":
        kd, ks = quantize_rows_int8(k)
        vd, vs = quantize_rows_int8(v)
        storage, ks_o, vs_o = O.INT8, ks, vs
        kw = dict(k_scales=_t(ks, cuda_device), v_scales=_t(vs, cuda_device),
                  scale_strides=(c["hkv"] * c["bs"], c["bs"], 1))
    else:
        kd, ks = quantize_pages_int8(O.round_bf16(k))
        vd, vs = quantize_pages_int8(O.round_bf16(v))
        storage = O.INT8
        ks_o = np.repeat(ks[:, :, None], c["bs"], axis=2)
        vs_o = np.repeat(vs[:, :, None], c["bs"], axis=2)
        kw = dict(k_scales=_t(ks, cuda_device), v_scales=_t(vs, cuda_device),
                  scale_strides=(c["hkv"], 1, 0))
    want = O.a2_compute(qm, kd, vd, bt, ctx, scale, storage=storage, num_kv_heads=c["hkv"],
                        block_size=c["bs"], k_scale=ks_o, v_scale=vs_o, causal=1,
                        soft_cap=c["cap"], sliding_window=c["window"], threads=O.num_threads())
    qdt = None if c["q_f32"] else torch.bfloat16
    kv_t = (lambda x: _t(x, cuda_device)) if c["kv"] != "bf16" else (lambda x: _t(x, cuda_device, torch.bfloat16))
    common = dict(num_kv_heads=c["hkv"], block_size=c["bs"], scale=scale, num_blocks=k.shape[0],
                  soft_cap=c["cap"], sliding_window=c["window"], **kw)
    if tq == 1:
        out = ops.paged_attention(_t(qm[:, 0], cuda_device, qdt), kv_t(kd), kv_t(vd), _t(bt, cuda_device),
                                  _t(ctx, cuda_device), **common)
        got = out.float().cpu().numpy()[:, None]
    else:
        out = ops.paged_attention_prefill(_t(qm, cuda_device, qdt), kv_t(kd), kv_t(vd), _t(bt, cuda_device),
                                          _t(ctx, cuda_device), causal=True, **common)
        got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), c
    if c["kv"] == "f32" and c["q_f32"]:
        err = np.abs(got - want).max()
        assert err <= 1e-4 * max(np.abs(want).max(), 1e-6), (c, err)
    else:
        np.testing.assert_allclose(got, want, atol=2e-2, rtol=0, err_msg=str(c))
    assert ops.device_status(cuda_device.index or 0) == 0
