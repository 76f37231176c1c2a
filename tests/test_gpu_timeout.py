"""Failure detection on the device, without a GPU fault: a bounded wait that gives up.

Every wait in the decode kernels and the tensor-memory multi-query kernel is bounded; when
one gives up the kernel raises GOLLEK_STATUS_TIMEOUT, stops, lets its issued copies land and
returns, so the context stays usable.  These tests make one wait run out on purpose through
two test hooks the library reads per call: GOLLEK_TEST_WAIT_LIMIT (a short bound for the
waits) and GOLLEK_TEST_SKIP_GROUP (CTA 0's producer never issues that group's -- for the
tensor-memory kernel, that tile's -- copies, so the consumer waiting for it gives up).
Nothing faults: the missing copy is simply never made.

What is checked: the status word reports the timeout (and the synchronous legacy symbol
returns GOLLEK_ERR_TIMEOUT), and the next normal call on the same split-K workspace --
caller-owned, not re-zeroed, or library-owned -- matches the oracle, i.e. the split-K
arrival counters were left consistent by the call that gave up.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import decode_case, oracle_decode

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bf16_case():
    # few long sequences: each (sequence, kv-head) is cut into split-K pieces across CTAs,
    # and CTA 0's range starts inside such a unit
    q, k, v, bt, ctx = decode_case([8000, 7000, 6000, 9000], hq=32, hkv=8, d=128, bs=16, seed=61,
                                   kv_std=0.5)
    return O.round_bf16(q), O.round_bf16(k), O.round_bf16(v), bt, ctx


def _run(dev, q, k, v, bt, ctx, workspace):
    from gollek_b200 import ops
    T = lambda x, dt=None: (torch.from_numpy(np.ascontiguousarray(x)).to(dev) if dt is None
                            else torch.from_numpy(np.ascontiguousarray(x)).to(dev).to(dt))
    return ops.paged_attention(T(q, torch.bfloat16), T(k, torch.bfloat16), T(v, torch.bfloat16),
                               T(bt), T(ctx), num_kv_heads=8, block_size=16, num_blocks=k.shape[0],
                               scale=1.0 / math.sqrt(128), workspace=workspace)


@pytest.mark.parametrize("own_workspace", [True, False])
def test_decode_wait_gives_up_then_next_call_is_correct(cuda_device, monkeypatch, own_workspace):
    from gollek_b200 import _lib, ops
    monkeypatch.setenv("GOLLEK_DECODE_PATH", "mma")  # the TMA kernel with the bounded waits
    q, k, v, bt, ctx = _bf16_case()
    want = oracle_decode(q, k, v, bt, ctx, 1 / math.sqrt(128), hkv=8, bs=16)
    ws = ops.new_workspace(4, 32, 8, 128, cuda_device) if own_workspace else None
    ops.device_status(cuda_device.index, clear=True)

    monkeypatch.setenv("GOLLEK_TEST_WAIT_LIMIT", "20000")
    monkeypatch.setenv("GOLLEK_TEST_SKIP_GROUP", "0")
    _run(cuda_device, q, k, v, bt, ctx, ws)
    torch.cuda.synchronize()
    st = ops.device_status(cuda_device.index, clear=True)
    assert st & _lib.STATUS_TIMEOUT, st

    monkeypatch.delenv("GOLLEK_TEST_WAIT_LIMIT")
    monkeypatch.delenv("GOLLEK_TEST_SKIP_GROUP")
    for _ in range(2):  # the same workspace, not re-zeroed by the caller
        out = _run(cuda_device, q, k, v, bt, ctx, ws)
        torch.cuda.synchronize()
        assert ops.device_status(cuda_device.index, clear=True) == 0
        np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)


def test_legacy_symbol_reports_the_timeout(cuda_device, monkeypatch):
    """paged_attention_launch waits for its stream and turns the status into its return
    code: GOLLEK_ERR_TIMEOUT after a wait gave up, 0 and correct results on the next call."""
    from gollek_b200 import _lib, ops
    rng = np.random.default_rng(62)
    ctx = np.array([3000, 2500, 4000, 1000], np.int32)
    H, D, BS = 8, 64, 16
    q, k, v, bt, ctx = decode_case(ctx, hq=H, hkv=H, d=D, bs=BS, seed=62)
    dev = cuda_device
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    out = torch.empty((4, H, D), dtype=torch.float32, device=dev)
    ops.device_status(dev.index, clear=True)
    monkeypatch.setenv("GOLLEK_TEST_WAIT_LIMIT", "20000")
    monkeypatch.setenv("GOLLEK_TEST_SKIP_GROUP", "0")
    with pytest.raises(_lib.GollekError) as e:
        ops.paged_attention_launch(out, T(q), T(k), T(v), T(bt), T(ctx), 0.125)
    assert e.value.code == _lib.ERR_TIMEOUT
    monkeypatch.delenv("GOLLEK_TEST_WAIT_LIMIT")
    monkeypatch.delenv("GOLLEK_TEST_SKIP_GROUP")
    ops.paged_attention_launch(out, T(q), T(k), T(v), T(bt), T(ctx), 0.125)
    want = O.a1_execute(q, k, v, bt, ctx, 0.125)
    err = np.abs(out.cpu().numpy() - want).max()
    assert err <= 1e-4 * max(1.0, float(np.abs(want).max()))


def test_tcgen05_multi_query_wait_gives_up_then_next_call_is_correct(cuda_device, monkeypatch):
    """The tensor-memory multi-query kernel (64 folded rows: 16 queries x GQA 4): CTA 0's
    producers never issue its first tile, so its score-MMA issuer's bounded wait gives up;
    the kernel raises GOLLEK_STATUS_TIMEOUT, every warp of that CTA leaves, and the next
    calls on the library's workspace (re-zeroed when the timeout is reported) match the
    oracle."""
    from gollek_b200 import _lib, ops
    tq, hq, hkv = 16, 32, 8
    q1, k, v, bt, ctx = decode_case([8000, 7000, 6000, 9000], hq=hq, hkv=hkv, d=128, bs=16, seed=63,
                                    kv_std=0.5)
    rng = np.random.default_rng(64)
    q = O.round_bf16(rng.standard_normal((len(ctx), tq, hq, 128)).astype(np.float32))
    kb, vb = O.round_bf16(k), O.round_bf16(v)
    scale = 1.0 / math.sqrt(128)
    want = O.a2_compute(q, kb, vb, bt, ctx, scale, num_kv_heads=hkv, block_size=16, causal=1,
                        threads=O.num_threads())
    dev = cuda_device
    T = lambda x, dt=None: (torch.from_numpy(np.ascontiguousarray(x)).to(dev) if dt is None
                            else torch.from_numpy(np.ascontiguousarray(x)).to(dev).to(dt))

    def run():
        return ops.paged_attention_prefill(T(q, torch.bfloat16), T(kb, torch.bfloat16), T(vb, torch.bfloat16),
                                           T(bt), T(ctx), num_kv_heads=hkv, block_size=16, scale=scale,
                                           causal=True, num_blocks=k.shape[0])

    ops.device_status(dev.index, clear=True)
    monkeypatch.setenv("GOLLEK_TEST_WAIT_LIMIT", "20000")
    monkeypatch.setenv("GOLLEK_TEST_SKIP_GROUP", "0")
    run()
    torch.cuda.synchronize()
    st = ops.device_status(dev.index, clear=True)
    assert st & _lib.STATUS_TIMEOUT, st

    monkeypatch.delenv("GOLLEK_TEST_WAIT_LIMIT")
    monkeypatch.delenv("GOLLEK_TEST_SKIP_GROUP")
    for _ in range(2):
        out = run()
        torch.cuda.synchronize()
        assert ops.device_status(dev.index, clear=True) == 0
        np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=0)
