"""The committed golden fixtures (tests/golden/golden.npz, made by tests/golden/make_golden.py).

CPU: the generator still produces the recorded inputs and the oracle still produces the
recorded outputs (bit for bit).  GPU: the CUDA paths against the recorded outputs, at the
tolerances of the other parity tests.
"""
import hashlib
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden import make_golden as G

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(os.path.join(HERE, "golden.npz")))


def test_fixture_inputs_regenerate(gold):
    c = G.case_config1()
    assert G.digest(c["q"], c["k"], c["v"], c["bt"], c["ctx"]) == str(gold["config1_in"])
    c = G.case_gqa_bf16()
    assert G.digest(c["q"], c["k"], c["v"], c["bt"], c["ctx"]) == str(gold["gqa_bf16_in"])
    c = G.case_append()
    assert G.digest(c["key"], c["val"], c["pos"], c["seq"], c["bt"]) == str(gold["append_in"])
    c = G.case_migrate()
    assert G.digest(c["pool_k"], c["pool_v"], c["src"], c["dst"]) == str(gold["migrate_in"])


def test_oracle_reproduces_fixtures(gold):
    res = G.outputs()
    for key in ("config1_out", "gqa_bf16_out", "int8_kv_out", "append_k", "append_v", "append_ks",
                "append_vs"):
        assert np.array_equal(res[key], gold[key]), key
    assert res["migrate_out"] == str(gold["migrate_out"])
    assert res["int8_kv_in"] == str(gold["int8_kv_in"])


# ------------------------------------------------------------------------- GPU

@pytest.mark.gpu
def test_gpu_against_fixtures(gold, cuda_device):
    import torch

    from gollek_b200 import ops
    T = lambda x, dt=None: (torch.from_numpy(np.ascontiguousarray(x)).to(cuda_device) if dt is None
                            else torch.from_numpy(np.ascontiguousarray(x)).to(cuda_device).to(dt))
    # config 1 through the legacy symbol
    c = G.case_config1()
    out = torch.empty((4, 8, 64), device=cuda_device)
    ops.paged_attention_launch(out, T(c["q"]), T(c["k"]), T(c["v"]), T(c["bt"]), T(c["ctx"]),
                               float(c["scale"]))
    want = gold["config1_out"]
    assert np.abs(out.cpu().numpy() - want).max() <= 1e-4 * np.abs(want).max()
    # bf16 GQA
    c = G.case_gqa_bf16()
    out = ops.paged_attention(T(c["q"], torch.bfloat16), T(c["k"], torch.bfloat16),
                              T(c["v"], torch.bfloat16), T(c["bt"]), T(c["ctx"]), num_kv_heads=8,
                              block_size=16, scale=float(c["scale"]), num_blocks=c["k"].shape[0])
    assert np.abs(out.float().cpu().numpy() - gold["gqa_bf16_out"]).max() <= 2e-2
    # int8 KV with the reference's per-token scales
    c = G.case_int8()
    out = ops.paged_attention(T(c["q"], torch.bfloat16), T(c["kq"]), T(c["vq"]), T(c["bt"]),
                              T(c["ctx"]), num_kv_heads=8, block_size=16, scale=float(c["scale"]),
                              num_blocks=c["kq"].shape[0], k_scales=T(c["ks"]), v_scales=T(c["vs"]),
                              scale_strides=(8 * 16, 16, 1))
    assert np.abs(out.float().cpu().numpy() - gold["int8_kv_out"]).max() <= 2e-2
    # append: bytes and scales bit-exact
    c = G.case_append()
    kb = torch.zeros((8, 4, 16, 64), dtype=torch.int8, device=cuda_device)
    vb = torch.zeros_like(kb)
    ks = torch.zeros((8, 4, 16), device=cuda_device)
    vs = torch.zeros_like(ks)
    ops.kv_append(T(c["key"]), T(c["val"]), T(c["pos"]), T(c["bt"]), kb, vb, block_size=16,
                  num_blocks=8, token_seq=T(c["seq"]), k_scales=ks, v_scales=vs,
                  scale_strides=(4 * 16, 16, 1))
    assert np.array_equal(kb.cpu().numpy().reshape(-1), gold["append_k"])
    assert np.array_equal(vb.cpu().numpy().reshape(-1), gold["append_v"])
    assert np.array_equal(ks.cpu().numpy().reshape(-1), gold["append_ks"])
    assert np.array_equal(vs.cpu().numpy().reshape(-1), gold["append_vs"])
    # migration: the decode pool's digest
    c = G.case_migrate()
    pk, pv = T(c["pool_k"]), T(c["pool_v"])
    blk = c["L"] * c["bpb"]
    ops.kv_migrate(pk, pv, pk, pv, T(c["src"]), T(c["dst"]), src_block_stride=blk,
                   dst_block_stride=blk, bytes_per_block=blk)
    torch.cuda.synchronize()
    assert G.digest(pk.cpu().numpy(), pv.cpu().numpy()) == str(gold["migrate_out"])
