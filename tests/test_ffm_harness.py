"""The library called as Gollek's Java FFM binding calls it (tests/ffm/ffm_harness.c).

The harness resolves each entry point by name and calls it through a function-pointer type
built only from the FFM descriptors' value layouts (JAVA_INT / JAVA_LONG / JAVA_FLOAT /
ADDRESS), in the descriptors' order -- PagedAttentionBinding.java:200-227 for the symbols
the reference already binds, the integration guide's descriptors for the new ones -- so a
descriptor that disagrees with the library's signature fails here.  Without a GPU it runs
the host-side argument checks; on a GPU it runs the legacy symbol, the engine entry point,
the append and the migration on device buffers, and the outputs are checked against the
oracle (1e-4 relative for fp32 attention, bit for bit for the appended and migrated bytes).
"""
import math
import os
import subprocess

import numpy as np
import pytest

from gollek_b200.build import LIB_PATH

HERE = os.path.dirname(os.path.abspath(__file__))
CUDA = "/usr/local/cuda"


def _build(tmp_path):
    exe = str(tmp_path / "ffm_harness")
    cmd = ["gcc", "-O1", "-std=c11", "-o", exe, os.path.join(HERE, "ffm", "ffm_harness.c"),
           f"-I{CUDA}/include", f"-L{CUDA}/lib64", "-lcudart", "-ldl", f"-Wl,-rpath,{CUDA}/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def _lib():
    from gollek_b200 import _lib
    _lib.load()  # builds the library if its sources changed
    return LIB_PATH


def test_ffm_descriptors_bind_and_validate(tmp_path):
    """Every descriptor resolves and the host-side checks answer as the header says."""
    exe = _build(tmp_path)
    r = subprocess.run([exe, "abi", _lib()], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "abi ok=1" in r.stdout


@pytest.mark.gpu
def test_ffm_calls_on_device_match_oracle(tmp_path, cuda_device):
    from oracle import oracle as O
    exe = _build(tmp_path)
    out = str(tmp_path / "ffm.bin")
    r = subprocess.run([exe, "gpu", _lib(), out], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    S, H, D, BS, NB, MAXB = 4, 8, 64, 16, 256, 32
    raw = np.fromfile(out, dtype=np.uint8)
    sizes = [("q", S * H * D, np.float32), ("k", NB * H * BS * D, np.float32),
             ("v", NB * H * BS * D, np.float32), ("bt", S * MAXB, np.int32), ("ctx", S, np.int32),
             ("out_legacy", S * H * D, np.float32), ("out_v2", S * H * D, np.float32),
             ("key", S * H * D, np.float32), ("val", S * H * D, np.float32),
             ("k_after", NB * H * BS * D, np.float32), ("v_after", NB * H * BS * D, np.float32)]
    arr, off = {}, 0
    for name, n, dt in sizes:
        nbytes = n * np.dtype(dt).itemsize
        arr[name] = raw[off:off + nbytes].view(dt)
        off += nbytes
    assert off == raw.size
    q = arr["q"].reshape(S, H, D)
    k = arr["k"].reshape(NB, H, BS, D).copy()
    v = arr["v"].reshape(NB, H, BS, D).copy()
    bt = arr["bt"].reshape(S, MAXB)
    ctx = arr["ctx"]

    want = O.a1_execute(q, k, v, bt, ctx, 0.125)
    scale_ref = max(float(np.abs(want).max()), 1e-6)
    assert np.abs(arr["out_legacy"].reshape(S, H, D) - want).max() <= 1e-4 * scale_ref
    want2 = O.a2_compute(q, k, v, bt, ctx, 0.125, num_kv_heads=H, block_size=BS)[:, 0]
    assert np.abs(arr["out_v2"].reshape(S, H, D) - want2).max() <= 1e-4 * scale_ref

    # each sequence's last token rewritten (position ctx - 1), then three pages migrated
    kf, vf = k.reshape(-1).copy(), v.reshape(-1).copy()
    rc = O.update_cache(arr["key"].reshape(S, H, D), arr["val"].reshape(S, H, D), ctx - 1, bt,
                        storage=O.FP32, k_slab=kf, v_slab=vf, block_size=BS)
    assert rc == 0
    src = np.array([bt[0, 0], bt[1, 1], bt[3, 2]], np.int32)
    dst = np.array([250, 251, 252], np.int32)
    page = H * BS * D * 4
    kb, vb = kf.view(np.uint8), vf.view(np.uint8)
    O.migrate(kb, vb, kb, vb, src, dst, 1, page)
    assert np.array_equal(arr["k_after"].view(np.uint32), kf.view(np.uint32))
    assert np.array_equal(arr["v_after"].view(np.uint32), vf.view(np.uint32))
