"""gollek_paged_attention_v2_noalloc: decode attention for callers that cannot allocate.

Some hosts of this library cannot call cudaMalloc or pass a workspace: code running while
another component captures a CUDA graph, real-time hosts that forbid allocation after
start-up, and JVM/FFM hosts whose allocators know nothing of device memory.  The no-alloc
entry point serves them from a static device array built into the library.  This test
calls it through the C ABI twice in a row and checks each result against the ordinary
entry point, gollek_paged_attention_v2: both run the same kernel over the same split of the
work, so the outputs must be identical bit for bit.  Each result is also checked against
the CPU oracle (the reference's PagedAttentionVectorAPI restated) within the bf16 tolerance
the other decode tests use (2e-2 absolute).  An oversized request must be refused without
a launch.

The file name sorts last so that a run stopping at the first failure has run every other
test first.
"""
import ctypes
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import decode_case

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _call(fn, out, q, k, v, bt, ctx, num_blocks, *extra):
    from gollek_b200 import _lib
    return fn(out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), None, None, bt.data_ptr(),
              ctx.data_ptr(), q.shape[0], q.shape[1], 8, q.shape[2], 16, bt.shape[1], num_blocks, 0,
              _lib.BF16, _lib.BF16, 0, 0, 0, 1.0 / math.sqrt(q.shape[2]), 0.0, 0, *extra)


def test_no_alloc_matches_v2_twice(cuda_device):
    from gollek_b200 import _lib
    lib = _lib.load()
    # long contexts so that (sequence, kv-head) pairs split across CTAs and the split-K
    # scratch is really used
    qn, kn, vn, btn, ctxn = decode_case([7000, 3000, 500, 8192], hq=32, hkv=8, d=128, bs=16,
                                        seed=77, kv_std=0.5)
    dev = cuda_device
    q = torch.from_numpy(O.round_bf16(qn)).to(dev).to(torch.bfloat16)
    k = torch.from_numpy(O.round_bf16(kn)).to(dev).to(torch.bfloat16)
    v = torch.from_numpy(O.round_bf16(vn)).to(dev).to(torch.bfloat16)
    bt = torch.from_numpy(btn).to(dev)
    ctx = torch.from_numpy(ctxn).to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    ref = torch.empty_like(q)
    ws = torch.zeros(lib.gollek_paged_attention_workspace_size(4, 32, 8, 128), dtype=torch.uint8,
                     device=dev)
    rc = _call(lib.gollek_paged_attention_v2, ref, q, k, v, bt, ctx, kn.shape[0], ws.data_ptr(),
               ws.numel(), stream)
    assert rc == 0, lib.gollek_last_error_string()

    torch.cuda.synchronize()
    want = O.a2_compute(O.round_bf16(qn)[:, None], O.round_bf16(kn), O.round_bf16(vn), btn, ctxn,
                        1.0 / math.sqrt(128), num_kv_heads=8, block_size=16,
                        threads=O.num_threads())[:, 0]

    for _ in range(2):  # the scratch keeps the last call's contents; two calls in a row
        out = torch.full_like(q, float("nan"))
        rc = _call(lib.gollek_paged_attention_v2_noalloc, out, q, k, v, bt, ctx, kn.shape[0], stream)
        assert rc == 0, lib.gollek_last_error_string()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)  # same kernel, same partition: identical bits
        diff = np.abs(out.float().cpu().numpy() - want).max()
        assert diff <= 2e-2, diff


def test_no_alloc_refuses_oversized_requests(cuda_device):
    from gollek_b200 import _lib
    lib = _lib.load()
    need = lib.gollek_paged_attention_workspace_size(4096, 32, 8, 128)
    assert need > (32 << 20)
    d = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    rc = lib.gollek_paged_attention_v2_noalloc(d, d, d, d, None, None, d, d, 4096, 32, 8, 128, 16,
                                               64, 0, 0, _lib.BF16, _lib.BF16, 0, 0, 0, 0.1, 0.0, 0,
                                               None)
    assert rc == _lib.ERR_WORKSPACE
    assert b"static buffer" in lib.gollek_last_error_string()
