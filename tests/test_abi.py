"""The C ABI: the library loads, exports every symbol the header declares, and rejects
bad arguments with status codes before touching a device (runs without a GPU)."""
import ctypes
import os
import re

import pytest

from gollek_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gollek_kernels.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*GOLLEK_API\s+(?:const\s+char\s*\*|int|size_t)\s*(\w+)\s*\(", text,
                      flags=re.M)


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_header_declares_the_reference_symbols():
    syms = header_symbols()
    # PagedAttentionBinding.java:48-50 binds exactly these three names
    for name in ("paged_attention_launch", "gollek_cuda_device_count", "gollek_cuda_device_name"):
        assert name in syms
    assert len(syms) == len(set(syms))


def test_library_exports_every_header_symbol(lib):
    syms = header_symbols()
    assert set(syms) == set(_lib.SIGNATURES), "ctypes table out of sync with the header"
    for name in syms:
        assert hasattr(lib, name), f"missing export {name}"


def test_library_exports_nothing_else_public():
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(header_symbols()) <= exported
    ours = {s for s in exported if s.startswith(("gollek_", "paged_attention"))}
    assert ours == set(header_symbols())


def test_version_and_error_string(lib):
    assert lib.gollek_version().startswith(b"gollek-b200")
    assert lib.gollek_last_error_string() == b""


def test_invalid_arguments_rejected_without_a_device(lib):
    rc = lib.gollek_paged_attention_v2(None, None, None, None, None, None, None, None, 1, 8, 8, 64,
                                       16, 4, 0, 0, 0, 0, 0, 0, 0, 1.0, 0.0, 0, None, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    assert b"null" in lib.gollek_last_error_string()
    dummy = ctypes.c_void_p(16)
    rc = lib.gollek_paged_attention_v2(dummy, dummy, dummy, dummy, None, None, dummy, dummy, 1, 6,
                                       4, 64, 16, 4, 0, 0, 0, 0, 0, 0, 0, 1.0, 0.0, 0, None, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT  # 6 q heads over 4 kv heads
    rc = lib.gollek_paged_attention_v2(dummy, dummy, dummy, dummy, None, None, dummy, dummy, 1, 8,
                                       8, 64, 16, 4, 0, 0, 0, _lib.I8, 0, 0, 0, 1.0, 0.0, 0, None, 0,
                                       None)
    assert rc == _lib.ERR_INVALID_ARGUMENT  # int8 without scales
    rc = lib.gollek_kv_append(dummy, dummy, _lib.F32, None, dummy, dummy, 4, 0, dummy, dummy, None,
                              None, _lib.I4, 1, 1, 63, 16, 0, 0, 0, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED  # odd head_dim for int4
    rc = lib.gollek_kv_migrate(dummy, None, dummy, dummy, dummy, dummy, 1, 0, 0, 16, 16, 16, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT  # src_v NULL but dst_v set
    rc = lib.gollek_kv_migrate(dummy, dummy, dummy, dummy, dummy, dummy, 1, 4, 4, 16, 16, 32, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT  # a bounded pool's blocks would overlap
    rc = lib.gollek_kv_migrate(dummy, dummy, dummy, dummy, dummy, dummy, 1, -1, 4, 16, 16, 16, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT  # negative pool size
    rc = lib.gollek_kv_append(dummy, dummy, _lib.F32, None, dummy, dummy, 4, 0, dummy, dummy, dummy,
                              dummy, _lib.I8, 1, 1, 64, 16, 0, 8, 1, 0, None)
    assert rc == _lib.ERR_UNSUPPORTED  # int8 append into per-(page, head) scales


def test_prefill_arguments_rejected_without_a_device(lib):
    d = ctypes.c_void_p(16)
    args = lambda tq, window, causal: (d, d, d, d, None, None, d, d, 2, tq, 8, 8, 128, 16, 4, 0, 0,
                                       _lib.F32, _lib.F32, 0, 0, 0, 0.1, 0.0, window, causal, None,
                                       0, None)
    assert lib.gollek_paged_attention_prefill(*args(0, 0, 1)) == _lib.ERR_INVALID_ARGUMENT
    assert lib.gollek_paged_attention_prefill(*args(4, 32, 0)) == _lib.ERR_UNSUPPORTED
    assert b"causal" in lib.gollek_last_error_string()
    n = lib.gollek_paged_attention_prefill_workspace_size(4, 8, 32, 8, 128)
    assert n >= lib.gollek_paged_attention_workspace_size(32, 32, 8, 128) + 32 * 4
    assert lib.gollek_paged_attention_prefill_workspace_size(4, 0, 32, 8, 128) == 0


def test_workspace_size_is_host_arithmetic(lib):
    n = lib.gollek_paged_attention_workspace_size(64, 32, 8, 128)
    slot = (2 * 4 + 4 * 128) * 4
    assert n >= 64 * 8 * 64 * slot
    assert lib.gollek_paged_attention_workspace_size(64, 30, 8, 128) == 0


@pytest.mark.skipif(_lib.load().gollek_cuda_device_count() > 0, reason="a GPU is present")
def test_no_device_behaviour(lib):
    """Like PagedAttentionCpuFallbackTest.bindingFallback: no device -> count 0, and the
    legacy call reports no device instead of computing on the CPU."""
    assert lib.gollek_cuda_device_count() == 0
    buf = ctypes.create_string_buffer(64)
    assert lib.gollek_cuda_device_name(buf, 64) == _lib.ERR_NO_DEVICE
    d = ctypes.c_void_p(16)
    assert lib.paged_attention_launch(d, d, d, d, d, d, 1, 1, 2, 4, 1, 1.0) == _lib.ERR_NO_DEVICE
