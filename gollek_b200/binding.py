"""PagedAttentionBinding -- the Python mirror of Gollek's FFM binding.

Mirrors optimization/gollek-plugin-paged-attention/src/main/java/tech/kayys/gollek/kernel/paged/
PagedAttentionBinding.java (initialize :69-86, initializeFallback :91-95, getInstance :103-109,
isNativeAvailable :114-116, pagedAttentionLaunch :140-177, getCudaDeviceCount :184-196,
reset :245-247) over libgollek_kernels.so.

One deliberate difference: the reference falls back to a Java CPU loop when the native
library is missing.  This build has no CPU path, so a launch on an instance without
the native library raises instead of computing on the host.
"""
from __future__ import annotations

import logging
import threading

from . import _lib

LOG = logging.getLogger("gollek_b200.binding")

FN_PAGED_ATTENTION = "paged_attention_launch"
FN_CUDA_DEVICE_COUNT = "gollek_cuda_device_count"
FN_CUDA_DEVICE_NAME = "gollek_cuda_device_name"


def _addr(x) -> int | None:
    """A device address from an int or a torch tensor."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


class PagedAttentionBinding:
    _instance: "PagedAttentionBinding | None" = None
    _lock = threading.Lock()

    def __init__(self, lib):
        self._lib = lib
        self._native = lib is not None
        self._bound = {}
        if self._native:
            for name in (FN_PAGED_ATTENTION, FN_CUDA_DEVICE_COUNT, FN_CUDA_DEVICE_NAME):
                fn = getattr(lib, name, None)
                if fn is None:
                    LOG.warning("Native symbol not found: %s (some features may be unavailable)", name)
                else:
                    self._bound[name] = fn

    # ---- initialization -------------------------------------------------------
    @classmethod
    def initialize(cls, library_path: str | None = None) -> bool:
        """Load libgollek_kernels.so (the in-tree build when no path is given)."""
        with cls._lock:
            if cls._instance is not None:
                LOG.warning("PagedAttentionBinding already initialized")
                return cls._instance._native
            try:
                lib = _lib.load(library_path, build_if_missing=library_path is None)
                cls._instance = cls(lib)
                LOG.info("PagedAttention native binding loaded from %s", library_path or _lib.LIB_PATH)
                return True
            except OSError as e:
                LOG.warning("Failed to load PagedAttention native library from %s: %s",
                            library_path, e)
                cls._instance = cls(None)
                return False

    @classmethod
    def initialize_fallback(cls) -> None:
        """An instance without the native library (launches raise: no CPU path)."""
        with cls._lock:
            if cls._instance is None:
                cls._instance = cls(None)

    @classmethod
    def get_instance(cls) -> "PagedAttentionBinding":
        if cls._instance is None:
            raise RuntimeError("PagedAttentionBinding not initialized. Call initialize() first.")
        return cls._instance

    @classmethod
    def reset(cls) -> None:
        with cls._lock:
            cls._instance = None

    def is_native_available(self) -> bool:
        return self._native

    # ---- kernel invocation ----------------------------------------------------
    def paged_attention_launch(self, output, query, key_cache, value_cache, block_tables,
                               context_lens, num_seqs: int, num_heads: int, head_dim: int,
                               block_size: int, max_blocks_per_seq: int, scale: float) -> int:
        """Device pointers (ints or CUDA tensors) in; returns 0 or an error code."""
        if not self._native:
            raise RuntimeError("paged_attention_launch: native library not loaded "
                               "(this build has no CPU fallback)")
        fn = self._bound.get(FN_PAGED_ATTENTION)
        if fn is None:
            raise RuntimeError("paged_attention_launch not bound")
        return int(fn(_addr(output), _addr(query), _addr(key_cache), _addr(value_cache),
                      _addr(block_tables), _addr(context_lens), int(num_seqs), int(num_heads),
                      int(head_dim), int(block_size), int(max_blocks_per_seq), float(scale)))

    def get_cuda_device_count(self) -> int:
        if not self._native:
            return 0
        fn = self._bound.get(FN_CUDA_DEVICE_COUNT)
        if fn is None:
            return 0
        try:
            return int(fn())
        except Exception as e:  # mirrors the Java warn-and-return-0
            LOG.warning("Failed to query CUDA device count: %s", e)
            return 0

    def get_cuda_device_name(self) -> str:
        if not self._native or FN_CUDA_DEVICE_NAME not in self._bound:
            return ""
        import ctypes
        buf = ctypes.create_string_buffer(256)
        rc = self._bound[FN_CUDA_DEVICE_NAME](buf, 256)
        return buf.value.decode() if rc == 0 else ""
