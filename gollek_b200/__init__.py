"""gollek_b200 -- B200-native (sm_100a) paged-KV attention hot path for Gollek.

The product is libgollek_kernels.so (C ABI in include/gollek_kernels.h).  This package
builds it in-tree, loads it (gollek_b200._lib), wraps it for torch tensors
(gollek_b200.ops) and mirrors the reference's Java host classes on top of it:
  binding.PagedAttentionBinding      <- kernel/paged/PagedAttentionBinding.java
  kv_cache.PagedKVCacheManager, ...  <- kvcache/PagedKVCacheManager.java, PhysicalBlockPool.java
  prefill_decode.PrefillDecodeDisaggService <- prefilldecode/PrefillDecodeDisaggService.java
  engine.BlockManager / KVCacheSession / paged_attention_compute
                                     <- safetensor engine generation/kv, generation/attention
"""
__version__ = "0.1.0"
