"""pa_b200 -- B200 (sm_100a) paged attention, a drop-in for gb10-attn's kernels.

Submodules:
  ops      the reference's operator API (paged_attention, _v2, _v3,
           choose_num_splits, paged_attention_prefill, _prefill_wmma) over the
           in-tree torch shim and libpa_b200.so
  kv       KV pool: KVConfig, ModelConfig, TorchBlockAllocator, LayeredPool
  harness  peak-bandwidth provenance, cold pools, traffic models
  dist     batch- and sequence-sharded multi-GPU decode
  _lib     ctypes binding of the C ABI (include/pa_b200.h)
"""
__all__ = ["ops", "kv", "harness", "dist"]
__version__ = "0.1.0"
