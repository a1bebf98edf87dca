"""The reference's operator API, B200 implementation.

gb10-attn's kernels are used as torch extension functions (built by
hetero-serve with ``torch.utils.cpp_extension.load_inline``; declarations in
``kernels/paged_attn_v1.h:13-15``, ``paged_attn_v2.h:13-15``,
``paged_attn_v3.h:13-17``, ``paged_attn_prefill.h:13-15``,
``paged_attn_wmma.h:13-15``).  This module exposes the same functions with the
same signatures from the in-tree C++ shim (``csrc/torch_shim.cpp``) over
``libpa_b200.so``::

    paged_attention(q, k_cache, v_cache, block_tables, context_lens, scale)
    paged_attention_v2(q, k_cache, v_cache, block_tables, context_lens, scale)
    paged_attention_v3(q, k_cache, v_cache, block_tables, context_lens, scale, num_splits)
    choose_num_splits(num_seqs, num_heads, max_context)
    paged_attention_prefill(q, k_cache, v_cache, block_tables, context_lens, scale)
    paged_attention_prefill_wmma(q, k_cache, v_cache, block_tables, context_lens, scale)

plus ``paged_attention_v3_lse``, ``paged_attention_prefill_simt``,
``write_kv``, ``validate_block_tables`` and ``merge_states``.  Importing this
module fails loudly when the extension has not been built.
"""
from __future__ import annotations

import importlib
from pathlib import Path

import torch  # noqa: F401  (loads libtorch before the extension)

_SHIM = Path(__file__).resolve().parent / "_pa_b200_torch.so"
if not _SHIM.exists():
    raise ImportError(f"{_SHIM} is missing: build it with `python gb10-attn_b200/build.py` "
                      "(or __graft_entry__.build()); there is no fallback implementation")
_ext = importlib.import_module(__package__ + "._pa_b200_torch")

paged_attention = _ext.paged_attention
paged_attention_v2 = _ext.paged_attention_v2
paged_attention_v3 = _ext.paged_attention_v3
paged_attention_v3_lse = _ext.paged_attention_v3_lse
choose_num_splits = _ext.choose_num_splits
paged_attention_prefill = _ext.paged_attention_prefill
paged_attention_prefill_wmma = _ext.paged_attention_prefill_wmma
paged_attention_prefill_simt = _ext.paged_attention_prefill_simt
write_kv = _ext.write_kv
validate_block_tables = _ext.validate_block_tables
merge_states = _ext.merge_states
paged_attention_v3_fp8 = _ext.paged_attention_v3_fp8
write_kv_scaled = _ext.write_kv_scaled
append_kv = _ext.append_kv
write_kv_batch = _ext.write_kv_batch
decode_layer_step = _ext.decode_layer_step

__all__ = ["paged_attention", "paged_attention_v2", "paged_attention_v3",
           "paged_attention_v3_lse", "choose_num_splits", "paged_attention_prefill",
           "paged_attention_prefill_wmma", "paged_attention_prefill_simt", "write_kv",
           "validate_block_tables", "merge_states", "paged_attention_v3_fp8",
           "write_kv_scaled", "append_kv", "write_kv_batch", "decode_layer_step", "shim_path"]


def shim_path() -> Path:
    return _SHIM
