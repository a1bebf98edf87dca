"""Causal chunked prefill on the GPU against the oracle (max-abs 2e-3)."""
from __future__ import annotations

import numpy as np
import pytest

from abi_helpers import abi_prefill, max_abs, to_dev
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def case(seed, B, Sq, H, HKV, D, BS, ctx, dtype):
    _, k, v, bt, c = orc.make_decode_case(seed, B, H, HKV, D, BS, ctx)
    q = np.random.default_rng(seed + 1000).standard_normal((B, Sq, H, D), dtype=np.float32)
    return q, orc.round_to(k, dtype), orc.round_to(v, dtype), bt, c


@pytest.mark.parametrize("entry", ["pa_paged_attention_prefill", "pa_paged_attention_prefill_simt",
                                   "pa_paged_attention_prefill_wmma"])
@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_tensor_dtypes(entry, dtype, D):
    q, k, v, bt, ctx = case(30 + D, 2, 96, 8, 2, D, 16, [96, 300], dtype)
    out = abi_prefill(q, k, v, bt, ctx, D ** -0.5, dtype, entry=entry)
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, D ** -0.5, threads=8)) <= 2e-3


@pytest.mark.parametrize("dtype,D,BS", [("float32", 64, 16), ("float64", 32, 8),
                                        ("float16", 256, 16), ("float32", 128, 5)])
def test_prefill_cuda_core_dtypes(dtype, D, BS):
    q, k, v, bt, ctx = case(40, 2, 33, 4, 4, D, BS, [40, 33], dtype)
    out = abi_prefill(q, k, v, bt, ctx, D ** -0.5, dtype)
    tol = 2e-3 if dtype in ("float16", "bfloat16") else 1e-4
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, D ** -0.5)) <= tol


def test_padded_query_slots_are_zero():
    # Sq > ctx: the first Sq - ctx slots see no key (paged_attn_prefill.cu:70-74)
    q, k, v, bt, ctx = case(41, 2, 40, 4, 2, 64, 16, [10, 64], "float16")
    out = abi_prefill(q, k, v, bt, ctx, 0.125, "float16")
    assert np.all(out[0, :30] == 0)
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, 0.125)) <= 2e-3


def test_chunk_after_cached_prefix():
    # the chunk is the trailing 64 tokens of a 1000-token context
    q, k, v, bt, ctx = case(42, 3, 64, 8, 8, 128, 16, [1000, 64, 513], "bfloat16")
    out = abi_prefill(q, k, v, bt, ctx, 0.088, "bfloat16")
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, 0.088, threads=8)) <= 2e-3


def test_shim_prefill_and_wmma_checks():
    import torch
    from pa_b200 import ops
    q, k, v, bt, ctx = case(43, 2, 32, 4, 2, 64, 16, [32, 50], "float16")
    args = [to_dev(q), to_dev(k, "float16"), to_dev(v, "float16"), to_dev(bt), to_dev(ctx)]
    ref = orc.prefill(q, k, v, bt, ctx, 0.125)
    assert max_abs(ops.paged_attention_prefill(*args, 0.125).cpu().numpy(), ref) <= 2e-3
    assert max_abs(ops.paged_attention_prefill_wmma(*args, 0.125).cpu().numpy(), ref) <= 2e-3
    k32 = args[1].float()
    with pytest.raises(RuntimeError, match="the WMMA path needs an fp16 KV cache"):
        ops.paged_attention_prefill_wmma(args[0], k32, k32, *args[3:], 0.125)
    k8 = torch.zeros((8, 8, 2, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="block_size == 16"):
        ops.paged_attention_prefill_wmma(args[0], k8, k8, *args[3:], 0.125)
    with pytest.raises(RuntimeError, match=r"q must be \[B, S, H, D\]"):
        ops.paged_attention_prefill(args[0][0], *args[1:], 0.125)


@pytest.mark.parametrize("dtype,D", [("bfloat16", 128), ("float16", 128), ("bfloat16", 64),
                                     ("float16", 64)])
def test_tensor_core_path_multi_tile_gqa(dtype, D):
    # 3 query tiles of 128 rows, a 700-token context (ragged last page and
    # last KV tile), GQA 8q/2kv: the tcgen05 path against oracle and SIMT path
    q, k, v, bt, ctx = case(44, 2, 300, 8, 2, D, 16, [700, 300], dtype)
    scale = D ** -0.5
    ref = orc.prefill(q, k, v, bt, ctx, scale, threads=8)
    tc = abi_prefill(q, k, v, bt, ctx, scale, dtype)
    simt = abi_prefill(q, k, v, bt, ctx, scale, dtype, entry="pa_paged_attention_prefill_simt")
    assert max_abs(tc, ref) <= 2e-3
    assert max_abs(simt, ref) <= 2e-3


def test_tensor_core_path_block_size_32_and_padding():
    # block_size 32 (two 16-row boxes per page); Sq > ctx for seq 0 (padded rows)
    q, k, v, bt, ctx = case(45, 2, 150, 4, 4, 128, 32, [100, 400], "bfloat16")
    out = abi_prefill(q, k, v, bt, ctx, 0.088, "bfloat16")
    assert np.all(out[0, :50] == 0)
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, 0.088, threads=8)) <= 2e-3


@pytest.mark.parametrize("dtype,D,BS", [("bfloat16", 128, 16), ("float16", 64, 16),
                                        ("bfloat16", 128, 32)])
def test_tensor_core_path_pages_in_order(dtype, D, BS):
    # pages allocated in order (block id = page index, as a fresh allocator
    # hands them out): every full KV tile is one run of pool rows; the second
    # sequence's table is reversed in its second half so runs and scattered
    # tiles meet in one launch; a ragged context leaves a partial last tile
    q, k, v, _, ctx = case(46, 2, 260, 8, 4, D, BS, [900, 700], dtype)
    pages = [-(-int(c) // BS) for c in ctx]
    bt = np.zeros((2, max(pages)), np.int32)
    bt[0, :pages[0]] = np.arange(pages[0])
    second = np.arange(pages[0], pages[0] + pages[1])
    half = pages[1] // 2
    second[half:] = second[half:][::-1]
    bt[1, :pages[1]] = second
    scale = D ** -0.5
    out = abi_prefill(q, k, v, bt, ctx, scale, dtype)
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, scale, threads=8)) <= 2e-3


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_pair_path_repeats_bit_for_bit(dtype):
    # The CTA pairs hand S, P and O between the softmax warps and the tensor
    # core through barriers with relaxed semantics (the tcgen05 fences order
    # that tensor-memory data).  A missing order would show up as results
    # that change from launch to launch: 20 launches over 3 x 8 heads x 2
    # items of 512 rows must give identical bits, and the first must match
    # the oracle.
    q, k, v, bt, ctx = case(48, 3, 1000, 8, 4, 128, 16, [1000, 1200, 1500], dtype)
    scale = 128 ** -0.5
    kd, vd = to_dev(k, dtype), to_dev(v, dtype)
    first = abi_prefill(q, kd, vd, bt, ctx, scale, dtype)
    assert max_abs(first, orc.prefill(q, k, v, bt, ctx, scale, threads=8)) <= 2e-3
    for _ in range(19):
        again = abi_prefill(q, kd, vd, bt, ctx, scale, dtype)
        assert np.array_equal(again.view(np.uint32), first.view(np.uint32))


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_pair_path_ragged_items_and_empty_chains(dtype):
    # head_dim 128 on CTA pairs, 512 query rows per pair as two chains of 256:
    # 3 x 40 heads x 2 items = 240 items.  Sq = 600: the second item's second
    # chain (rows 768..) is empty; ctx 100 < Sq leaves the first item's first
    # chain with no visible key while its second chain has one tile; ctx 900
    # puts a cached prefix before the chunk.
    q, k, v, bt, ctx = case(47, 3, 600, 40, 8, 128, 16, [900, 600, 100], dtype)
    scale = 128 ** -0.5
    out = abi_prefill(q, k, v, bt, ctx, scale, dtype)
    assert np.all(out[2, :500] == 0)
    assert max_abs(out, orc.prefill(q, k, v, bt, ctx, scale, threads=8)) <= 2e-3
