"""Parity at BASELINE.json's own shapes: the B200 kernels, called through the
C ABI, against the scalar fp32 oracle on the same seeded inputs.

The oracle restates the reference's CPU decode
(gb10-attn rocm/hip/paged_attn_v1_hip.cpp:104-141) and its causal prefill rule
(kernels/paged_attn_prefill.cu:62-74).  Tolerance: max-abs 2e-3 for fp16 /
bf16 pools (fp32 accumulation), 1e-4 for the fp32 pool of configs[0].

Inputs are made with torch's CPU generator (the 10^8-value pools of these
shapes take numpy seconds per array); values are N(0, 1) and, for 16-bit
pools, rounded to the pool type before the oracle sees them, so both sides
read the same numbers.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from abi_helpers import abi_decode, abi_prefill, max_abs
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

THREADS = min(os.cpu_count() or 1, 64)
TORCH_DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def randn(shape, seed: int, dtype: str = "float32") -> np.ndarray:
    g = torch.Generator().manual_seed(seed)
    t = torch.randn(shape, generator=g)
    return t.to(TORCH_DT[dtype]).float().numpy()


def page_tables(ctx, BS: int, seed: int, base: int = 0):
    """Block tables over a seeded permutation of sum(ceil(ctx/BS)) pages,
    offset by `base`; returns (tables [B, MB] int32, pages used)."""
    need = [-(-int(c) // BS) for c in ctx]
    total = sum(need)
    perm = np.random.default_rng(seed).permutation(total).astype(np.int64) + base
    bt = np.zeros((len(ctx), max(need)), np.int64)
    cur = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[cur:cur + n]
        bt[b, n:] = perm[cur]
        cur += n
    return bt.astype(np.int32), total


@pytest.mark.parametrize("entry", ["pa_paged_attention", "pa_paged_attention_v2",
                                   "pa_paged_attention_v3"])
def test_config1_fixture_fp32(entry):
    """1 layer, H=12, D=64, block_size 16, B=4, ctx 2048, fp32
    q/K/V ~ N(0,1) from a seed, the block table a seeded permutation of 512
    physical blocks, scale 1/sqrt(64), output [4, 12, 64]."""
    q, k, v, bt, ctx = orc.make_decode_case(2026, 4, 12, 12, 64, 16, 2048)
    assert k.shape == (512, 16, 12, 64)
    assert sorted(bt.ravel().tolist()) == list(range(512))
    out = abi_decode(q, k, v, bt, ctx, 64 ** -0.5, "float32", entry=entry)
    assert out.shape == (4, 12, 64)
    ref = orc.decode(q, k, v, bt, ctx, 64 ** -0.5, threads=THREADS)
    assert max_abs(out, ref) <= 1e-4


def test_config2_full_layer_fp16():
    """configs[1], one full layer call: B=64, ctx 2048, H=HKV=12, D=64, fp16
    pool, random block tables (4096 pages, seeded permutation)."""
    B, H, D, BS, CTX = 64, 12, 64, 16, 2048
    bt, nb = page_tables([CTX] * B, BS, 21)
    q = randn((B, H, D), 22)
    k = randn((nb, BS, H, D), 23, "float16")
    v = randn((nb, BS, H, D), 24, "float16")
    ctx = np.full(B, CTX, np.int32)
    out = abi_decode(q, k, v, bt, ctx, D ** -0.5, "float16")
    ref = orc.decode(q, k, v, bt, ctx, D ** -0.5, threads=THREADS)
    assert max_abs(out, ref) <= 2e-3


def test_config3_seeded_contexts_on_pool_beyond_2_31(dev):
    """32 query / 8 KV heads, D=128, bf16, B=8, contexts
    U[1024, 32768] from rng(2026) (the bench's draw), one K and one V tensor
    of 140,000 x 16 x 8 x 128 = 2.29e9 elements each, the pages used placed
    at the top of the pool so every element offset is beyond 2^31."""
    H, HKV, D, BS, B, NB = 32, 8, 128, 16, 8, 140_000
    ctx = np.random.default_rng(2026).integers(1024, 32769, size=B).astype(np.int32)
    top = NB - sum(-(-int(c) // BS) for c in ctx)
    bt, used = page_tables(ctx, BS, 31, base=top)
    assert NB * BS * HKV * D > 2 ** 31 and top * BS * HKV * D > 2 ** 31
    q = randn((B, H, D), 32)
    k = randn((used, BS, HKV, D), 33, "bfloat16")
    v = randn((used, BS, HKV, D), 34, "bfloat16")
    kd = torch.empty((NB, BS, HKV, D), dtype=torch.bfloat16, device=dev)
    vd = torch.empty((NB, BS, HKV, D), dtype=torch.bfloat16, device=dev)
    kd[top:] = torch.from_numpy(k).to(dev, torch.bfloat16)
    vd[top:] = torch.from_numpy(v).to(dev, torch.bfloat16)
    out = abi_decode(q, kd, vd, bt, ctx, D ** -0.5, "bfloat16")
    del kd, vd
    torch.cuda.empty_cache()
    ref = orc.decode(q, k, v, bt - top, ctx, D ** -0.5, threads=THREADS)
    assert max_abs(out, ref) <= 2e-3


def test_config4_prefill_all_query_tiles():
    """causal prefill, B=4, Sq = ctx = 4096, 32 heads (MHA),
    D=128, bf16 pool in 16-token pages.  The kernel runs all 32 heads; the
    oracle checks heads 0 and 31 (every one of the 32 query tiles of 128 rows
    and every key tile of those heads)."""
    B, S, H, D, BS = 4, 4096, 32, 128, 16
    bt, nb = page_tables([S] * B, BS, 41)
    q = randn((B, S, H, D), 42)
    k = randn((nb, BS, H, D), 43, "bfloat16")
    v = randn((nb, BS, H, D), 44, "bfloat16")
    ctx = np.full(B, S, np.int32)
    out = abi_prefill(q, k, v, bt, ctx, D ** -0.5, "bfloat16")
    heads = [0, H - 1]
    sub = lambda x: np.ascontiguousarray(x[:, :, heads])  # noqa: E731
    ref = orc.prefill(sub(q), sub(k), sub(v), bt, ctx, D ** -0.5, threads=THREADS)
    assert max_abs(out[:, :, heads], ref) <= 2e-3
