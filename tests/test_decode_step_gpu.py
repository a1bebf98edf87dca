"""One layer of a decode step (pa_decode_layer_step / ops.decode_layer_step /
TorchBlockAllocator.decode_step), an addition beyond the reference: q / out in
bf16 or fp16 give exactly the fp32 path's output rounded to that type, and the
fused K/V append leaves the pool and the output bit-identical to pa_append_kv
followed by pa_paged_attention_v3 -- split and unsplit sequences, GQA, pages
that start with the new token, empty sequences, more than 1024 sequences (the
plan-kernel path)."""
from __future__ import annotations

import pytest
import torch

from pa_b200 import ops
from pa_b200.kv import KVConfig, ModelConfig, TorchBlockAllocator

pytestmark = pytest.mark.gpu

TDT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def same(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bit-level equality with NaN rows allowed in the same places."""
    na, nb = torch.isnan(a), torch.isnan(b)
    return bool(torch.equal(na, nb)) and bool(torch.equal(a[~na], b[~nb]))


def setup(pool_dtype, ctxs, H, HKV, D, BS=16, seed=0, spare=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nb = sum((c + spare + BS - 1) // BS for c in ctxs) + 4
    k = torch.randn((nb, BS, HKV, D), generator=g, device="cuda").to(TDT[pool_dtype])
    v = torch.randn((nb, BS, HKV, D), generator=g, device="cuda").to(TDT[pool_dtype])
    mb = max((c + spare + BS - 1) // BS for c in ctxs)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + 1))
    bt = torch.zeros((len(ctxs), mb), dtype=torch.int32)
    cur = 0
    for b, c in enumerate(ctxs):
        n = (c + spare + BS - 1) // BS
        bt[b, :n] = perm[cur:cur + n].int()
        cur += n
    return k, v, bt.cuda(), g


SHAPES = [  # (contexts, H, HKV, D)
    ([37, 2048, 0, 1, 4000, 16, 300], 8, 2, 64),
    ([5000, 7, 130], 32, 8, 128),
    ([64] * 20, 12, 12, 64),
]


@pytest.mark.parametrize("io", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("pool_dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("shape", range(len(SHAPES)))
def test_io_dtype_is_the_fp32_output_rounded(io, pool_dtype, shape):
    ctxs, H, HKV, D = SHAPES[shape]
    k, v, bt, g = setup(pool_dtype, ctxs, H, HKV, D, seed=shape)
    ctx = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    q = torch.randn((len(ctxs), H, D), generator=g, device="cuda").to(io)
    none = torch.empty(0, device="cuda")
    got = ops.decode_layer_step(q, k, v, bt, ctx, D ** -0.5, none, none)
    assert got.dtype == io
    want = ops.paged_attention_v3(q.float(), k, v, bt, ctx, D ** -0.5, 0)
    torch.cuda.synchronize()
    assert same(got, want.to(io))


@pytest.mark.parametrize("pool_dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("shape", range(len(SHAPES)))
def test_fused_append_equals_append_then_decode(pool_dtype, shape):
    ctxs, H, HKV, D = SHAPES[shape]
    ctxs = [c + 1 if c else 0 for c in ctxs]  # context_lens count the new token
    k, v, bt, g = setup(pool_dtype, ctxs, H, HKV, D, seed=10 + shape)
    ctx = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    B = len(ctxs)
    q = torch.randn((B, H, D), generator=g, device="cuda")
    kn = torch.randn((B, HKV, D), generator=g, device="cuda")
    vn = torch.randn((B, HKV, D), generator=g, device="cuda")
    k2, v2 = k.clone(), v.clone()
    got = ops.decode_layer_step(q, k, v, bt, ctx, D ** -0.5, kn, vn)
    # the same step in two launches: the batched append, then the decode
    pos = (ctx - 1).to(torch.int32)
    empty = torch.empty(0)
    ops.append_kv([k2], [v2], bt, pos, kn[None], vn[None], empty, empty)
    want = ops.paged_attention_v3(q, k2, v2, bt, ctx, D ** -0.5, 0)
    torch.cuda.synchronize()
    assert torch.equal(k.view(torch.uint8), k2.view(torch.uint8))
    assert torch.equal(v.view(torch.uint8), v2.view(torch.uint8))
    assert same(got, want)


def test_fused_append_many_sequences_plan_kernel_path():
    B, H, HKV, D, BS = 1100, 4, 4, 64, 16
    ctxs = [1 + (i * 37) % 90 for i in range(B)]
    k, v, bt, g = setup("float16", ctxs, H, HKV, D, BS, seed=21)
    ctx = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    q = torch.randn((B, H, D), generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.randn((B, HKV, D), generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn((B, HKV, D), generator=g, device="cuda").to(torch.bfloat16)
    k2, v2 = k.clone(), v.clone()
    got = ops.decode_layer_step(q, k, v, bt, ctx, D ** -0.5, kn, vn)
    empty = torch.empty(0)
    ops.append_kv([k2], [v2], bt, (ctx - 1).int(), kn[None], vn[None], empty, empty)
    want = ops.paged_attention_v3(q.float(), k2, v2, bt, ctx, D ** -0.5, 0)
    torch.cuda.synchronize()
    assert torch.equal(k.view(torch.int16), k2.view(torch.int16))
    assert torch.equal(v.view(torch.int16), v2.view(torch.int16))
    assert same(got, want.to(torch.bfloat16))


def test_fp8_pool_with_append_is_refused():
    k = torch.zeros((8, 16, 2, 64), dtype=torch.float8_e4m3fn, device="cuda")
    bt = torch.zeros((1, 2), dtype=torch.int32, device="cuda")
    ctx = torch.tensor([3], dtype=torch.int32, device="cuda")
    q = torch.randn((1, 2, 64), device="cuda")
    kn = torch.randn((1, 2, 64), device="cuda")
    with pytest.raises(RuntimeError):
        ops.decode_layer_step(q, k, k.clone(), bt, ctx, 0.125, kn, kn)


def test_engine_decode_step_over_layers():
    L, H, HKV, D = 3, 8, 2, 64
    m = ModelConfig(n_layer=L, n_head=H, head_dim=D, n_kv_head=HKV)
    a = TorchBlockAllocator(KVConfig(16, 64, "bfloat16"), m, "cuda")
    b = TorchBlockAllocator(KVConfig(16, 64, "bfloat16"), m, "cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    for alloc in (a, b):
        for layer in range(L):
            alloc.pool[layer, 0].copy_(torch.randn(alloc.pool[layer, 0].shape, generator=
                                                   torch.Generator(device="cuda").manual_seed(layer),
                                                   device="cuda").to(torch.bfloat16))
            alloc.pool[layer, 1].copy_(alloc.pool[layer, 0] * 0.5)
    seqs = [a.allocate(range(n)) for n in (40, 100, 7)]
    for n in (40, 100, 7):
        b.allocate(range(n))
    bt = a.block_table(seqs)
    ctx = torch.tensor([40, 100, 7], dtype=torch.int32, device="cuda")
    q = torch.randn((L, 3, H, D), generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.randn((L, 3, HKV, D), generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn((L, 3, HKV, D), generator=g, device="cuda").to(torch.bfloat16)
    got = a.decode_step(q, bt, ctx, kn, vn)
    b.append_kv(bt, (ctx - 1).int(), kn, vn)
    want = torch.stack([ops.paged_attention_v3(q[layer].float(), *b.layer_kv(layer), bt, ctx,
                                               D ** -0.5, 0) for layer in range(L)])
    torch.cuda.synchronize()
    assert got.shape == (L, 3, H, D) and got.dtype == torch.bfloat16
    assert same(got, want.to(torch.bfloat16))
    for layer in range(L):
        assert torch.equal(a.pool[layer].view(torch.int16), b.pool[layer].view(torch.int16))
