"""Many-sequence pool writer (pa_write_kv_batch / TorchBlockAllocator.
write_kv_batch): the pool after one batched call is bit-identical to the pool
after one write_kv per sequence, and to the numpy oracle's scatter, for every
pool dtype, ragged token counts (empty sequences included), nonzero starts
and more sequences than one launch takes (32)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from abi_helpers import ptr, stream
from oracle import oracle as orc
from pa_b200 import _lib
from pa_b200.kv import KVConfig, ModelConfig, TorchBlockAllocator

pytestmark = pytest.mark.gpu

BITS = {"float16": torch.int16, "bfloat16": torch.int16, "float32": torch.int32,
        "float64": torch.int64, "e4m3": torch.uint8}
NPBITS = {"float16": np.uint16, "bfloat16": np.uint16, "float32": np.uint32,
          "float64": np.uint64}


def pool_bits(alloc, dtype) -> torch.Tensor:
    L = alloc.model_cfg.n_layer
    t = torch.stack([alloc.pool[i] for i in range(L)]) if alloc.layered else alloc.pool
    return t.view(BITS[dtype]).cpu()


def make_batch(n_seq, L, H, D, BS, rng, src_dtype=torch.float32, max_tok=70):
    """n_seq sequences with disjoint pages: (block id lists, starts, ks, vs)."""
    ids, starts, ks, vs = [], [], [], []
    next_block = 0
    for i in range(n_seq):
        T = int(rng.integers(0, max_tok)) if i % 7 else 0  # every 7th sequence is empty
        start = int(rng.integers(0, 40))
        n_blocks = (start + T + BS - 1) // BS + 1
        ids.append(list(range(next_block, next_block + n_blocks))[::-1])  # pages out of order
        next_block += n_blocks
        starts.append(start)
        ks.append(torch.from_numpy(rng.standard_normal((L, H, T, D)).astype(np.float32) * 3)
                  .to("cuda", src_dtype))
        vs.append(torch.from_numpy(rng.standard_normal((L, H, T, D)).astype(np.float32) * 3)
                  .to("cuda", src_dtype))
    return ids, starts, ks, vs, next_block


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32", "float64", "e4m3"])
@pytest.mark.parametrize("layered", [True, False])
def test_batch_equals_per_sequence_writes(dtype, layered):
    rng = np.random.default_rng(11)
    L, H, D, BS = 3, 4, 64, 16
    ids, starts, ks, vs, nb = make_batch(41, L, H, D, BS, rng)
    m = ModelConfig(n_layer=L, n_head=H, head_dim=D)
    a = TorchBlockAllocator(KVConfig(BS, nb, dtype), m, "cuda", layered=layered)
    b = TorchBlockAllocator(KVConfig(BS, nb, dtype), m, "cuda", layered=layered)
    if dtype == "e4m3":
        sc = torch.from_numpy(rng.uniform(0.01, 0.05, (L, H)).astype(np.float32))
        for x in (a, b):
            x.set_scales(sc, sc * 1.5)
    a.write_kv_batch(ids, starts, ks, vs)
    for i in range(len(ids)):
        b.write_kv(ids[i], starts[i], ks[i], vs[i])
    torch.cuda.synchronize()
    assert torch.equal(pool_bits(a, dtype), pool_bits(b, dtype))
    if dtype != "e4m3":
        want = np.zeros((L, 2, nb, BS, H, D), NPBITS[dtype])
        for i in range(len(ids)):
            orc.write_kv(want, ids[i], starts[i], ks[i].cpu().numpy(), vs[i].cpu().numpy(), dtype)
        assert np.array_equal(pool_bits(a, dtype).numpy().view(NPBITS[dtype]), want)


@pytest.mark.parametrize("src", [torch.float16, torch.bfloat16])
def test_batch_half_sources_and_odd_shapes(src):
    # head_dim 40 with block_size 5: the scalar (one element per thread) path
    rng = np.random.default_rng(12)
    L, H, D, BS = 2, 3, 40, 5
    ids, starts, ks, vs, nb = make_batch(9, L, H, D, BS, rng, src_dtype=src, max_tok=30)
    m = ModelConfig(n_layer=L, n_head=H, head_dim=D)
    a = TorchBlockAllocator(KVConfig(BS, nb, "float16"), m, "cuda")
    b = TorchBlockAllocator(KVConfig(BS, nb, "float16"), m, "cuda")
    a.write_kv_batch(ids, starts, ks, vs)
    for i in range(len(ids)):
        b.write_kv(ids[i], starts[i], ks[i], vs[i])
    torch.cuda.synchronize()
    assert torch.equal(pool_bits(a, "float16"), pool_bits(b, "float16"))


def test_batch_bad_block_ids_reported_not_written():
    k0 = torch.zeros((4, 16, 2, 64), dtype=torch.float16, device="cuda")
    v0 = torch.zeros_like(k0)
    good = torch.tensor([2], dtype=torch.int32, device="cuda")
    bad = torch.tensor([1, 99], dtype=torch.int32, device="cuda")
    k = torch.ones((1, 2, 32, 64), device="cuda")
    seqs = (_lib.PaKvSeq * 2)()
    for i, (ids, n_tok) in enumerate([(good, 16), (bad, 32)]):
        seqs[i] = _lib.PaKvSeq(ptr(k), ptr(k), k.stride(0), k.stride(1), k.stride(2), ptr(ids),
                               ids.numel(), 0, n_tok)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kl = (ctypes.c_void_p * 1)(k0.data_ptr())
    vl = (ctypes.c_void_p * 1)(v0.data_ptr())
    st = _lib.call("pa_write_kv_batch", kl, vl, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32, seqs, 2,
                   1, 2, 64, 16, 4, None, None, ptr(status), stream())
    assert st == 0
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PA_DEVERR_BLOCK_ID
    assert (k0[1] == 1).all() and (k0[2] == 1).all() and (k0[[0, 3]] == 0).all()
