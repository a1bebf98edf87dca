"""One decode step's K/V append for a whole batch (pa_append_kv), an addition
beyond the reference: byte-exact against the oracle's scatter for every pool
dtype (fp8 with its scales), sequences without a token skipped, positions past
the block table and bad block ids reported and not written, and append ->
decode against the scalar oracle on the grown context."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from abi_helpers import max_abs, ptr, stream
from oracle import oracle as orc
from pa_b200 import _lib, ops
from pa_b200.kv import KVConfig, ModelConfig, TorchBlockAllocator

pytestmark = pytest.mark.gpu

BITS = {"float16": (torch.int16, np.uint16), "bfloat16": (torch.int16, np.uint16),
        "float32": (torch.int32, np.uint32), "e4m3": (torch.uint8, np.uint8)}


def pool_bits(alloc, dtype):
    L = alloc.model_cfg.n_layer
    tb, nb = BITS[dtype]
    t = torch.stack([alloc.pool[i].view(tb) for i in range(L)]) if alloc.layered \
        else alloc.pool.view(tb)
    return t.cpu().numpy().view(nb)


@pytest.mark.parametrize("dtype,layered", [("float16", True), ("bfloat16", False),
                                           ("float32", True), ("e4m3", True)])
def test_bit_exact_vs_oracle(dtype, layered):
    L, HKV, D, B = 3, 4, 64, 5
    m = ModelConfig(n_layer=L, n_head=HKV, head_dim=D)
    alloc = TorchBlockAllocator(KVConfig(16, 64, dtype), m, "cuda", layered=layered)
    rng = np.random.default_rng(3)
    ks = vs = None
    if dtype == "e4m3":
        ks = rng.uniform(0.005, 0.05, (L, HKV)).astype(np.float32)
        vs = rng.uniform(0.005, 0.05, (L, HKV)).astype(np.float32)
        alloc.set_scales(ks, vs)
    ctxs = [40, 17, 100, 0, 63]
    allocs = [alloc.allocate(range(n + 1)) for n in ctxs]  # room for the next token
    bt = alloc.block_table(allocs)
    want = pool_bits(alloc, dtype).copy()
    for step in range(3):
        positions = np.array([n + step if n + step < 16 * len(a.block_ids) else -1
                              for n, a in zip(ctxs, allocs)], np.int32)
        positions[1] = -1  # this sequence has no token this step
        k = (rng.standard_normal((L, B, HKV, D)) * 2).astype(np.float32)
        v = (rng.standard_normal((L, B, HKV, D)) * 2).astype(np.float32)
        alloc.append_kv(bt, torch.from_numpy(positions).cuda(), torch.from_numpy(k).cuda(),
                        torch.from_numpy(v).cuda())
        orc.append_kv(want, bt.cpu().numpy(), positions, k, v, dtype, ks, vs)
    torch.cuda.synchronize()
    assert np.array_equal(pool_bits(alloc, dtype), want)


def test_positions_past_the_table_and_bad_ids_are_reported_not_written():
    L, HKV, D, B, NB, BS = 2, 2, 64, 3, 8, 16
    k0 = torch.zeros((NB, BS, HKV, D), dtype=torch.float16, device="cuda")
    pools = [torch.zeros_like(k0) for _ in range(2 * L)]
    kl = (ctypes.c_void_p * L)(*[p.data_ptr() for p in pools[:L]])
    vl = (ctypes.c_void_p * L)(*[p.data_ptr() for p in pools[L:]])
    bt = torch.tensor([[0, 1], [2, 99], [4, 5]], dtype=torch.int32, device="cuda")
    pos = torch.tensor([32, 20, 5], dtype=torch.int32, device="cuda")  # 32: past 2 pages
    k = torch.ones((L, B, HKV, D), dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check("append", _lib.call("pa_append_kv", kl, vl, _lib.PA_DTYPE_F16, ptr(k), ptr(k),
                                   _lib.PA_DTYPE_F32, ptr(bt), 2, ptr(pos), B, L, HKV, D, BS,
                                   NB, None, None, ptr(status), stream()))
    torch.cuda.synchronize()
    st = int(status.item())
    assert st & _lib.PA_DEVERR_CONTEXT and st & _lib.PA_DEVERR_BLOCK_ID
    # only sequence 2's token (block 4, row 5) was written
    for p in pools:
        nz = torch.nonzero(p.float().abs().sum(dim=(2, 3))).cpu().tolist()
        assert nz == [[4, 5]]


def test_append_then_decode():
    # a decode step: append each sequence's next token, then decode over the
    # grown context; equal to the oracle on the whole K/V
    L, H, HKV, D = 2, 16, 4, 128
    m = ModelConfig(n_layer=L, n_head=H, head_dim=D, n_kv_head=HKV)
    alloc = TorchBlockAllocator(KVConfig(16, 200, "bfloat16"), m, "cuda")
    rng = np.random.default_rng(4)
    ctxs = [700, 1201, 15]
    allocs = [alloc.allocate(range(n + 1)) for n in ctxs]
    full_k = [rng.standard_normal((L, HKV, n + 1, D)).astype(np.float32) for n in ctxs]
    full_v = [rng.standard_normal((L, HKV, n + 1, D)).astype(np.float32) for n in ctxs]
    for a, k, v, n in zip(allocs, full_k, full_v, ctxs):
        alloc.write_kv(a.block_ids, 0, k[:, :, :n], v[:, :, :n])
    bt = alloc.block_table(allocs)
    k_new = np.stack([k[:, :, n] for k, n in zip(full_k, ctxs)], axis=1)  # [L, B, HKV, D]
    v_new = np.stack([v[:, :, n] for v, n in zip(full_v, ctxs)], axis=1)
    alloc.append_kv(bt, torch.tensor(ctxs, dtype=torch.int32).cuda(),
                    torch.from_numpy(k_new).cuda(), torch.from_numpy(v_new).cuda())
    q = rng.standard_normal((3, H, D)).astype(np.float32)
    layer = 1
    K, V = alloc.layer_kv(layer)
    ctx_new = torch.tensor([n + 1 for n in ctxs], dtype=torch.int32, device="cuda")
    out = ops.paged_attention_v3(torch.from_numpy(q).cuda(), K, V, bt, ctx_new, D ** -0.5, 0)
    kd = K.float().cpu().numpy()
    vd = V.float().cpu().numpy()
    want = orc.decode(q, kd, vd, bt.cpu().numpy(), ctx_new.cpu().numpy(), D ** -0.5)
    assert max_abs(out.cpu().numpy(), want) <= 2e-3
    # the appended rows are the bf16 rounding of the new tokens
    for b, n in enumerate(ctxs):
        blk = int(bt[b, n // 16])
        got = K[blk, n % 16].float().cpu().numpy()
        assert np.array_equal(got, orc.round_to(full_k[b][layer, :, n], "bfloat16"))
