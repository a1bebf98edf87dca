"""FP8 (E4M3) KV pool on the GPU, an addition beyond the reference: the decode
of a quantised pool against the scalar fp32 oracle run on the dequantised
values (max-abs 2e-3, the bar of every decode test), and the pool writer byte
for byte against the oracle's quantiser (x / scale, round to nearest even,
saturating)."""
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

TOL = 2e-3


def fp8_case(seed, B, H, HKV, D, BS, ctx):
    """A decode case whose K/V heads differ in magnitude, quantised with the
    usual per-head scale amax / 448.  Returns device pools (e4m3) and scales,
    and the dequantised fp32 values the oracle sees."""
    q, k, v, bt, ctxs = orc.make_decode_case(seed, B, H, HKV, D, BS, ctx)
    rng = np.random.default_rng(seed + 1000)
    gain = rng.uniform(0.25, 4.0, (2, HKV)).astype(np.float32)
    k = k * gain[0][None, None, :, None]
    v = v * gain[1][None, None, :, None]
    ks = (np.abs(k).max(axis=(0, 1, 3)) / 448).astype(np.float32)
    vs = (np.abs(v).max(axis=(0, 1, 3)) / 448).astype(np.float32)
    kb = orc.quantize_e4m3(k, ks[None, None, :, None])
    vb = orc.quantize_e4m3(v, vs[None, None, :, None])
    kd = orc.e4m3_bits_to_f32(kb) * ks[None, None, :, None]
    vd = orc.e4m3_bits_to_f32(vb) * vs[None, None, :, None]
    dev = dict(k=torch.from_numpy(kb).cuda().view(torch.float8_e4m3fn),
               v=torch.from_numpy(vb).cuda().view(torch.float8_e4m3fn),
               ks=torch.from_numpy(ks).cuda(), vs=torch.from_numpy(vs).cuda())
    return q, kd.astype(np.float32), vd.astype(np.float32), bt, ctxs, dev


def abi_fp8(q, dev, bt, ctx, scale, num_splits=0, status=None):
    qd = torch.from_numpy(q).cuda()
    btd = torch.from_numpy(np.asarray(bt, np.int32)).cuda()
    ctxd = torch.from_numpy(np.asarray(ctx, np.int32)).cuda()
    B, H, D = qd.shape
    NB, BS, HKV, _ = dev["k"].shape
    MB = btd.shape[1]
    out = torch.empty((B, H, D), device="cuda", dtype=torch.float32)
    lse = torch.empty((B, H), device="cuda", dtype=torch.float32)
    n = ctypes.c_size_t(0)
    _lib.check("ws", _lib.call("pa_decode_workspace_size", B, H, HKV, D, _lib.PA_DTYPE_E4M3, BS,
                               MB, num_splits, ctypes.byref(n)))
    ws = torch.empty(max(n.value, 1), device="cuda", dtype=torch.uint8)
    _lib.check("pa_paged_attention_v3_fp8", _lib.call(
        "pa_paged_attention_v3_fp8", ptr(out), ptr(lse), ptr(qd), ptr(dev["k"]), ptr(dev["v"]),
        ptr(dev["ks"]), ptr(dev["vs"]), _lib.PA_DTYPE_E4M3, ptr(btd), ptr(ctxd), B, H, HKV, D, BS,
        NB, MB, float(scale), num_splits, ptr(ws), n.value, ptr(status), stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy(), lse.cpu().numpy()


def oracle_lse(q, k, bt, ctx, scale):
    """ln sum_j exp(scale q.k_j) per (b, h), in float64 from the dequantised K."""
    B, H, D = q.shape
    NB, BS, HKV, _ = k.shape
    out = np.full((B, H), -np.inf)
    for b in range(B):
        n = int(ctx[b])
        if n <= 0:
            continue
        pos = np.arange(n)
        rows = k[bt[b][pos // BS], pos % BS].astype(np.float64)  # [n, HKV, D]
        for h in range(H):
            s = rows[:, h // (H // HKV)] @ q[b, h].astype(np.float64) * scale
            mx = s.max()
            out[b, h] = mx + np.log(np.exp(s - mx).sum())
    return out


@pytest.mark.parametrize("B,H,HKV,D,BS,ctx", [
    (4, 12, 12, 64, 16, 2048),              # config-2 geometry (gpt2)
    (3, 32, 8, 128, 16, [5000, 1, 3000]),   # GQA, ragged
    (2, 8, 2, 32, 16, [700, 1500]),
    (2, 4, 4, 256, 16, [900, 64]),
    (3, 16, 4, 128, 8, [333, 1200, 17]),    # block size 8
    (2, 8, 8, 64, 48, [1000, 77]),          # 32-token tiles straddle 48-token pages
    (2, 4, 4, 64, 1, [200, 33]),            # one token per page
])
def test_decode_matches_oracle(B, H, HKV, D, BS, ctx):
    q, kd, vd, bt, ctxs, dev = fp8_case(70 + D, B, H, HKV, D, BS, ctx)
    scale = D ** -0.5
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    got, lse = abi_fp8(q, dev, bt, ctxs, scale, status=status)
    want = orc.decode(q, kd, vd, bt, ctxs, scale)
    assert int(status.item()) == 0
    assert max_abs(got, want) <= TOL
    assert max_abs(lse, oracle_lse(q, kd, bt, ctxs, scale)) <= TOL


def test_empty_sequences_and_explicit_splits():
    q, kd, vd, bt, ctxs, dev = fp8_case(81, 3, 8, 8, 64, 16, [0, 900, 4000])
    for splits in (0, 1, 7):
        got, _ = abi_fp8(q, dev, bt, ctxs, 0.125, num_splits=splits)
        want = orc.decode(q, kd, vd, bt, ctxs, 0.125)
        assert np.isnan(got[0]).all()
        assert max_abs(got[1:], want[1:]) <= TOL


def test_torch_shim_matches_abi():
    q, kd, vd, bt, ctxs, dev = fp8_case(82, 2, 32, 8, 128, 16, [3000, 1234])
    got, lse = abi_fp8(q, dev, bt, ctxs, 128 ** -0.5)
    out2, lse2 = ops.paged_attention_v3_fp8(torch.from_numpy(q).cuda(), dev["k"], dev["v"],
                                            torch.from_numpy(bt).cuda(),
                                            torch.from_numpy(ctxs).cuda(), 128 ** -0.5,
                                            dev["ks"], dev["vs"], 0)
    assert np.array_equal(out2.cpu().numpy(), got)
    assert np.array_equal(lse2.cpu().numpy(), lse)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        ops.paged_attention_v3_fp8(torch.from_numpy(q).cuda(), dev["k"].view(torch.uint8),
                                   dev["v"].view(torch.uint8), torch.from_numpy(bt).cuda(),
                                   torch.from_numpy(ctxs).cuda(), 0.1, dev["ks"], dev["vs"], 0)


def pool_bytes(alloc):
    L = alloc.model_cfg.n_layer
    t = torch.stack([alloc.pool[i].view(torch.uint8) for i in range(L)]) if alloc.layered \
        else alloc.pool.view(torch.uint8)
    return t.cpu().numpy()


@pytest.mark.parametrize("layered,D", [(True, 64), (False, 128), (True, 36)])
def test_write_kv_bit_exact(layered, D):
    L, HKV = 3, 4
    m = ModelConfig(n_layer=L, n_head=HKV, head_dim=D)
    alloc = TorchBlockAllocator(KVConfig(16, 40, "e4m3"), m, "cuda", layered=layered)
    rng = np.random.default_rng(9)
    ks = rng.uniform(0.002, 0.05, (L, HKV)).astype(np.float32)
    vs = rng.uniform(0.002, 0.05, (L, HKV)).astype(np.float32)
    alloc.set_scales(ks, vs)
    want = np.zeros((L, 2, 40, 16, HKV, D), np.uint8)
    ids = alloc.allocate(range(96)).block_ids
    for T, start in [(50, 0), (7, 50), (33, 57)]:
        k = (rng.standard_normal((L, HKV, T, D)) * 3).astype(np.float32)
        v = (rng.standard_normal((L, HKV, T, D)) * 3).astype(np.float32)
        k[0, 0, 0, :8] = [1e6, -1e6, 0.0, -0.0, 1e-12, -1e-12, 448 * ks[0, 0], 30.0]
        alloc.write_kv(ids, start, k, v)
        orc.write_kv(want, ids, start, k, v, "e4m3", ks, vs)
    torch.cuda.synchronize()
    assert np.array_equal(pool_bytes(alloc), want)


def test_write_then_decode_end_to_end():
    # the allocator's writer fills an FP8 pool, the decode reads it with the
    # same layer's scales: equal to the oracle on the dequantised pool
    L, H, HKV, D = 2, 16, 4, 128
    m = ModelConfig(n_layer=L, n_head=H, head_dim=D, n_kv_head=HKV)
    alloc = TorchBlockAllocator(KVConfig(16, 300, "e4m3"), m, "cuda")
    rng = np.random.default_rng(10)
    ctxs = [1500, 2200]
    k_all = [rng.standard_normal((L, HKV, n, D)).astype(np.float32) for n in ctxs]
    v_all = [rng.standard_normal((L, HKV, n, D)).astype(np.float32) for n in ctxs]
    amax_k = np.max([np.abs(k).max(axis=(2, 3)) for k in k_all], axis=0)
    amax_v = np.max([np.abs(v).max(axis=(2, 3)) for v in v_all], axis=0)
    alloc.set_scales(amax_k / 448, amax_v / 448)
    allocs = [alloc.allocate(range(n)) for n in ctxs]
    for a, k, v in zip(allocs, k_all, v_all):
        alloc.write_kv(a.block_ids, 0, k, v)
    bt = alloc.block_table(allocs)
    ctx_d = torch.tensor(ctxs, dtype=torch.int32, device="cuda")
    q = rng.standard_normal((2, H, D)).astype(np.float32)
    layer = 1
    ks, vs = alloc.layer_scales(layer)
    K, V = alloc.layer_kv(layer)
    out, _ = ops.paged_attention_v3_fp8(torch.from_numpy(q).cuda(), K, V, bt, ctx_d, D ** -0.5,
                                        ks, vs, 0)
    kd = orc.e4m3_bits_to_f32(K.view(torch.uint8).cpu().numpy()) * \
        ks.cpu().numpy()[None, None, :, None]
    vd = orc.e4m3_bits_to_f32(V.view(torch.uint8).cpu().numpy()) * \
        vs.cpu().numpy()[None, None, :, None]
    want = orc.decode(q, kd.astype(np.float32), vd.astype(np.float32), bt.cpu().numpy(),
                      np.asarray(ctxs, np.int32), D ** -0.5)
    assert max_abs(out.cpu().numpy(), want) <= TOL
