"""KV-pool writer on the GPU: bit-exact against the numpy oracle, including a
monolithic pool past 2^31 elements -- the shape at which the reference's pool
write faulted (b=64, ctx=2048: 8448 blocks, gb10-attn README.md:109-132)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from abi_helpers import TORCH_DT
from oracle import oracle as orc
from pa_b200 import ops
from pa_b200.kv import KVConfig, ModelConfig, TorchBlockAllocator

pytestmark = pytest.mark.gpu

BITS = {"float16": torch.int16, "bfloat16": torch.int16, "float32": torch.int32,
        "float64": torch.int64}
NPBITS = {"float16": np.uint16, "bfloat16": np.uint16, "float32": np.uint32,
          "float64": np.uint64}


def pool_bits(alloc) -> np.ndarray:
    L = alloc.model_cfg.n_layer
    t = torch.stack([alloc.pool[i] for i in range(L)]) if alloc.layered else alloc.pool
    dt = str(t.dtype).replace("torch.", "")
    return t.cpu().view(BITS[dt]).numpy().view(NPBITS[dt])


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32", "float64"])
@pytest.mark.parametrize("layered", [True, False])
def test_bit_exact_vs_oracle(dtype, layered):
    m = ModelConfig(n_layer=3, n_head=4, head_dim=64)
    alloc = TorchBlockAllocator(KVConfig(16, 40, dtype), m, "cuda", layered=layered)
    rng = np.random.default_rng(1)
    want = np.zeros((3, 2, 40, 16, 4, 64), NPBITS[dtype])
    ids = alloc.allocate(range(96)).block_ids
    for T, start in [(50, 0), (7, 50), (33, 57)]:
        k = (rng.standard_normal((3, 4, T, 64)) * 3).astype(np.float32)
        v = (rng.standard_normal((3, 4, T, 64)) * 3).astype(np.float32)
        alloc.write_kv(ids, start, k, v)
        orc.write_kv(want, ids, start, k, v, dtype)
    torch.cuda.synchronize()
    assert np.array_equal(pool_bits(alloc), want)


@pytest.mark.parametrize("src", ["float16", "bfloat16"])
def test_half_sources_from_device(src):
    m = ModelConfig(n_layer=2, n_head=8, head_dim=128)
    alloc = TorchBlockAllocator(KVConfig(16, 20, "bfloat16"), m, "cuda")
    rng = np.random.default_rng(2)
    k32 = rng.standard_normal((2, 8, 70, 128)).astype(np.float32)
    v32 = rng.standard_normal((2, 8, 70, 128)).astype(np.float32)
    k = torch.from_numpy(k32).to("cuda", TORCH_DT[src])
    v = torch.from_numpy(v32).to("cuda", TORCH_DT[src])
    ids = alloc.allocate(range(70)).block_ids
    alloc.write_kv(ids, 0, k, v)
    want = np.zeros((2, 2, 20, 16, 8, 128), np.uint16)
    orc.write_kv(want, ids, 0, k.float().cpu().numpy(), v.float().cpu().numpy(), "bfloat16")
    torch.cuda.synchronize()
    assert np.array_equal(pool_bits(alloc), want)


def test_odd_block_size_and_head_dim_scalar_path():
    m = ModelConfig(n_layer=1, n_head=3, head_dim=36)  # D % 8 != 0 -> per-element path
    alloc = TorchBlockAllocator(KVConfig(7, 12, "float16"), m, "cuda")
    rng = np.random.default_rng(3)
    k = rng.standard_normal((1, 3, 40, 36)).astype(np.float32)
    v = rng.standard_normal((1, 3, 40, 36)).astype(np.float32)
    ids = alloc.allocate(range(45)).block_ids
    alloc.write_kv(ids, 5, k, v)
    want = np.zeros((1, 2, 12, 7, 3, 36), np.uint16)
    orc.write_kv(want, ids, 5, k, v, "float16")
    torch.cuda.synchronize()
    assert np.array_equal(pool_bits(alloc), want)


def test_out_of_range_ids_reported_not_written():
    k0 = torch.zeros((4, 16, 2, 64), dtype=torch.float16, device="cuda")
    v0 = torch.zeros_like(k0)
    ids = torch.tensor([1, 99], dtype=torch.int32, device="cuda")
    k = torch.ones((1, 2, 32, 64), device="cuda")
    from abi_helpers import ptr, stream
    from pa_b200 import _lib
    import ctypes
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kl = (ctypes.c_void_p * 1)(k0.data_ptr())
    vl = (ctypes.c_void_p * 1)(v0.data_ptr())
    st = _lib.call("pa_write_kv", kl, vl, _lib.PA_DTYPE_F16, ptr(k), ptr(k), _lib.PA_DTYPE_F32,
                   k.stride(0), k.stride(1), k.stride(2), ptr(ids), 2, 0, 32, 1, 2, 64, 16, 4,
                   ptr(status), stream())
    assert st == 0
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PA_DEVERR_BLOCK_ID
    assert (k0[1] == 1).all() and (k0[[0, 2, 3]] == 0).all()


def test_monolithic_pool_beyond_2_31_elements():
    """gpt2 (12 layers, 12 heads, D=64, fp16) with 8448 blocks in ONE
    [12, 2, 8448, 16, 12, 64] tensor: 2.49e9 elements, layer 11 starts 2.28e9
    elements in (docs/REPORT.md:141-160).  Write a 2048-token sequence into
    the highest blocks and check every byte written."""
    m = ModelConfig()  # gpt2
    NB = 8448
    alloc = TorchBlockAllocator(KVConfig(16, NB, "float16"), m, "cuda", layered=False,
                                zero=False)
    assert alloc.pool.numel() > 2**31
    ids = list(range(NB - 128, NB))
    rng = np.random.default_rng(4)
    k = rng.standard_normal((12, 12, 2048, 64)).astype(np.float32)
    v = rng.standard_normal((12, 12, 2048, 64)).astype(np.float32)
    alloc.write_kv(ids, 0, k, v)
    torch.cuda.synchronize()
    got = alloc.pool[:, :, NB - 128:].cpu().view(torch.int16).numpy().view(np.uint16)
    want = np.zeros((12, 2, 128, 16, 12, 64), np.uint16)
    orc.write_kv(want, list(range(128)), 0, k, v, "float16")
    assert np.array_equal(got, want)
    hr = alloc.capacity_headroom()
    assert hr["int32_margin_elements"] < 0  # past the reference's wall, still correct
    del alloc
    torch.cuda.empty_cache()


def test_layered_pool_indexing_matches_monolithic():
    m = ModelConfig(n_layer=3, n_head=2, head_dim=32)
    lay = TorchBlockAllocator(KVConfig(4, 6, "float32"), m, "cuda")
    mono = torch.randn((3, 2, 6, 4, 2, 32), device="cuda")
    for i in range(3):
        lay.pool[i] = mono[i]
    assert torch.equal(lay.pool[1, 0], mono[1, 0])
    ids = torch.tensor([5, 0, 2], device="cuda")
    assert torch.equal(lay.pool[:, :, ids], mono[:, :, ids])
    lay.pool[2, 1] = torch.zeros_like(mono[2, 1])
    mono[2, 1] = 0
    assert torch.equal(torch.stack([lay.pool[i] for i in range(3)]), mono)
    assert ops is not None
