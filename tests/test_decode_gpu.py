"""Split-KV decode on the GPU, through the C ABI, against the CPU oracle
(tolerance: max-abs 2e-3, the bar for fp16/bf16 pools with fp32 accumulation;
fp32/fp64 pools are held to 1e-4)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from abi_helpers import abi_decode, max_abs, to_dev, TORCH_DT
from oracle import oracle as orc
from pa_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {"float16": 2e-3, "bfloat16": 2e-3, "float32": 1e-4, "float64": 1e-4}


def case(seed, B, H, HKV, D, BS, ctx, dtype, **kw):
    q, k, v, bt, c = orc.make_decode_case(seed, B, H, HKV, D, BS, ctx, **kw)
    return q, orc.round_to(k, dtype), orc.round_to(v, dtype), bt, c


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32", "float64"])
@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_dtypes_and_head_dims(dtype, D):
    q, k, v, bt, ctx = case(100 + D, 3, 4, 2, D, 16, [1, 45, 260], dtype)
    scale = D ** -0.5
    out = abi_decode(q, k, v, bt, ctx, scale, dtype)
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, scale)) <= TOL[dtype]


@pytest.mark.parametrize("H,HKV", [(1, 1), (12, 12), (8, 4), (12, 4), (32, 8), (16, 1),
                                   (32, 2), (6, 2), (64, 4)])
def test_gqa_groupings(H, HKV):
    q, k, v, bt, ctx = case(7, 2, H, HKV, 128, 16, [33, 130], "bfloat16")
    out = abi_decode(q, k, v, bt, ctx, 0.088, "bfloat16")
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, 0.088)) <= 2e-3


@pytest.mark.parametrize("BS", [1, 3, 8, 16, 32, 64])
def test_block_sizes(BS):
    q, k, v, bt, ctx = case(8, 3, 4, 4, 64, BS, [1, 17, 95], "float16")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16")
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, 0.125)) <= 2e-3


@pytest.mark.parametrize("num_splits", [0, 1, 2, 3, 16, 64])
def test_explicit_num_splits(num_splits):
    q, k, v, bt, ctx = case(9, 4, 12, 12, 64, 16, [2048, 100, 7, 1000], "float16")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16", num_splits=num_splits)
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, 0.125)) <= 2e-3


@pytest.mark.parametrize("entry", ["pa_paged_attention", "pa_paged_attention_v2",
                                   "pa_paged_attention_v3"])
def test_v1_v2_v3_entry_points(entry):
    q, k, v, bt, ctx = case(10, 5, 12, 12, 64, 16, [512, 1, 77, 300, 16], "float16")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16", entry=entry)
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, 0.125)) <= 2e-3


def test_long_single_sequence_split_over_all_sms():
    # one sequence spread over every CTA: exercises the last-arriver merge
    q, k, v, bt, ctx = case(11, 1, 32, 8, 128, 16, [32768], "bfloat16")
    out = abi_decode(q, k, v, bt, ctx, 0.088, "bfloat16")
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, 0.088, threads=8)) <= 2e-3


def test_ragged_batch_many_sequences():
    rng = np.random.default_rng(12)
    ctxs = rng.integers(1, 700, size=67).tolist()
    q, k, v, bt, ctx = case(12, 67, 8, 2, 64, 16, ctxs, "float16")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16")
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, 0.125, threads=8)) <= 2e-3


def test_empty_contexts_give_nan_like_reference_v3():
    q, k, v, bt, ctx = case(13, 4, 4, 2, 64, 16, [0, 20, 0, 5], "float16")
    ctx = np.array([0, 20, -3, 5], np.int32)
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16")
    assert np.isnan(out[0]).all() and np.isnan(out[2]).all()
    ref = orc.decode(q, k, v, bt, ctx, 0.125)
    assert max_abs(out[[1, 3]], ref[[1, 3]]) <= 2e-3


def test_all_empty_batch():
    q, k, v, bt, ctx = case(14, 3, 4, 4, 64, 16, [0, 0, 0], "float16")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16")
    assert np.isnan(out).all()


def test_lse_output():
    q, k, v, bt, ctx = case(15, 3, 8, 2, 128, 16, [1, 90, 1500], "bfloat16")
    scale = 0.088
    out, lse = abi_decode(q, k, v, bt, ctx, scale, "bfloat16", want_lse=True)
    # ln sum_j exp(scale q.k_j) in float64
    for b in range(3):
        for h in range(8):
            g = h // 4
            n = int(ctx[b])
            ks = np.stack([k[bt[b, j // 16], j % 16, g] for j in range(n)]).astype(np.float64)
            s = scale * ks @ q[b, h].astype(np.float64)
            want = s.max() + np.log(np.exp(s - s.max()).sum())
            assert abs(lse[b, h] - want) < 1e-3


@pytest.mark.parametrize("num_splits", [0, 40])
def test_long_sequences_two_level_merge(num_splits):
    """Two long GQA sequences spread over every SM (automatic splitting) or
    over 40 CTAs each: a sequence spans more than 8 CTAs, so its pieces merge
    in runs of 8 and then across runs; out and lse both checked."""
    q, k, v, bt, ctx = case(16, 2, 32, 8, 128, 16, [9000, 3001], "bfloat16")
    scale = 0.088
    out, lse = abi_decode(q, k, v, bt, ctx, scale, "bfloat16", want_lse=True,
                          num_splits=num_splits)
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, scale)) <= 2e-3
    for b in range(2):
        n = int(ctx[b])
        ks = k[bt[b, :(n + 15) // 16]].reshape(-1, 8, 128)[:n].astype(np.float64)
        for h in (0, 5, 31):
            s = scale * ks[:, h // 4] @ q[b, h].astype(np.float64)
            want = s.max() + np.log(np.exp(s - s.max()).sum())
            assert abs(lse[b, h] - want) < 1e-3


def test_weighted_split_ragged_batch():
    """Enough tiles over the automatic split (148 CTAs on a B200) that the
    split weights each sequence start as extra tiles: ragged lengths, an
    empty sequence and a one-token one; out and lse against the oracle."""
    ctxs = [9000, 0, 7000, 1, 8500, 9000, 40]
    q, k, v, bt, ctx = case(17, len(ctxs), 8, 2, 64, 16, ctxs, "float16")
    scale = 0.125
    out, lse = abi_decode(q, k, v, bt, ctx, scale, "float16", want_lse=True)
    want = orc.decode(q, k, v, bt, ctx, scale)
    live = [b for b, c in enumerate(ctxs) if c > 0]
    assert max_abs(out[live], want[live]) <= 2e-3
    assert np.isnan(out[1]).all()  # empty sequence: NaN row, as the v3 entry point
    for b in (0, 3, 6):
        n = int(ctx[b])
        ks = k[bt[b, :(n + 15) // 16]].reshape(-1, 2, 64)[:n].astype(np.float64)
        for h in (0, 7):
            s_ = scale * ks[:, h // 4] @ q[b, h].astype(np.float64)
            assert abs(lse[b, h] - (s_.max() + np.log(np.exp(s_ - s_.max()).sum()))) < 1e-3


def test_hip_selftest_fixture():
    """The reference's own HIP self-test (mt19937(7) inputs, tolerance 3e-4,
    rocm/hip/paged_attn_v1_hip.cpp:151-198) run on the B200 kernel."""
    q, k, v, bt, ctx = orc.fixture_hip_selftest()
    scale = float(1.0 / np.sqrt(np.float32(32)))
    out = abi_decode(q, k, v, bt, ctx, scale, "float32")
    assert max_abs(out, orc.decode(q, k, v, bt, ctx, scale)) < 3e-4


def test_out_of_range_block_ids_are_reported_not_read():
    q, k, v, bt, ctx = case(16, 2, 4, 4, 64, 16, [40, 40], "float16")
    bt = bt.copy()
    bt[1, 1] = 10_000_000  # far outside the pool
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16", status=status)
    assert int(status.item()) & _lib.PA_DEVERR_BLOCK_ID
    # sequence 0 is untouched by the bad entry
    assert max_abs(out[0], orc.decode(q[:1], k, v, bt[:1], ctx[:1], 0.125)[0]) <= 2e-3


def test_context_longer_than_table_is_clamped_and_reported():
    q, k, v, bt, ctx = case(17, 2, 4, 4, 64, 16, [32, 32], "float16")
    ctx = np.array([32, 5000], np.int32)  # table holds 2 blocks = 32 tokens
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = abi_decode(q, k, v, bt, ctx, 0.125, "float16", status=status)
    assert int(status.item()) & _lib.PA_DEVERR_CONTEXT
    ref = orc.decode(q, k, v, bt, np.array([32, 32], np.int32), 0.125)
    assert max_abs(out, ref) <= 2e-3


def test_pool_beyond_2_31_elements():
    """Config-3 geometry (8 KV heads x 128, bf16): a [NB, 16, 8, 128] pool with
    NB > 131072 has more than 2^31 elements per K tensor; the blocks used sit
    at the top of it, so every offset crosses 2^31."""
    NB = 140_000
    H, HKV, D, BS = 32, 8, 128, 16
    assert NB * BS * HKV * D > 2**31
    ctxs = [300, 1025]
    q, kc, vc, btc, ctx = case(18, 2, H, HKV, D, BS, ctxs, "bfloat16")
    used = btc.max() + 1
    hi = NB - used  # map compact block i -> NB - used + i
    bt = (btc + hi).astype(np.int32)
    k = torch.zeros((NB, BS, HKV, D), dtype=torch.bfloat16, device="cuda")
    v = torch.zeros_like(k)
    k[hi:] = torch.from_numpy(kc).to("cuda", torch.bfloat16)
    v[hi:] = torch.from_numpy(vc).to("cuda", torch.bfloat16)
    out = abi_decode(q, k, v, bt, ctx, 0.088, "bfloat16")
    assert max_abs(out, orc.decode(q, kc, vc, btc, ctx, 0.088)) <= 2e-3
    del k, v
    torch.cuda.empty_cache()


def test_torch_shim_matches_abi_and_checks_args():
    from pa_b200 import ops
    q, k, v, bt, ctx = case(19, 3, 12, 4, 128, 16, [100, 200, 3], "float16")
    dev = "cuda"
    args = [to_dev(q), to_dev(k, "float16"), to_dev(v, "float16"), to_dev(bt), to_dev(ctx)]
    ref = orc.decode(q, k, v, bt, ctx, 0.088)
    for fn in (ops.paged_attention, ops.paged_attention_v2):
        assert max_abs(fn(*args, 0.088).cpu().numpy(), ref) <= 2e-3
    assert max_abs(ops.paged_attention_v3(*args, 0.088, 0).cpu().numpy(), ref) <= 2e-3
    assert max_abs(ops.paged_attention_v3(*args, 0.088, 5).cpu().numpy(), ref) <= 2e-3
    # int64 block tables / context lengths are converted like the reference does
    a64 = args[:3] + [args[3].long(), args[4].long()]
    assert max_abs(ops.paged_attention_v3(*a64, 0.088, 0).cpu().numpy(), ref) <= 2e-3
    with pytest.raises(RuntimeError, match="n_head must be divisible by n_kv_head"):
        ops.paged_attention_v3(to_dev(q[:, :10]), *args[1:], 0.088, 0)
    bad = torch.zeros((2, 4, 4, 48), dtype=torch.float16, device=dev)
    with pytest.raises(RuntimeError, match="head_dim must be a multiple of the warp size"):
        ops.paged_attention_v2(torch.zeros((1, 4, 48), device=dev), bad, bad, args[3][:1],
                               args[4][:1], 0.1)
    assert ops.choose_num_splits(64, 12, 2048) == orc.choose_num_splits(
        64, 12, 2048, torch.cuda.get_device_properties(0).multi_processor_count)


def test_stream_semantics_follow_current_torch_stream():
    from pa_b200 import ops
    q, k, v, bt, ctx = case(20, 8, 12, 12, 64, 16, 1024, "float16")
    args = [to_dev(q), to_dev(k, "float16"), to_dev(v, "float16"), to_dev(bt), to_dev(ctx)]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = ops.paged_attention_v3(*args, 0.125, 0)
    s.synchronize()
    assert max_abs(out.cpu().numpy(), orc.decode(q, k, v, bt, ctx, 0.125, threads=8)) <= 2e-3


def test_validate_block_tables():
    from pa_b200 import ops
    bt = torch.tensor([[0, 1, 99], [2, -1, 0]], dtype=torch.int32, device="cuda")
    ctx = torch.tensor([48, 17], dtype=torch.int32, device="cuda")
    bad_ids, long_ctx = ops.validate_block_tables(bt, ctx, 10, 16)
    assert bad_ids == 2 and long_ctx == 0
    ctx2 = torch.tensor([49, 1], dtype=torch.int32, device="cuda")
    assert ops.validate_block_tables(bt, ctx2, 100, 16) == (0, 1)


def test_repeated_calls_reuse_workspace_state():
    # one workspace reused call after call: the merge counters carry each
    # launch's tag, so what an earlier call left reads as zero
    q, k, v, bt, ctx = case(21, 2, 8, 8, 64, 16, [3000, 5000], "float16")
    ref = orc.decode(q, k, v, bt, ctx, 0.125, threads=8)
    for _ in range(3):
        assert max_abs(abi_decode(q, k, v, bt, ctx, 0.125, "float16"), ref) <= 2e-3
