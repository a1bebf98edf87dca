"""The CPU oracle against the reference's own outputs and its internal
consistency (CPU only)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("tokens,dim", [(2048, 64), (64, 128), (257, 32)])
def test_scalar_lane_bit_exact_vs_reference(tokens, dim):
    """pao_scores / pao_softmax == gb10-attn arm_cpu/src/scalar.cpp, bit for bit,
    on the inputs of the reference's own bench (arm_cpu/src/bench.cpp:56-63)."""
    g = np.load(GOLDEN / "arm_scalar.npz")
    query, keys = orc.fixture_arm_bench(tokens, dim)
    raw, sm = orc.scores_softmax(query, keys)
    assert np.array_equal(raw, g[f"t{tokens}_d{dim}_scores"])
    assert np.array_equal(sm, g[f"t{tokens}_d{dim}_softmax"])


def _ref_kernels():
    p = GOLDEN / "ref_kernels.npz"
    if not p.exists():
        pytest.skip("ref_kernels.npz not generated yet (needs a GPU run of make_golden.py)")
    return np.load(p)


def test_decode_vs_reference_kernels():
    """Oracle decode == the reference's v1/v2/v3 CUDA kernels' outputs (within the
    kernels' own fast-math error, observed <= 1.1e-6 in docs/REPORT.md:43)."""
    g = _ref_kernels()
    names = sorted({k.split("/")[0] for k in g.files if k.endswith("/v3")})
    assert names
    for n in names:
        q, k, v = g[f"{n}/q"], g[f"{n}/k"].astype(np.float32), g[f"{n}/v"].astype(np.float32)
        out = orc.decode(q, k, v, g[f"{n}/bt"], g[f"{n}/ctx"], float(g[f"{n}/scale"]))
        for which in ("v1", "v2", "v3"):
            np.testing.assert_allclose(out, g[f"{n}/{which}"], atol=2e-5, rtol=0, err_msg=n)


def test_hip_selftest_fixture_vs_reference_kernels():
    """The reference HIP self-test fixture (mt19937(7), tolerance 3e-4 at
    rocm/hip/paged_attn_v1_hip.cpp:198): inputs regenerated identically, oracle
    output within that tolerance of the reference kernels'."""
    g = _ref_kernels()
    q, k, v, bt, ctx = orc.fixture_hip_selftest()
    assert np.array_equal(q, g["hip_selftest/q"]) and np.array_equal(k, g["hip_selftest/k"])
    out = orc.decode(q, k, v, bt, ctx, float(g["hip_selftest/scale"]))
    for which in ("v1", "v2", "v3", "v3_s3"):
        assert np.abs(out - g[f"hip_selftest/{which}"]).max() < 3e-4


def test_prefill_vs_reference_kernels():
    g = _ref_kernels()
    for n in sorted({k.split("/")[0] for k in g.files if k.endswith("/prefill")}):
        q, k, v = g[f"{n}/q"], g[f"{n}/k"].astype(np.float32), g[f"{n}/v"].astype(np.float32)
        out = orc.prefill(q, k, v, g[f"{n}/bt"], g[f"{n}/ctx"], float(g[f"{n}/scale"]))
        np.testing.assert_allclose(out, g[f"{n}/prefill"], atol=2e-5, rtol=0, err_msg=n)
        # the reference's WMMA path rounds Q and P to half: its own error bound
        assert np.abs(out - g[f"{n}/wmma"]).max() < 2e-3, n


def test_choose_num_splits_vs_reference_kernels():
    g = _ref_kernels()
    sms = int(g["choose_num_splits/sms"])
    for (b, h, c), want in zip(g["choose_num_splits/args"], g["choose_num_splits/values"]):
        assert orc.choose_num_splits(int(b), int(h), int(c), sms) == int(want)


@pytest.mark.parametrize("b,h,c,sms,want", [
    (64, 12, 2048, 148, 64), (4, 12, 2048, 148, 64), (1, 12, 512, 148, 64),
    (1, 1, 32, 148, 64), (512, 12, 8192, 148, 64), (1024, 32, 64, 148, 2), (2048, 32, 40, 148, 1),
    (0, 0, 0, 148, 64), (16, 12, 512, 48, 16), (32, 12, 2048, 48, 64)])
def test_choose_num_splits_formula(b, h, c, sms, want):
    """kernels/paged_attn_v3.cu:181-189, evaluated by hand for these inputs."""
    have = max(b * h, 1)
    expect = max(1, min(max(max(c // 32, 1), max((sms * 8 + have - 1) // have, 1)), 64))
    assert expect == want
    assert orc.choose_num_splits(b, h, c, sms) == want


@pytest.mark.parametrize("S", [1, 2, 7, 64])
def test_split_merge_equals_two_pass(S):
    q, k, v, bt, ctx = orc.make_decode_case(5, B=3, H=6, HKV=2, D=64, BS=16, ctx=[1, 50, 333])
    a = orc.decode(q, k, v, bt, ctx, 0.125)
    b = orc.decode_split(q, k, v, bt, ctx, 0.125, S)
    assert np.abs(a - b).max() < 1e-5


def test_empty_context_is_nan_like_v3():
    q, k, v, bt, ctx = orc.make_decode_case(6, B=2, H=2, HKV=2, D=32, BS=16, ctx=[0, 20])
    a = orc.decode(q, k, v, bt, ctx, 0.2)
    b = orc.decode_split(q, k, v, bt, ctx, 0.2, 4)
    assert np.isnan(a[0]).all() and np.isnan(b[0]).all()
    assert np.isfinite(a[1]).all()


def test_threads_do_not_change_results():
    q, k, v, bt, ctx = orc.make_decode_case(7, B=4, H=12, HKV=12, D=64, BS=16, ctx=300)
    assert np.array_equal(orc.decode(q, k, v, bt, ctx, 0.125, threads=1),
                          orc.decode(q, k, v, bt, ctx, 0.125, threads=5))


def test_prefill_causal_rule_and_padding():
    _, k, v, bt, ctx = orc.make_decode_case(8, B=2, H=2, HKV=1, D=32, BS=16, ctx=[5, 40])
    Sq = 8
    q = np.random.default_rng(0).standard_normal((2, Sq, 2, 32), dtype=np.float32)
    out = orc.prefill(q, k, v, bt, ctx, 0.3)
    # seq 0 has 5 tokens but 8 query slots: slots 0..2 see no key -> zeros
    assert np.all(out[0, :3] == 0)
    # each query row equals a decode of the same q over its causal prefix
    for b in range(2):
        for s in range(Sq):
            n = int(ctx[b]) - Sq + s + 1
            if n <= 0:
                continue
            d = orc.decode(q[b, s][None], k, v, bt[b][None], [n], 0.3)
            assert np.abs(d[0] - out[b, s]).max() < 1e-6


def test_write_kv_oracle_scatter():
    L, H, T, D, BS, NB = 2, 3, 21, 8, 4, 12
    rng = np.random.default_rng(1)
    k = rng.standard_normal((L, H, T, D), dtype=np.float32)
    v = rng.standard_normal((L, H, T, D), dtype=np.float32)
    pool = np.zeros((L, 2, NB, BS, H, D), np.uint32)
    ids = [7, 2, 9, 0, 5, 11, 3]
    start = 3
    orc.write_kv(pool, ids, start, k, v, "float32")
    for t in range(T):
        p = start + t
        for layer in range(L):
            got = pool[layer, 0, ids[p // BS], p % BS].view(np.float32)
            assert np.array_equal(got, k[layer, :, t, :])


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.0078125, 1.01171875, -2.5e-3, 3.0e38, np.inf], np.float32)
    bits = orc.f32_to_bf16_bits(x)
    # ties to even: 1 + 2^-8 -> 1.0 ; 1 + 3*2^-8 -> 1 + 2^-6
    assert orc.bf16_bits_to_f32(bits[1]) == 1.0
    assert orc.bf16_bits_to_f32(bits[3]) == np.float32(1.015625)
    assert np.isinf(orc.bf16_bits_to_f32(bits[6]))
