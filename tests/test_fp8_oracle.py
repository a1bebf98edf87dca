"""The oracle's FP8 E4M3 restatement (OCP 8-bit floating point, e4m3fn) on
CPU: known answers, round-to-nearest-even at every midpoint, saturation, and
agreement with torch's own float8_e4m3fn cast over a million values (the
reference has no FP8 pool, so torch's cast is the independent pin)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from pa_b200 import _lib


@pytest.mark.parametrize("x,bits", [
    (0.0, 0x00), (-0.0, 0x80), (1.0, 0x38), (-1.0, 0xB8), (448.0, 0x7E), (-448.0, 0xFE),
    (2.0 ** -9, 0x01), (7 * 2.0 ** -9, 0x07), (2.0 ** -6, 0x08), (3.25, 0x45),
    (1.0625, 0x38),     # tie between 1 and 1.125 -> even mantissa (1.0)
    (1.1875, 0x3A),     # tie between 1.125 and 1.25 -> 1.25
    (2.0 ** -10, 0x00),  # tie between 0 and the smallest subnormal -> 0
    (464.0, 0x7E), (1e6, 0x7E), (-1e6, 0xFE), (float("inf"), 0x7E),  # saturating
])
def test_known_answers(x, bits):
    assert int(orc.f32_to_e4m3_bits(np.float32(x)).reshape(-1)[0]) == bits


def test_every_value_round_trips_and_every_midpoint_rounds_to_even():
    b = np.arange(256, dtype=np.uint8)
    b = b[(b & 0x7F) != 0x7F]
    assert np.array_equal(orc.f32_to_e4m3_bits(orc.e4m3_bits_to_f32(b)), b)
    pos = orc.e4m3_bits_to_f32(np.arange(0x7F, dtype=np.uint8)).astype(np.float64)
    mid = ((pos[1:] + pos[:-1]) / 2).astype(np.float32)
    got = orc.f32_to_e4m3_bits(mid)
    lo = np.arange(0x7E, dtype=np.uint8)
    assert np.array_equal(got, np.where(lo % 2 == 0, lo, lo + 1))


def test_matches_torch_cast():
    rng = np.random.default_rng(0)
    y = (rng.standard_normal(1_000_000) * np.exp(rng.uniform(-14, 6.5, 1_000_000)))
    y = y.astype(np.float32)
    y = y[np.abs(y) <= 448]  # torch's cast does not saturate; the pool writer does
    want = torch.from_numpy(y).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(orc.f32_to_e4m3_bits(y), want)


def test_quantize_divides_in_fp32_first():
    x = np.float32(1.0) + np.float32(2.0 ** -20)
    s = np.float32(3.0)
    assert np.array_equal(orc.quantize_e4m3(x, s), orc.f32_to_e4m3_bits(np.float32(x / s)))


def test_fp8_entry_points_check_before_the_device():
    bad = _lib.PA_ERR_DTYPE
    # the FP8 decode wants an E4M3 pool
    assert _lib.call("pa_paged_attention_v3_fp8", None, None, None, None, None, None, None,
                     _lib.PA_DTYPE_F16, None, None, 4, 12, 12, 64, 16, 10, 4, 0.125, 0, None,
                     0, None, None) == bad
    # FP8 pools are decode-only: every prefill entry point refuses them
    n = ctypes.c_size_t(0)
    assert _lib.call("pa_prefill_workspace_size", 1, 4, 8, 8, 64, _lib.PA_DTYPE_E4M3, 16, 4,
                     ctypes.byref(n)) == bad
    for entry in ("pa_paged_attention_prefill", "pa_paged_attention_prefill_simt",
                  "pa_paged_attention_prefill_wmma"):
        assert _lib.call(entry, None, None, None, None, _lib.PA_DTYPE_E4M3, None, None, 1, 4,
                         8, 8, 64, 16, 10, 4, 0.125, None, 0, None, None) == bad
