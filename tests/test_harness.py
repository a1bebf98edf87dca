"""Benchmark logic: peak-bandwidth provenance, cold pools, traffic models (CPU)."""
from __future__ import annotations

import numpy as np
import pytest

from pa_b200 import harness


def test_peak_bandwidth_gb10_is_not_doubled():
    # probe_arch.py:96-117 / docs/REPORT.md:50-78: GB10 LPDDR5X reports the
    # effective rate; 8533 MT/s x 256 bit / 8 = 273 GB/s, doubling gives 546.
    d = harness.peak_bandwidth("NVIDIA GB10", 8_533_000, 256)
    assert d["peak_GBs_no_double"] == pytest.approx(273.1, abs=0.1)
    assert d["peak_GBs_doubled"] == pytest.approx(546.1, abs=0.1)
    assert d["peak_GBs"] == 273.0 and d["peak_GBs_source"] == "vendor spec"


def test_peak_bandwidth_t4_and_unknown():
    assert harness.peak_bandwidth("Tesla T4", 5_001_000, 256)["peak_GBs"] == 320.0
    d = harness.peak_bandwidth("Some GPU", 1_000_000, 512)
    assert d["peak_GBs"] == d["peak_GBs_doubled"] == 128.0
    assert "UNVERIFIED" in d["peak_GBs_source"]


def test_peak_bandwidth_b200_prefers_measured(tmp_path, monkeypatch):
    p = tmp_path / "peaks.json"
    p.write_text('{"hbm_gbs": 6452.5, "gpu_name": "NVIDIA B200", "how": "copy"}')
    monkeypatch.setenv("PA_MEASURED_PEAKS", str(p))
    d = harness.peak_bandwidth("NVIDIA B200", 3_996_000, 8192)
    assert d["peak_GBs"] == 6452.5 and d["peak_GBs_spec"] == 8000.0
    assert d["peak_GBs_source"].startswith("measured")


def test_cold_pool_count():
    l2 = 126 * 2**20
    assert harness.cold_pool_count(402_653_184, l2) == 2      # 4 x L2 / 403 MB
    assert harness.cold_pool_count(25_165_824, 24 * 2**20) == 4  # the reference's b=4 case
    assert harness.cold_pool_count(1, l2, requested=7) == 7


def test_cold_regions_are_disjoint_and_cover_needs():
    need = [3, 0, 5, 1]
    regs = harness.cold_regions(need, 4, 40, seed=3)
    seen = set()
    for bt in regs:
        ids = set()
        for b, n in enumerate(need):
            ids.update(bt[b, :n].tolist())
        assert len(ids) == sum(need)
        assert not (ids & seen)
        seen |= ids
    with pytest.raises(ValueError):
        harness.cold_regions(need, 5, 40)


def test_decode_bytes_config2_matches_reference_figure():
    # docs/REPORT.md:124: b=64 ctx=2048 gpt2 fp16 = 402.7 MB of K and V
    kv = harness.reference_decode_bytes(64, 2048, 12, 64, 2)
    assert kv == 402_653_184
    full = harness.decode_bytes([2048] * 64, 12, 12, 64, 2, 16)
    assert full == kv + 2 * 64 * 12 * 64 * 4 + 64 * 128 * 4


def test_decode_bytes_gqa_counts_kv_heads():
    a = harness.decode_bytes([100], 32, 8, 128, 2, 16)
    assert a == 100 * 2 * 8 * 128 * 2 + 2 * 32 * 128 * 4 + 7 * 4


def test_prefill_flops():
    # Sq == ctx: query s sees s+1 keys -> sum = Sq(Sq+1)/2
    f = harness.prefill_flops([4096] * 4, 4096, 32, 128)
    assert f == 4 * 128 * 32 * 4 * (4096 * 4097 // 2)
    # padded slots (Sq > ctx) contribute nothing
    assert harness.prefill_flops([2], 4, 1, 1) == 4 * (1 + 2)
