"""Benchmark logic of the reference harness: peak-bandwidth provenance, L2
size, cold KV pools and the traffic / flop models.

* ``peak_bandwidth`` restates ``harness/probe_arch.py:96-117``: prefer a vendor
  figure for known parts, else derive ``clock x bus / 8`` both without and
  with the DDR x2, and always return the provenance string beside the number
  (the reference's 2x-denominator bug, ``docs/REPORT.md:50-78``).  On B200 the
  driver-measured copy bandwidth (``MEASURED_PEAKS.json``) is the roofline
  denominator; the spec figure is reported beside it.
* ``cold_regions`` restates the ``--cold-pools N`` logic of hetero-serve's
  ``scripts/bench_kernel.py`` (un-vendored; semantics ``docs/REPORT.md:
  110-114``, output line ``results/c000-20260901-225701-verify/
  cold_b4_c2048.txt:11``): N disjoint block regions of one pool, block tables
  rotated across iterations so a region is evicted before it is read again;
  N = 0 sizes the rotation to a multiple of L2 (4x in the reference).
* ``decode_bytes`` is the algorithmic traffic of a decode: KV read once per KV
  head (``HKV``, not ``H`` as ``docs/REPORT.md:35-37`` wrote, which overcounts
  GQA), plus q, out and the block-table reads; ``reference_decode_bytes`` is
  the reference's own ``2*B*C*H*D*itemsize``.
"""
from __future__ import annotations

import json
import math
import os
from pathlib import Path

import numpy as np

# Published peak DRAM bandwidth (GB/s).  B200: 8 TB/s HBM3e (DGX figure;
# HGX lists 7.7); the other two are the reference's table (probe_arch.py:104).
KNOWN_PEAK_GBS = {"NVIDIA B200": 8000.0, "NVIDIA GB10": 273.0, "Tesla T4": 320.0}


def _measured_peaks() -> dict | None:
    for p in (Path(os.environ.get("PA_MEASURED_PEAKS", "")),
              Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"):
        if p and p.is_file():
            try:
                return json.loads(p.read_text())
            except (OSError, ValueError):
                return None
    return None


def peak_bandwidth(name: str, memory_clock_khz: int | None = None,
                   bus_width_bits: int | None = None) -> dict:
    """Peak DRAM bandwidth with provenance (GB/s)."""
    d: dict = {"device_name": name}
    if memory_clock_khz and bus_width_bits:
        d["peak_GBs_no_double"] = round(memory_clock_khz * 1e3 * bus_width_bits / 8 / 1e9, 1)
        d["peak_GBs_doubled"] = round(memory_clock_khz * 1e3 * 2 * bus_width_bits / 8 / 1e9, 1)
    known = KNOWN_PEAK_GBS.get(name)
    if known:
        d["peak_GBs_spec"] = known
        d["peak_GBs"] = known
        d["peak_GBs_source"] = "vendor spec"
    elif "peak_GBs_doubled" in d:
        d["peak_GBs"] = d["peak_GBs_doubled"]
        d["peak_GBs_source"] = ("derived, clock x2 -- UNVERIFIED; if this is 2x the spec sheet "
                                "the part reports an effective rate and needs a table entry")
    meas = _measured_peaks()
    if meas and meas.get("hbm_gbs") and (meas.get("gpu_name") == name or "B200" in name):
        d["peak_GBs_measured"] = float(meas["hbm_gbs"])
        d["peak_GBs"] = float(meas["hbm_gbs"])
        d["peak_GBs_source"] = "measured copy bandwidth (MEASURED_PEAKS.json: " + \
            str(meas.get("how", "copy_"))[:60] + ")"
    return d


def device_peak_bandwidth(device: int = 0) -> dict:
    import torch
    props = torch.cuda.get_device_properties(device)
    clk = getattr(props, "memory_clock_rate", None)
    bus = getattr(props, "memory_bus_width", None)
    return peak_bandwidth(props.name, clk, bus)


def l2_cache_bytes(device: int = 0) -> int:
    """L2 size from the driver (cudaDevAttrL2CacheSize via torch's props)."""
    import torch
    props = torch.cuda.get_device_properties(device)
    v = getattr(props, "L2_cache_size", 0) or getattr(props, "l2_cache_size", 0)
    if v:
        return int(v)
    for mod in ("cuda.bindings.runtime", "cuda.cudart"):
        try:
            import importlib
            rt = importlib.import_module(mod)
            err, val = rt.cudaDeviceGetAttribute(rt.cudaDeviceAttr.cudaDevAttrL2CacheSize, device)
            if int(err) == 0 and val:
                return int(val)
        except Exception:  # noqa: BLE001 - probe every binding
            continue
    raise RuntimeError("L2 cache size unavailable")


def cold_pool_count(region_bytes: int, l2_bytes: int, requested: int = 0,
                    factor: float = 4.0) -> int:
    """Number of disjoint regions to rotate through: ``requested`` if > 0,
    else enough that the rotation footprint is >= factor x L2."""
    if requested > 0:
        return requested
    return max(1, math.ceil(factor * l2_bytes / max(region_bytes, 1)))


def cold_regions(blocks_per_seq: list[int], n_regions: int, num_blocks: int,
                 seed: int = 0, max_blocks: int | None = None) -> list[np.ndarray]:
    """Block tables for n_regions disjoint block regions of one pool.

    Region r owns blocks [r*need, (r+1)*need) of a seeded permutation of the
    pool's blocks (need = sum of blocks_per_seq); its table gives sequence b
    the next blocks_per_seq[b] of them.  Returns one int32 [B, MB] array per
    region."""
    need = int(sum(blocks_per_seq))
    if need * n_regions > num_blocks:
        raise ValueError(f"{n_regions} regions of {need} blocks exceed the pool ({num_blocks})")
    rng = np.random.default_rng(seed)
    perm = rng.permutation(num_blocks).astype(np.int32)
    mb = max_blocks or max(max(blocks_per_seq), 1)
    out = []
    for r in range(n_regions):
        ids = perm[r * need:(r + 1) * need]
        bt = np.zeros((len(blocks_per_seq), mb), np.int32)
        cur = 0
        for b, n in enumerate(blocks_per_seq):
            bt[b, :n] = ids[cur:cur + n]
            bt[b, n:] = ids[cur] if n else 0
            cur += n
        out.append(bt)
    return out


def decode_bytes(context_lens, num_heads: int, num_kv_heads: int, head_dim: int,
                 itemsize: int, block_size: int) -> int:
    """Algorithmic bytes of one decode call: every cached K and V element once
    (per KV head), q and out in fp32, and the block-table entries used."""
    ctx = np.maximum(np.asarray(context_lens, np.int64), 0)
    B = len(ctx)
    kv = int(ctx.sum()) * 2 * num_kv_heads * head_dim * itemsize
    qo = 2 * B * num_heads * head_dim * 4
    bt = int(((ctx + block_size - 1) // block_size).sum()) * 4
    return kv + qo + bt


def reference_decode_bytes(batch: int, context: int, heads: int, head_dim: int,
                           itemsize: int) -> int:
    """The reference's traffic model: 2 * B * C * H * D * itemsize."""
    return 2 * batch * context * heads * head_dim * itemsize


def prefill_flops(context_lens, num_queries: int, num_heads: int, head_dim: int) -> int:
    """Causal prefill flops: 4*D per (query, visible key) per head (QK^T + PV)."""
    s = np.arange(num_queries, dtype=np.int64)
    total = 0
    for c in np.asarray(context_lens, np.int64):
        # query s sees keys [0, c - Sq + s]
        total += int(np.maximum(c - num_queries + s + 1, 0).sum())
    return 4 * head_dim * num_heads * total
