"""Benchmark: paged-attention decode, achieved HBM GB/s on cold pools.

Workload: GPT-2 geometry decode step, 12 layers,
H = HKV = 12, D = 64, block_size 16, batch 64, context 2048, fp16 KV pool,
synthetic N(0, 1) data.  A step = one decode token for every sequence through
all 12 layers (12 ``paged_attention_v3`` calls, one per layer's pool view).
Cold pools: 4 disjoint block regions of the pool, rotated step by step, so
each step reads 4.84 GB and the rotation spans 19.3 GB (L2 is 126 MB): every
KV byte comes from HBM.

value      kernel-only throughput: algorithmic bytes (KV once per KV head + q +
           out + block-table entries) / device time of the K timed steps,
           inputs resident in HBM, CUDA events, max over ranks.
e2e        the same metric through the public API (pa_b200.ops, the torch
           shim over the C ABI) with q in pinned HOST memory: each step copies
           q (and the step's block table) host->device and the outputs
           device->host inside the timed region.
roofline   the decode kernel: bytes per launch / launch time, against the
           measured copy bandwidth of this pool's B200s.
N > 1      one process per GPU (torchrun); each rank runs the same per-GPU
           workload (weak scaling, batch sharding: no collective on the data
           path); value = all ranks' bytes / slowest rank's time.

--workload config5 (torchrun) prints the multi-GPU
lines: the batch shard at 64 sequences x ctx 8192 per GPU, and one 1,048,576-
token GQA sequence split over the ranks with its partials merged over NVLink.

extra      (one GPU) the config-3 GQA decode, the config-4 prefill and its
           write_kv, and the configs[1] decode on an FP8 E4M3 pool, each as
           its own object with its roofline fraction; --workload config3 /
           config4 / fp8 run one of them alone (profiler captures).

--impl reference times the reference's scalar FP32 CPU decode (the oracle's
restatement of gb10-attn rocm/hip/paged_attn_v1_hip.cpp:104-141; the HIP file
itself does not build here) on the host cores, on a bounded sample of the
same workload, and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "gb10-attn_b200"))
sys.path.insert(0, str(REPO))

METRIC = "decode achieved HBM GB/s (% of B200 peak), cold pools; tokens/s at 1/2/4/8 GPUs"

# configs[1] geometry (layers / regions can be reduced for profiler captures)
H, HKV, D, BS, B, CTX = 12, 12, 64, 16, 64, 2048


def _env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


# the phase each rank is in, named in its error line if it fails
_STAGE = ["start"]


def _stage(name: str) -> None:
    _STAGE[0] = name


def _error_line(msg: str, impl: str) -> None:
    """One flushed JSON line on stdout from the failing rank (torchrun's
    summary on stderr would bury a message printed there)."""
    rank, _, world = _env_rank()
    print(json.dumps({"impl": impl, "error": msg[-2000:], "rank": rank, "world_size": world,
                      "where": _STAGE[0]}), flush=True)


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
        except (OSError, ValueError, KeyError):
            pass
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def _profile_traffic(kernel_key: str) -> float | None:
    """DRAM bytes per launch of a kernel from its committed ncu summary (a
    line 'traffic_bytes_per_launch: N' in profiles/<kernel_key>.md): ncu
    cannot run inside the timed process, so the figure comes from the capture
    of the same build, and the line names that file beside it."""
    return _profile_value(kernel_key, "traffic_bytes_per_launch")


def _profile_value(kernel_key: str, key: str) -> float | None:
    p = REPO / "profiles" / f"{kernel_key}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t = None
        self.window = [0.0, None]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.idx), "-lms", "20"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        self.window = [time.monotonic(), None]
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def __exit__(self, *exc):
        self.window[1] = time.monotonic()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.t:
                self.t.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # only the samples taken inside the `with` body (the start-up pre-roll is idle)
        t0, t1 = self.window if self.window[1] is not None else (self.window[0], float("inf"))
        for ts, line in self.lines:
            if not t0 <= ts <= t1:
                continue
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------

def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from pa_b200 import harness, ops

    L, REGIONS = args.layers, args.regions
    rank, local, world = _env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _stage("init_process_group")
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    _stage("pools")

    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    nb = B * (CTX // BS) * REGIONS  # 32768 blocks per layer pool with 4 regions
    # one [2, NB, BS, HKV, D] tensor per layer (the reference's per-layer pool)
    pools = []
    for _ in range(L):
        t = torch.empty((2, nb, BS, HKV, D), dtype=torch.float16, device=dev)
        t.normal_(generator=gen)
        pools.append(t)
    q_dev = torch.randn((L, B, H, D), generator=gen, device=dev, dtype=torch.float32)
    ctx_np = np.full(B, CTX, np.int32)
    tables = harness.cold_regions([CTX // BS] * B, REGIONS, nb, seed=rank)
    bt_dev = [torch.from_numpy(t).to(dev) for t in tables]
    ctx_dev = torch.from_numpy(ctx_np).to(dev)
    scale = D ** -0.5
    # each call returns its own output tensor; keeping references (not copying
    # into one buffer) leaves nothing but decode kernels on the stream
    outs = [None] * L
    stream = torch.cuda.current_stream()

    bytes_per_call = harness.decode_bytes(ctx_np, H, HKV, D, 2, BS)
    bytes_per_step = L * bytes_per_call

    def layer_call(layer: int, q, bt, ctx):
        return ops.paged_attention_v3(q, pools[layer][0], pools[layer][1], bt, ctx, scale, 0)

    def step(i: int):
        bt = bt_dev[i % REGIONS]
        for layer in range(L):
            outs[layer] = layer_call(layer, q_dev[layer], bt, ctx_dev)

    _stage("correctness_gate")
    ref_err = correctness_gate(torch, layer_call, pools[0], q_dev[0], tables[0], bt_dev[0],
                               ctx_dev, scale, dev)
    if ref_err > 2e-3:
        raise SystemExit(f"correctness gate failed: max-abs {ref_err}")

    _stage("warmup")
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    _stage("timed")

    # --- kernel-only timed region -----------------------------------------
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_ms = ev0.elapsed_time(ev1)

    # --- per-launch decode time (same stream, events around each call) -----
    _stage("launch_timing")
    n_launch = min(L * 4, max(L * args.steps, 4))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_launch)]
    torch.cuda.synchronize()
    for j, (a, b_) in enumerate(evs):
        layer = j % L
        a.record(stream)
        outs[layer] = layer_call(layer, q_dev[layer], bt_dev[(j // L) % REGIONS], ctx_dev)
        b_.record(stream)
    torch.cuda.synchronize()
    launch_ms = statistics.mean(a.elapsed_time(b_) for a, b_ in evs)

    # --- end to end through the public API with host buffers ---------------
    _stage("e2e")
    if args.no_e2e:
        e2e_ms, h2d, d2h = float("nan"), 0, 0
    else:
        e2e_ms, h2d, d2h = run_e2e(torch, dist, args, layer_call, q_dev, tables, ctx_np, dev,
                                   stream, world, L, REGIONS)

    # max over ranks
    _stage("max_over_ranks")
    times = torch.tensor([t_ms, e2e_ms, launch_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, launch_ms = (float(x) for x in times.cpu())

    total_bytes = bytes_per_step * args.steps * world
    value = total_bytes / (t_ms * 1e-3) / 1e9
    e2e_val = total_bytes / (e2e_ms * 1e-3) / 1e9 if e2e_ms == e2e_ms else None
    peaks = _peaks()
    # decode-kernel roofline: bytes of one layer call / mean call time over the
    # timed region (events on the launching stream).  With B <= 1024 rows the
    # plan is built inside the decode kernel, so a call is one launch.
    call_ms = t_ms / (args.steps * L)
    achieved = bytes_per_call / (call_ms * 1e-3) / 1e9
    traffic = _profile_traffic("decode_kernel_config2")
    clk = clocks.summary()

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic N(0,1) KV pool and q, seeded",
        "config": {"workload": f"configs[1]: gpt2 paged decode, {L} layers, B=64/GPU, ctx=2048, "
                               "H=HKV=12, D=64, block_size=16, fp16 KV, fp32 q/out",
                   "global_batch": B * world, "seq_len": CTX, "layers": L,
                   "parallelism": f"batch-sharded x{world} (no collective)",
                   "cold": f"{REGIONS} disjoint block regions rotated per step; inputs larger "
                           f"than L2 ({bytes_per_step / 1e9:.2f} GB/step, "
                           f"{REGIONS * bytes_per_step / 1e9:.1f} GB rotation)",
                   "tokens_per_s": round(B * world * args.steps / (t_ms * 1e-3), 1),
                   "pct_of_measured_hbm_peak": round(100 * value / world / peaks["hbm_gbs"], 1),
                   "pct_of_spec_8TBs": round(100 * value / world / 8000.0, 1),
                   "correctness_gate_max_abs": ref_err},
        "e2e": {"value": round(e2e_val, 1) if e2e_val else None, "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "tokens_per_s": round(B * world * args.steps / (e2e_ms * 1e-3), 1)
                if e2e_val else None},
        "gpu_launches": (1 if B <= 1024 else 2) * L * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                       "profiles/decode_kernel_config2.md",
                     "peak_source": peaks["src"],
                     "kernel": "pa::decode::decode_kernel<__half,64,1> (plan built in-kernel)",
                     "bytes_per_launch": bytes_per_call,
                     "launch_us": round(call_ms * 1e3, 2),
                     "isolated_launch_us": round(launch_ms * 1e3, 2)},
        "clocks": clk,
    }
    if world == 1 and not args.no_extra:
        del pools, outs
        torch.cuda.empty_cache()
        _stage("extra")
        line["extra"] = {"config3_gqa_long_context": run_config3(torch, ops, harness, dev,
                                                                 stream, args, peaks),
                         "config4_prefill": run_config4(torch, ops, harness, dev, stream, args),
                         "fp8_kv_config2_geometry": run_fp8(torch, ops, harness, dev, stream,
                                                            args, peaks)}
        fp8 = line["extra"]["fp8_kv_config2_geometry"]
        fp8["tokens_per_s_vs_fp16_line"] = round(
            fp8["tokens_per_s"] / line["config"]["tokens_per_s"], 3)
    if world > 1 and not args.no_extra:
        # BASELINE.json configs[4] on the same ranks: the batch shard at
        # ctx 8192 and the 1 M-token sequence shard with its exchange
        del pools, outs
        torch.cuda.empty_cache()
        line["extra"] = {"config5_multi_gpu": measure_config5(torch, dist, args, rank, world,
                                                              dev, peaks)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        _stage("cpu_baseline")
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_config3(torch, ops, harness, dev, stream, args, peaks) -> dict:
    """bf16 GQA long-context decode, 32 query / 8 KV
    heads, D=128, block_size 16, B=8, ctx ~ U[1024, 32768] (seeded), one K and
    one V tensor of [140000, 16, 8, 128] = 2.29e9 elements each (> 2^31), the
    blocks used drawn from the top of the pool so every offset crosses 2^31.
    4 disjoint regions rotated per call (each call reads ~0.55 GB)."""
    H3, HKV3, D3, BS3, B3, NB3, REG = 32, 8, 128, 16, 8, args.pool_blocks, 4
    rng = np.random.default_rng(2026)
    ctx = rng.integers(1024, 32769, size=B3).astype(np.int32)
    need = [int(-(-c // BS3)) for c in ctx]
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    kv = torch.empty((2, NB3, BS3, HKV3, D3), dtype=torch.bfloat16, device=dev)
    kv.normal_(generator=gen)
    top = NB3 - REG * sum(need)          # regions live in the top of the pool
    tables = [t + top for t in harness.cold_regions(need, REG, REG * sum(need), seed=7)]
    bt = [torch.from_numpy(t.astype(np.int32)).to(dev) for t in tables]
    ctx_d = torch.from_numpy(ctx).to(dev)
    q = torch.randn((B3, H3, D3), generator=gen, device=dev)
    scale = D3 ** -0.5

    def call(i):
        return ops.paged_attention_v3(q, kv[0], kv[1], bt[i % REG], ctx_d, scale, 0)

    # gate: two sequences against a dense fp32 reference
    got = call(0)
    err = 0.0
    for b in (0, B3 - 1):
        blocks = torch.from_numpy(tables[0][b, :need[b]].astype(np.int64)).to(dev)
        kk = kv[0][blocks].float().reshape(-1, HKV3, D3)[:ctx[b]]
        vv = kv[1][blocks].float().reshape(-1, HKV3, D3)[:ctx[b]]
        kk = kk.repeat_interleave(H3 // HKV3, dim=1)
        vv = vv.repeat_interleave(H3 // HKV3, dim=1)
        sc = torch.einsum("hd,thd->ht", q[b], kk) * scale
        want = torch.einsum("ht,thd->hd", torch.softmax(sc, -1), vv)
        err = max(err, float((got[b] - want).abs().max()))
        del kk, vv
    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    n = max(50, args.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n):
        call(i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    per_call = harness.decode_bytes(ctx, H3, HKV3, D3, 2, BS3)
    gbs = per_call / (ms * 1e-3) / 1e9
    del kv
    torch.cuda.empty_cache()
    return {"value": round(gbs, 1), "unit": "GB/s",
            "pct_of_measured_hbm_peak": round(100 * gbs / peaks["hbm_gbs"], 1),
            "traffic_bytes_per_launch": _profile_traffic("decode_kernel_config3"),
            "traffic_source": "profiles/decode_kernel_config3.md",
            "us_per_call": round(ms * 1e3, 2), "bytes_per_call": per_call,
            "calls": n, "context_lens": ctx.tolist(), "pool_elements_per_tensor": NB3 * BS3 * HKV3 * D3,
            "tokens_per_s": round(B3 / (ms * 1e-3), 1), "correctness_gate_max_abs": err,
            "kernel": "pa::decode::decode_kernel<__nv_bfloat16,128,4> (warp-specialised)"}


def run_fp8(torch, ops, harness, dev, stream, args, peaks) -> dict:
    """The config-2 decode (gpt2, B=64, ctx 2048, 12 layers, 4 cold regions)
    on an FP8 E4M3 pool with per-KV-head scales (paged_attention_v3_fp8): half
    the K/V bytes of the fp16 line.  An addition beyond the reference; timed
    like the headline (device events around the whole loop)."""
    L, REG = args.layers, args.regions
    nb = B * (CTX // BS) * REG
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321)
    pools, scales = [], []
    for _ in range(L):
        t = torch.empty((2, nb, BS, HKV, D), dtype=torch.float16, device=dev)
        t.normal_(generator=gen)
        pools.append(t.to(torch.float8_e4m3fn))
        del t
        scales.append(torch.rand((2, HKV), generator=gen, device=dev) * 0.02 + 0.01)
    q = torch.randn((L, B, H, D), generator=gen, device=dev)
    ctx = np.full(B, CTX, np.int32)
    tables = harness.cold_regions([CTX // BS] * B, REG, nb, seed=11)
    bt = [torch.from_numpy(t).to(dev) for t in tables]
    ctx_d = torch.from_numpy(ctx).to(dev)
    scale = D ** -0.5
    outs = [None] * L

    def call(layer, i):
        return ops.paged_attention_v3_fp8(q[layer], pools[layer][0], pools[layer][1],
                                          bt[i % REG], ctx_d, scale, scales[layer][0],
                                          scales[layer][1], 0)[0]

    # gate: two sequences of layer 0 against dense fp32 on the dequantised pool
    got = call(0, 0)
    err = 0.0
    for b in (0, B - 1):
        blocks = torch.from_numpy(tables[0][b].astype(np.int64)).to(dev)
        kk = pools[0][0][blocks].float().reshape(-1, HKV, D) * scales[0][0][None, :, None]
        vv = pools[0][1][blocks].float().reshape(-1, HKV, D) * scales[0][1][None, :, None]
        sc = torch.einsum("hd,thd->ht", q[0, b], kk) * scale
        want = torch.einsum("ht,thd->hd", torch.softmax(sc, -1), vv)
        err = max(err, float((got[b] - want).abs().max()))
    if err > 2e-3:
        raise SystemExit(f"fp8 correctness gate failed: max-abs {err}")

    def step(i):
        for layer in range(L):
            outs[layer] = call(layer, i)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    n = max(20, args.steps // 4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    per_call = harness.decode_bytes(ctx, H, HKV, D, 1, BS)
    gbs = L * per_call / (ms * 1e-3) / 1e9
    del pools, outs
    torch.cuda.empty_cache()
    return {"value": round(gbs, 1), "unit": "GB/s",
            "pct_of_measured_hbm_peak": round(100 * gbs / peaks["hbm_gbs"], 1),
            "ms_per_step": round(ms, 4), "bytes_per_call": per_call, "steps": n,
            "tokens_per_s": round(B / (ms * 1e-3), 1), "correctness_gate_max_abs": err,
            "config": f"configs[1] geometry on an e4m3 pool, {L} layers, {REG} cold regions, "
                      "per-KV-head scales",
            "kernel": "pa::decode::decode_kernel<__nv_fp8_e4m3,64,1> (light CTA, 32-token stages)"}


def correctness_gate(torch, layer_call, pool, q, bt_np, bt_dev, ctx_dev, scale, dev) -> float:
    """The reference's bench checks each path before timing it
    (docs/REPORT.md:41-43): here the full B=64 layer-0 call against a dense
    torch fp32 gather + softmax reference."""
    got = layer_call(0, q, bt_dev, ctx_dev)
    blocks = torch.from_numpy(bt_np[:, :CTX // BS].astype(np.int64)).to(dev)
    err = 0.0
    for b0 in range(0, B, 8):
        idx = blocks[b0:b0 + 8].reshape(-1)
        kk = pool[0][idx].float().reshape(-1, CTX, HKV, D)
        vv = pool[1][idx].float().reshape(-1, CTX, HKV, D)
        s = torch.einsum("bhd,bthd->bht", q[b0:b0 + 8], kk) * scale
        want = torch.einsum("bht,bthd->bhd", torch.softmax(s, -1), vv)
        err = max(err, float((got[b0:b0 + 8] - want).abs().max()))
    return err


def run_e2e(torch, dist, args, layer_call, q_dev, tables, ctx_np, dev, stream, world, L,
            REGIONS):
    """Same decode steps through the public API with host buffers, as a serving
    loop runs them: every step copies its q (all layers), block table and
    context lengths from pinned host memory to the device and reads every
    layer's output back to pinned host memory, all inside the timed region.
    The copies go on a side stream, pipelined by one step: step i+1's inputs
    travel (into the other of two device input slots) while step i computes,
    and step i's outputs are read back once its last layer is done.  A step's
    12 layer kernels follow each other with no event between them, so each
    launch overlaps the previous one's tail (programmatic dependent launch)."""
    q_host = torch.empty(tuple(q_dev.shape), dtype=torch.float32).pin_memory()
    q_host.copy_(q_dev.cpu())
    bt_host = [torch.from_numpy(t).pin_memory() for t in tables]
    ctx_host = torch.from_numpy(ctx_np).pin_memory()
    out_host = torch.empty(tuple(q_dev.shape), dtype=torch.float32).pin_memory()
    qd = [torch.empty_like(q_dev) for _ in range(2)]
    btd = [torch.empty(tuple(tables[0].shape), dtype=torch.int32, device=dev) for _ in range(2)]
    cd = [torch.empty(len(ctx_np), dtype=torch.int32, device=dev) for _ in range(2)]
    copy = torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_step = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    held = [[], []]  # each slot's outputs, alive until their read-back is done

    def upload(i: int):
        """Step i's inputs into slot i % 2, on the copy stream."""
        s = i % 2
        with torch.cuda.stream(copy):
            btd[s].copy_(bt_host[i % REGIONS], non_blocking=True)
            cd[s].copy_(ctx_host, non_blocking=True)
            qd[s].copy_(q_host, non_blocking=True)
            ev_in[s].record(copy)

    def e2e_step(i: int, last: bool):
        s = i % 2
        # step i-2's outputs are released once the compute stream has waited
        # for their read-back (stream-ordered reuse, no allocator sync)
        stream.wait_event(d2h_done[s])
        held[s].clear()
        stream.wait_event(ev_in[s])
        if not last:
            # the other slot is free once step i-1's kernels are done with it
            copy.wait_event(ev_step[1 - s])
            upload(i + 1)
        for layer in range(L):
            held[s].append(layer_call(layer, qd[s][layer], btd[s], cd[s]))
        ev_step[s].record(stream)
        with torch.cuda.stream(copy):
            copy.wait_event(ev_step[s])
            for layer in range(L):
                out_host[layer].copy_(held[s][layer], non_blocking=True)
            d2h_done[s].record(copy)

    n_warm = max(2, args.warmup)
    upload(0)
    for i in range(n_warm):
        e2e_step(i, i + 1 == n_warm)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    done = torch.cuda.Event()
    e0.record(stream)
    copy.wait_event(e0)  # no copy of the timed steps starts before e0
    upload(0)
    for i in range(args.steps):
        e2e_step(i, i + 1 == args.steps)
    done.record(copy)
    stream.wait_event(done)  # the last read-back is inside the timed region
    e1.record(stream)
    torch.cuda.synchronize()
    # the pipelined loop must read back what a plain call computes
    s = (args.steps - 1) % 2
    want = layer_call(L - 1, qd[s][L - 1], btd[s], cd[s]).cpu()
    if not torch.equal(out_host[L - 1], want):
        diff = float((out_host[L - 1] - want).abs().nan_to_num(float("inf")).max())
        raise SystemExit(f"e2e read-back differs from a direct call (max-abs {diff:.3e}; "
                         "the decode is bit-deterministic, so any difference is an ordering "
                         "error)")
    h2d = q_host.numel() * 4 + bt_host[0].numel() * 4 + ctx_host.numel() * 4
    d2h = out_host.numel() * 4
    return e0.elapsed_time(e1), h2d, d2h


# ---------------------------------------------------------------------------
# the CPU reference arm / baseline
# ---------------------------------------------------------------------------

_CPU_CASE: list = []


def _cpu_case():
    """The config-2 layer inputs for the CPU timings, made once: N(0,1) q
    and fp16-representable K/V (fp32 arrays), a seeded permutation of the
    4096 pages as block table.  torch's CPU generator (multi-threaded) makes
    the 200 M values in a fraction of numpy's time; the values do not affect
    the timing."""
    if not _CPU_CASE:
        import torch
        g = torch.Generator().manual_seed(7)
        nb = B * CTX // BS
        q = torch.randn((B, H, D), generator=g).numpy()
        k = torch.randn((nb, BS, HKV, D), generator=g).half().float().numpy()
        v = torch.randn((nb, BS, HKV, D), generator=g).half().float().numpy()
        bt = np.random.default_rng(7).permutation(nb).astype(np.int32).reshape(B, CTX // BS)
        _CPU_CASE.append((q, k, v, bt, np.full(B, CTX, np.int32)))
    return _CPU_CASE[0]


def cpu_sample(seconds: float, threads: int):
    """Times the oracle restatement of the reference's scalar FP32 CPU decode
    on layer calls of the config-2 workload (fp16 values upcast to fp32, as
    the reference's CPU path computes in fp32) until `seconds` have passed.
    Returns (GB/s by the same algorithmic-bytes model, calls, sample text)."""
    from oracle import oracle as orc
    from pa_b200 import harness

    q, k, v, bt, ctx = _cpu_case()
    orc.decode(q[:1], k, v, bt[:1], ctx[:1], D ** -0.5, threads=1)  # warm
    per_call = harness.decode_bytes(ctx, H, HKV, D, 2, BS)
    n, t0 = 0, time.perf_counter()
    while True:
        orc.decode(q, k, v, bt, ctx, D ** -0.5, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = n * per_call / el / 1e9
    sample = (f"{n} full layer calls (B=64, ctx=2048, H=12, D=64) of the config-2 workload, "
              f"{el:.1f} s, {threads} threads")
    return gbs, n, sample


def simd_note() -> str:
    """The reference's SIMD CPU lane (arm_cpu, NEON / SVE) runs on aarch64
    hosts only; its own dispatcher refuses other ISAs."""
    import platform
    isa = platform.machine()
    if isa in ("aarch64", "arm64"):
        return f"not timed: host ISA is {isa}, but only the scalar lane is built here"
    return f"unavailable: host ISA is {isa} (the reference's SIMD lane is aarch64 NEON/SVE)"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or platform.machine()


def arm_bench_scalar() -> dict:
    """The reference's own CPU microbenchmark, arm_cpu's arm_attn_bench
    (built from its sources into oracle/_ref/ by oracle/build_ref.py): scalar
    scores + softmax of one 2048-token, 64-dim head (no V, no paging)."""
    exe = REPO / "oracle" / "_ref" / "arm_attn_bench"
    cmd = ["--backend", "scalar", "--tokens", "2048", "--dim", "64", "--csv"]
    if not exe.exists():
        return {"unavailable": "oracle/_ref/arm_attn_bench was not built (reference sources "
                               "absent at build time)"}
    try:
        r = subprocess.run([str(exe), *cmd], capture_output=True, text=True, timeout=120)
    except (OSError, subprocess.TimeoutExpired) as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}
    lines = [x for x in r.stdout.splitlines() if x.strip()]
    if r.returncode != 0 or len(lines) < 2:
        return {"unavailable": f"exit {r.returncode}: {r.stderr.strip()[-200:]}"}
    row = dict(zip(lines[0].split(","), lines[1].split(",")))
    return {"command": "arm_attn_bench " + " ".join(cmd), "backend": row.get("backend"),
            "effective_key_gbs": float(row["effective_key_gbs"]),
            "ns_per_dot": float(row["ns_per_dot"]), "gflops": float(row["gflops"]),
            "seconds": float(row["seconds"]), "iters": int(row["iters"]), "threads": 1}


def cpu_baseline(seconds: float) -> dict:
    """The reference's scalar FP32 CPU decode (the oracle's restatement) on
    the config-2 workload, single-threaded as the reference runs it and on
    every host thread (one (sequence, head) per task), plus the reference's
    own arm_attn_bench scalar run; about `seconds` of CPU work in all."""
    threads = os.cpu_count() or 1
    gbs1, _, sample1 = cpu_sample(seconds / 2, 1)
    gbs, _, sample = cpu_sample(seconds / 2, threads)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": sample, "threads": threads, "cpu_model": cpu_model(),
            "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "sample": sample1},
            "arm_attn_bench_scalar": arm_bench_scalar(), "simd": simd_note()}


def run_config4(torch, ops, harness, dev, stream, args) -> dict:
    """bf16 causal prefill, B=4, Sq = ctx = 4096,
    32 heads (MHA), D=128, block_size 16, K/V written into the paged pool by
    write_kv (timed too), q fp32 per the reference signature.  Tensor roofline:
    algorithmic flops 4*D per (query, visible key) per head."""
    from pa_b200.kv import KVConfig, ModelConfig, TorchBlockAllocator
    B4, S4, H4, D4, BS4 = 4, 4096, 32, 128, 16
    alloc = TorchBlockAllocator(KVConfig(BS4, B4 * S4 // BS4 + 8, "bfloat16"),
                                ModelConfig(n_layer=1, n_head=H4, head_dim=D4), dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    allocs = [alloc.allocate(range(S4)) for _ in range(B4)]
    ks = [torch.randn((1, H4, S4, D4), generator=gen, device=dev) for _ in range(B4)]
    vs = [torch.randn((1, H4, S4, D4), generator=gen, device=dev) for _ in range(B4)]
    for a, kk, vv in zip(allocs, ks, vs):  # warm-up pass (also fills the pool)
        alloc.write_kv(a.block_ids, 0, kk, vv)
    id_lists = [a.block_ids for a in allocs]
    alloc.write_kv_batch(id_lists, [0] * B4, ks, vs)
    torch.cuda.synchronize()
    reps = 5
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    for _ in range(reps):  # the reference's call: one write_kv per sequence
        for a, kk, vv in zip(allocs, ks, vs):
            alloc.write_kv(a.block_ids, 0, kk, vv)
    w1.record(stream)
    torch.cuda.synchronize()
    wkv_seq_ms = w0.elapsed_time(w1) / reps
    w0.record(stream)
    for _ in range(reps):  # all four sequences in one call
        alloc.write_kv_batch(id_lists, [0] * B4, ks, vs)
    w1.record(stream)
    torch.cuda.synchronize()
    wkv_ms = w0.elapsed_time(w1) / reps
    wkv_bytes = B4 * 2 * H4 * S4 * D4 * (4 + 2)  # fp32 read + bf16 write
    kc, vc = alloc.layer_kv(0)
    bt = alloc.block_table(allocs)
    ctx = torch.full((B4,), S4, dtype=torch.int32, device=dev)
    q = torch.randn((B4, S4, H4, D4), generator=gen, device=dev)
    scale = D4 ** -0.5

    def call():
        return ops.paged_attention_prefill(q, kc, vc, bt, ctx, scale)

    out = call()
    # gate: sequence 0, head 0, all 4096 rows, dense fp32 causal reference
    kk = ks[0][0, 0].to(torch.bfloat16).float()
    vv = vs[0][0, 0].to(torch.bfloat16).float()
    sc = (q[0, :, 0] @ kk.T) * scale
    sc = sc.masked_fill(torch.triu(torch.ones(S4, S4, dtype=torch.bool, device=dev), 1),
                        float("-inf"))
    want = torch.softmax(sc, -1) @ vv
    err = float((out[0, :, 0] - want).abs().max())
    del kk, vv, sc, want, ks, vs
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    n = max(250, args.steps // 2)  # ~0.35 s: long enough for a few dozen clock samples
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        e0.record(stream)
        for _ in range(n):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    flops = harness.prefill_flops([S4] * B4, S4, H4, D4)
    tflops = flops / (ms * 1e-3) / 1e12
    peak = _peak_tflops()
    return {"value": round(tflops, 1), "unit": "TFLOP/s",
            "pct_of_measured_bf16_peak": round(100 * tflops / peak["bf16_tflops"], 1),
            "pct_of_measured_bf16_sustained_peak": round(100 * tflops / peak["bf16_sustained"], 1)
            if peak.get("bf16_sustained") else None,
            "peak_source": peak["src"], "ms_per_call": round(ms, 4), "flops_per_call": flops,
            "calls": n, "correctness_gate_max_abs": err,
            "clocks": clocks.summary(),
            "tensor_pipe_active_pct": _profile_value("prefill_pair_config4", "tensor_pipe_active_pct"),
            "tensor_pipe_source": "ncu sm__pipe_tensor_cycles_active, profiles/prefill_pair_config4.md",
            "traffic_bytes_per_launch": _profile_traffic("prefill_pair_config4"),
            "kernel": "pa::prefill::prefill_pair_kernel<__nv_bfloat16> (tcgen05 cta_group::2 "
                      "CTA pairs, bf16 hi/lo)",
            "write_kv": {"value": round(wkv_bytes / (wkv_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                         "pct_of_measured_hbm_peak": round(100 * wkv_bytes / (wkv_ms * 1e-3) / 1e9
                                                           / _peaks()["hbm_gbs"], 1),
                         "bytes": wkv_bytes, "ms": round(wkv_ms, 3),
                         "note": "4 sequences x 4096 tokens x 32 heads, fp32 device source, "
                                 "through TorchBlockAllocator.write_kv_batch (one launch), "
                                 "mean of 5 passes after one",
                         "per_sequence_calls": {
                             "value": round(wkv_bytes / (wkv_seq_ms * 1e-3) / 1e9, 1),
                             "unit": "GB/s", "ms": round(wkv_seq_ms, 3),
                             "note": "the reference's form: four TorchBlockAllocator.write_kv "
                                     "calls"},
                         "kernel_traffic_bytes_per_launch": _profile_value(
                             "write_kv_config4", "batch_traffic_bytes_per_launch"),
                         "traffic_source": "profiles/write_kv_config4.md (the batched launch)"}}


def _peak_tflops() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"bf16_tflops": float(d["bf16_tflops"]),
                    "bf16_sustained": float(d.get("bf16_tflops_sustained", 0)) or None,
                    "src": "measured (burst; sustained beside it)"}
        except (OSError, ValueError, KeyError):
            pass
    return {"bf16_tflops": 1590.0, "src": "fallback"}


def run_config4_only(args) -> None:
    """--workload config4: the causal prefill alone (profiling)."""
    import torch

    from pa_b200 import harness, ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = run_config4(torch, ops, harness, dev, torch.cuda.current_stream(), args)
    print(json.dumps({"metric": "causal prefill TFLOP/s", "value": r["value"], "unit": "TFLOP/s",
                      "n_gpus": 1, "workload": "configs[3]", "detail": r}), flush=True)


def run_config3_only(args) -> None:
    """--workload config3: the GQA long-context decode alone (profiler target)."""
    import torch

    from pa_b200 import harness, ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = run_config3(torch, ops, harness, dev, torch.cuda.current_stream(), args, _peaks())
    print(json.dumps({"metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": 1,
                      "workload": "configs[2]", "detail": r}), flush=True)


def run_fp8_only(args) -> None:
    """--workload fp8: the FP8-pool decode at configs[1] geometry alone."""
    import torch

    from pa_b200 import harness, ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = run_fp8(torch, ops, harness, dev, torch.cuda.current_stream(), args, _peaks())
    print(json.dumps({"metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": 1,
                      "workload": "configs[1] geometry, e4m3 pool", "detail": r}), flush=True)


def run_config5(args) -> None:
    """--workload config5: the configs[4] lines alone (torchrun)."""
    import datetime

    import torch
    import torch.distributed as dist

    rank, local, world = _env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _stage("init_process_group")
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    r = measure_config5(torch, dist, args, rank, world, dev, _peaks())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line = {"metric": METRIC, "workload": "configs[4]", "n_gpus": world,
                "value": r["batch_shard"]["value"], "unit": "GB/s", "steps": args.steps,
                "warmup": args.warmup, "scaling": "weak", "higher_is_better": True,
                "data": "synthetic N(0,1) KV pools and q, seeded", **r}
        print(json.dumps(line), flush=True)


def measure_config5(torch, dist, args, rank, world, dev, peaks) -> dict:
    """BASELINE.json configs[4], one process per GPU, called on every rank
    (the process group, if world > 1, is the caller's).  (A) batch shard:
    gpt2 fp16 decode, 64 sequences of ctx 8192 per GPU, `--layers` layer pools
    with 2 cold regions, no collective; (B) one sequence of 1,048,576 tokens,
    32 query / 8 KV heads, D=128, bf16, its token range split evenly over the
    ranks: each decodes its range into its exchange buffer and one launch
    merges the ranks' partials over peer memory (pa_b200.dist.PeerMerge); the
    NCCL all-gather variant (sequence_sharded_decode) and the decode alone are
    timed beside it.  Times are the max over ranks; the B output is checked
    against per-rank dense fp32 partials merged with the same rule.  Returns
    the result object (the same on every rank)."""
    from pa_b200 import dist as padist
    from pa_b200 import harness, ops

    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev)
    gen.manual_seed(5000 + rank)

    def max_over_ranks(ms: float) -> float:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, n: int) -> float:
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1))

    # (A) batch shard ------------------------------------------------------
    _stage("config5.batch_shard")
    BA, CTXA, RA, LA = 64, 8192, 2, args.layers
    nb = BA * (CTXA // BS) * RA
    pools = []
    for _ in range(LA):
        t = torch.empty((2, nb, BS, HKV, D), dtype=torch.float16, device=dev)
        t.normal_(generator=gen)
        pools.append(t)
    qa = torch.randn((LA, BA, H, D), generator=gen, device=dev)
    ctxa = np.full(BA, CTXA, np.int32)
    bta = [torch.from_numpy(t).to(dev) for t in harness.cold_regions([CTXA // BS] * BA, RA, nb,
                                                                        seed=rank)]
    ctxa_d = torch.from_numpy(ctxa).to(dev)
    outs = [None] * LA

    def step_a(i: int):
        for layer in range(LA):
            outs[layer] = ops.paged_attention_v3(qa[layer], pools[layer][0], pools[layer][1],
                                                 bta[i % RA], ctxa_d, D ** -0.5, 0)

    ms_a = timed(step_a, args.steps)
    bytes_a = LA * harness.decode_bytes(ctxa, H, HKV, D, 2, BS) * world * args.steps
    gbs_a = bytes_a / (ms_a * 1e-3) / 1e9
    del pools, outs, qa
    torch.cuda.empty_cache()

    # (B) one long sequence over the ranks ----------------------------------
    _stage("config5.sequence_shard")
    NT, H5, HKV5, D5, R5 = 1 << 20, 32, 8, 128, 2
    nt = NT // world  # this rank's token range [rank * nt, (rank + 1) * nt)
    need = nt // BS
    kv = torch.empty((2, R5 * need, BS, HKV5, D5), dtype=torch.bfloat16, device=dev)
    kv.normal_(generator=gen)
    perm = np.random.default_rng(77 + rank).permutation(R5 * need).astype(np.int32)
    btb = [torch.from_numpy(perm[r * need:(r + 1) * need].reshape(1, need).copy()).to(dev)
           for r in range(R5)]
    ctxb = torch.tensor([nt], dtype=torch.int32, device=dev)
    qgen = torch.Generator(device=dev)
    qgen.manual_seed(55)  # the same q on every rank
    qb = torch.randn((1, H5, D5), generator=qgen, device=dev)
    scale5 = D5 ** -0.5
    group = dist.group.WORLD if world > 1 else None

    pm = padist.PeerMerge(1, H5, D5) if world > 1 else None

    def decode_b(i: int):
        if world == 1:
            return ops.paged_attention_v3(qb, kv[0], kv[1], btb[i % R5], ctxb, scale5, 0)
        return pm.decode(qb, kv[0], kv[1], btb[i % R5], ctxb, scale5)

    def decode_b_nccl(i: int):
        return padist.sequence_sharded_decode(qb, kv[0], kv[1], btb[i % R5], ctxb, scale5, group)

    # gate: dense fp32 partial of this rank's range, merged over the ranks
    got = decode_b(0)
    blocks = btb[0][0].long()
    kk = kv[0][blocks].float().reshape(nt, HKV5, D5).repeat_interleave(H5 // HKV5, dim=1)
    sc = torch.einsum("hd,thd->ht", qb[0], kk) * scale5
    del kk
    m = sc.max(dim=1).values
    p_ = torch.exp(sc - m[:, None])
    del sc
    vv = kv[1][blocks].float().reshape(nt, HKV5, D5).repeat_interleave(H5 // HKV5, dim=1)
    o_loc = torch.einsum("ht,thd->hd", p_, vv) / p_.sum(1)[:, None]
    lse_loc = m + torch.log(p_.sum(1))
    del vv, p_
    if world > 1:
        outs_all = [torch.empty_like(o_loc) for _ in range(world)]
        lses_all = [torch.empty_like(lse_loc) for _ in range(world)]
        dist.all_gather(outs_all, o_loc)
        dist.all_gather(lses_all, lse_loc)
        ls = torch.stack(lses_all)
        w = torch.exp(ls - ls.max(0).values)
        want = (torch.stack(outs_all) * w[..., None]).sum(0) / w.sum(0)[:, None]
    else:
        want = o_loc
    err_b = float((got[0] - want).abs().max())
    if world > 1:
        err_b = max(err_b, float((decode_b_nccl(0)[0] - want).abs().max()))
        if int(pm.status.item()) != 0:
            raise SystemExit(f"config5: device status {int(pm.status.item())}")
    err_b = max_over_ranks(err_b)
    if err_b > 2e-3:
        raise SystemExit(f"config5 sequence-shard gate failed: max-abs {err_b}")
    torch.cuda.empty_cache()

    # the same decode without the exchange shows what the exchange adds; the
    # three loops alternate over three rounds (median each) so that clock
    # drift within the run does not bias one of them
    def decode_b_local(i: int):
        return ops.paged_attention_v3_lse(qb, kv[0], kv[1], btb[i % R5], ctxb, scale5, 0)

    rounds = {"peer": [], "nccl": [], "local": []}
    for _ in range(3):
        rounds["peer"].append(timed(decode_b, args.steps))
        if world > 1:
            rounds["nccl"].append(timed(decode_b_nccl, args.steps))
        rounds["local"].append(timed(decode_b_local, args.steps))
    ms_b = statistics.median(rounds["peer"])
    ms_b_nccl = statistics.median(rounds["nccl"]) if world > 1 else ms_b
    ms_b_local = statistics.median(rounds["local"])
    bytes_b = NT * HKV5 * D5 * 2 * 2 * args.steps
    if world > 1:
        if int(pm.status.item()) != 0:
            raise SystemExit(f"config5: device status {int(pm.status.item())}")
        pm.close()
    gbs_b = bytes_b / (ms_b * 1e-3) / 1e9
    return {
        "batch_shard": {
            "value": round(gbs_a, 1), "unit": "GB/s",
            "pct_of_measured_hbm_peak": round(100 * gbs_a / world / peaks["hbm_gbs"], 1),
            "config": f"gpt2 fp16, {BA} sequences x ctx {CTXA} per GPU, {LA} layers, "
                      f"{RA} cold regions; no collective",
            "ms_per_step": round(ms_a / args.steps, 4),
            "tokens_per_s": round(BA * world * args.steps / (ms_a * 1e-3), 1)},
        "sequence_sharded": {
            "value": round(gbs_b, 1), "unit": "GB/s",
            "pct_of_measured_hbm_peak": round(100 * gbs_b / world / peaks["hbm_gbs"], 1),
            "config": f"1 sequence of {NT} tokens, 32q/8kv, D=128, bf16, "
                      f"{nt} tokens ({nt * HKV5 * D5 * 4 / 1e9:.2f} GB K+V) per GPU",
            "us_per_step": round(ms_b / args.steps * 1e3, 2),
            "us_per_step_local_only": round(ms_b_local / args.steps * 1e3, 2),
            "exchange_us_per_step": round((ms_b - ms_b_local) / args.steps * 1e3, 2),
            "exchange": "peer memory: flags + peer loads + LSE merge in one launch "
                        "(pa_merge_peer_partials)" if world > 1 else "none (one GPU)",
            "us_per_step_nccl_all_gather": round(ms_b_nccl / args.steps * 1e3, 2),
            "nccl_exchange_us_per_step": round((ms_b_nccl - ms_b_local) / args.steps * 1e3, 2),
            "correctness_gate_max_abs": err_b},
    }


def run_reference(args) -> None:
    rank, _, world = _env_rank()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    per_step = []
    for _ in range(args.warmup):
        cpu_sample(0.0, threads)
    for _ in range(args.steps):
        gbs, _, sample = cpu_sample(args.ref_step_seconds, threads)
        per_step.append(gbs)
    value = statistics.mean(per_step)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": "configs[1] decode layer calls, B=64, ctx=2048, H=HKV=12, "
                               "D=64, fp16 values computed in fp32 on the host",
                   "parallelism": f"{threads} host threads, rank 0 only"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample, "threads": threads,
                         "cpu_model": cpu_model(), "simd": simd_note()},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=3.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=12,
                    help="layer pools per decode step (configs[1]: 12)")
    ap.add_argument("--cold-pools", "--regions", dest="regions", type=int, default=4,
                    help="disjoint KV block regions rotated step by step (the reference "
                         "harness's --cold-pools)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the config-3 GQA measurement")
    ap.add_argument("--workload", choices=["config2", "config3", "config4", "config5", "fp8"],
                    default="config2",
                    help="config2 (default): the headline line with every extra; config3 / "
                         "config4 / config5 / fp8: one BASELINE config alone (the GQA decode, "
                         "the prefill, the multi-GPU lines under torchrun, the FP8-pool decode)")
    ap.add_argument("--pool-blocks", type=int, default=140_000,
                    help="config-3 pool blocks (140000: each K/V tensor > 2^31 elements)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    try:
        if args.impl == "reference":
            run_reference(args)
        elif args.workload == "config3":
            run_config3_only(args)
        elif args.workload == "config4":
            run_config4_only(args)
        elif args.workload == "config5":
            run_config5(args)
        elif args.workload == "fp8":
            run_fp8_only(args)
        else:
            run_b200(args)
    except SystemExit as e:
        if e.code in (None, 0):
            raise
        _error_line(str(e.code), args.impl)
        sys.exit(1)
    except BaseException as e:  # noqa: BLE001 -- every failure gets its line
        import traceback
        tb = traceback.extract_tb(e.__traceback__)
        at = f" at {Path(tb[-1].filename).name}:{tb[-1].lineno}" if tb else ""
        _error_line(f"{type(e).__name__}: {e}{at}", args.impl)
        sys.exit(1)


if __name__ == "__main__":
    main()
