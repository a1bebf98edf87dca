"""Sequence-sharded long-context decode over two GPUs: each rank decodes its
own token range of every sequence with the split-KV kernel, and the (out, lse)
partials are merged either after one NCCL all-gather (pa_merge_states) or
straight from the peer's memory (PeerMerge / pa_merge_peer_partials); checked
against the CPU oracle on the full context (max-abs 2e-3).  Needs two GPUs;
skipped otherwise."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc
from pa_b200.dist import PeerMerge, sequence_sharded_decode, shard_range

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q, k, v, bt, ctx, scale, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        BS = k.shape[1]
        pages = -(-int(ctx.max()) // BS)
        p0, p1 = shard_range(pages, world, rank)
        bt_local = bt[:, p0:max(p1, p0 + 1)].contiguous()
        ctx_local = torch.clamp(ctx - p0 * BS, min=0)
        ctx_local = torch.minimum(ctx_local, torch.full_like(ctx_local, (p1 - p0) * BS))
        out = sequence_sharded_decode(q.to(dev), k.to(dev, torch.bfloat16), v.to(dev, torch.bfloat16),
                                      bt_local.to(dev), ctx_local.to(dev), scale)
        torch.cuda.synchronize()
        result.put((rank, out.cpu().numpy()))
    finally:
        dist.destroy_process_group()


def _local_range(bt, ctx, BS, world, rank):
    pages = -(-int(ctx.max()) // BS)
    p0, p1 = shard_range(pages, world, rank)
    bt_local = bt[:, p0:max(p1, p0 + 1)].contiguous()
    ctx_local = torch.clamp(ctx - p0 * BS, min=0)
    ctx_local = torch.minimum(ctx_local, torch.full_like(ctx_local, (p1 - p0) * BS))
    return bt_local, ctx_local


def _peer_worker(rank, world, port, qs, k, v, bt, ctx, scale, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    pm = None
    try:
        bt_local, ctx_local = _local_range(bt, ctx, k.shape[1], world, rank)
        kd, vd = k.to(dev, torch.bfloat16), v.to(dev, torch.bfloat16)
        btd, ctxd = bt_local.to(dev), ctx_local.to(dev)
        B, H, D = qs.shape[1:]
        pm = PeerMerge(B, H, D)
        outs = []
        # more steps than slots: both slots are written, read and reused
        for q in qs:
            outs.append(pm.decode(q.to(dev), kd, vd, btd, ctxd, scale))
        nccl = sequence_sharded_decode(qs[0].to(dev), kd, vd, btd, ctxd, scale)
        torch.cuda.synchronize()
        status = int(pm.status.item())
        result.put((rank, [o.cpu().numpy() for o in outs], nccl.cpu().numpy(), status))
    finally:
        if pm is not None:
            pm.close()
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("ctxs", [[5000, 1200], [33, 4097]])
def test_sequence_sharded_decode_two_gpus(ctxs):
    q, k, v, bt, ctx = orc.make_decode_case(62, B=2, H=32, HKV=8, D=128, BS=16, ctx=ctxs)
    k, v = orc.round_to(k, "bfloat16"), orc.round_to(v, "bfloat16")
    scale = 128 ** -0.5
    want = orc.decode(q, k, v, bt, ctx, scale)
    ctxm = mp.get_context("spawn")
    result = ctxm.Queue()
    port = _free_port()
    args = (2, port, torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
            torch.from_numpy(bt), torch.from_numpy(ctx), scale, result)
    procs = [ctxm.Process(target=_worker, args=(r, *args)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(result.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        assert np.abs(got[r] - want).max() <= 2e-3


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("ctxs", [[5000, 1200], [33, 4097]])
def test_sequence_sharded_decode_peer_memory_two_gpus(ctxs):
    steps = 5
    q, k, v, bt, ctx = orc.make_decode_case(63, B=2, H=32, HKV=8, D=128, BS=16, ctx=ctxs)
    k, v = orc.round_to(k, "bfloat16"), orc.round_to(v, "bfloat16")
    scale = 128 ** -0.5
    rng = np.random.default_rng(64)
    qs = np.stack([q] + [rng.standard_normal(q.shape).astype(np.float32)
                         for _ in range(steps - 1)])
    want = [orc.decode(qi, k, v, bt, ctx, scale) for qi in qs]
    ctxm = mp.get_context("spawn")
    result = ctxm.Queue()
    port = _free_port()
    args = (2, port, torch.from_numpy(qs), torch.from_numpy(k), torch.from_numpy(v),
            torch.from_numpy(bt), torch.from_numpy(ctx), scale, result)
    procs = [ctxm.Process(target=_peer_worker, args=(r, *args)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, outs, nccl, status = result.get(timeout=240)
        got[r] = (outs, nccl, status)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        outs, nccl, status = got[r]
        assert status == 0
        for i in range(steps):
            assert np.abs(outs[i] - want[i]).max() <= 2e-3
        # the NCCL path merges the same partials: same result to rounding
        assert np.abs(outs[0] - nccl).max() <= 1e-5
    # both ranks compute the merged rows in the same order: bit-identical
    for i in range(steps):
        assert np.array_equal(got[0][0][i], got[1][0][i])
