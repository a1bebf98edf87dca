"""Sequence-sharded long-context decode over two GPUs (NCCL): each rank
decodes its own token range of every sequence with the split-KV kernel
(paged_attention_v3_lse), the (out, lse) partials cross NVLink in one
all-gather, and pa_merge_states merges them; checked against the CPU oracle
on the full context (max-abs 2e-3).  Needs two GPUs; skipped otherwise."""
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
from pa_b200.dist import sequence_sharded_decode, shard_range

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
