"""Multi-GPU host logic on CPU ranks (gloo, world_size 2): batch-shard ranges,
and the sequence-sharded long-context decode of pa_b200.dist -- local partial
(out, lse) per rank, one all-gather, log-sum-exp merge -- with the oracle
standing in for the GPU partial kernel."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pa_b200.dist import gather_states, sequence_sharded_decode, shard_range


def test_shard_range_covers_everything():
    for n in (0, 1, 7, 64, 513):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert max(h - lo for lo, h in parts) - min(h - lo for lo, h in parts) <= 1


def _partial_oracle(q, k, v, bt, ctx, scale):
    """(normalised out, natural-log lse) of a local token range, in float64."""
    from oracle import oracle as orc
    q, k, v = q.numpy(), k.numpy(), v.numpy()
    bt, ctx = bt.numpy(), ctx.numpy()
    B, H, D = q.shape
    BS, HKV = k.shape[1], k.shape[2]
    out = orc.decode(q, k, v, bt, ctx, scale)
    lse = np.full((B, H), -np.inf, np.float32)
    for b in range(B):
        n = int(ctx[b])
        if n <= 0:
            out[b] = 0.0
            continue
        for h in range(H):
            g = h // (H // HKV)
            ks = np.stack([k[bt[b, j // BS], j % BS, g] for j in range(n)]).astype(np.float64)
            s = scale * ks @ q[b, h].astype(np.float64)
            lse[b, h] = s.max() + np.log(np.exp(s - s.max()).sum())
    return torch.from_numpy(out), torch.from_numpy(lse)


def _merge_cpu(outs, lses):
    m = lses.max(0).values
    w = torch.where(torch.isinf(lses), torch.zeros_like(lses), torch.exp(lses - m))
    den = w.sum(0)
    return (outs * w.unsqueeze(-1)).sum(0) / den.unsqueeze(-1), m + torch.log(den)


def _worker(rank, world, port, q, k, v, bt, ctx, scale, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # rank r holds tokens [lo, hi) of every sequence: its pages are the
        # corresponding slice of the block table (block-aligned split)
        BS = k.shape[1]
        n = int(ctx.max())
        pages = -(-n // BS)
        p0, p1 = shard_range(pages, world, rank)
        bt_local = bt[:, p0:max(p1, p0 + 1)].clone()
        ctx_local = torch.clamp(ctx - p0 * BS, min=0)
        ctx_local = torch.minimum(ctx_local, torch.full_like(ctx_local, (p1 - p0) * BS))
        out = sequence_sharded_decode(q, k, v, bt_local, ctx_local, scale,
                                      partial_fn=_partial_oracle, merge_fn=_merge_cpu)
        outs, lses = gather_states(out, torch.zeros(out.shape[:2]))
        assert outs.shape[0] == world
        if rank == 0:
            result.put(out.numpy())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ctxs", [[700, 700], [1000, 37]])
def test_sequence_sharded_decode_two_gloo_ranks(ctxs):
    from oracle import oracle as orc
    q, k, v, bt, ctx = orc.make_decode_case(61, B=2, H=8, HKV=2, D=32, BS=16, ctx=ctxs)
    scale = 32 ** -0.5
    want = orc.decode(q, k, v, bt, ctx, scale)
    ctxm = mp.get_context("spawn")
    result = ctxm.Queue()
    port = _free_port()
    args = (2, port, torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
            torch.from_numpy(bt), torch.from_numpy(ctx), scale, result)
    procs = [ctxm.Process(target=_worker, args=(r, *args)) for r in range(2)]
    for p in procs:
        p.start()
    got = result.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.abs(got - want).max() < 1e-5
