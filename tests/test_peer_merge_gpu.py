"""pa_merge_peer_partials on one GPU: the peers are emulated by exchange
buffers on the same device whose flags the test raises before the launch, so
no launch waits on another launch.  Checked against the log-sum-exp merge of
the reference's merge_splits_kernel (kernels/paged_attn_v3.cu:139-165),
restated in numpy; plus the timeout path (a flag that nothing raises)."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from abi_helpers import max_abs, ptr, stream
from pa_b200 import _lib

pytestmark = pytest.mark.gpu


def layout(rows, D):
    f = [ctypes.c_size_t(0) for _ in range(4)]
    _lib.check("layout", _lib.call("pa_peer_exchange_layout", rows, D,
                                   *[ctypes.byref(x) for x in f]))
    return [x.value for x in f]  # lse_offset, slot_bytes, flags_offset, total


def np_merge(outs, lses):
    """outs [R, rows, D], lses [R, rows] -> merged out, lse (NaN rows where
    every part is empty)."""
    mx = lses.max(0)
    with np.errstate(invalid="ignore", divide="ignore"):
        w = np.where(np.isneginf(lses), 0.0, np.exp(lses - mx))
        den = w.sum(0)
        num = np.einsum("rn,rnd->nd", w, np.where(np.isneginf(lses)[..., None], 0.0, outs))
        out = num / den[:, None]
        lse = np.where(den > 0, mx + np.log(den), -np.inf)
    return out, lse


def make_buffers(world, rows, D, epoch, seed, raise_flags_of=None):
    """One exchange buffer per emulated rank holding its partial in slot
    epoch & 1; flags of `raise_flags_of` ranks set to epoch in every buffer."""
    lse_off, slot, flags_off, total = layout(rows, D)
    rng = np.random.default_rng(seed)
    outs = rng.standard_normal((world, rows, D)).astype(np.float32)
    lses = (rng.standard_normal((world, rows)) * 3).astype(np.float32)
    lses[0, 1] = -np.inf          # rank 0 holds no token of row 1
    lses[:, 2] = -np.inf          # no rank holds a token of row 2 -> NaN
    outs[0, 1] = np.nan           # an empty range's out is never read
    outs[:, 2] = np.nan
    raise_flags_of = range(world) if raise_flags_of is None else raise_flags_of
    bufs = []
    for r in range(world):
        b = torch.zeros(total, dtype=torch.uint8, device="cuda:0")
        s = (epoch & 1) * slot
        b[s:s + rows * D * 4].view(torch.float32).copy_(torch.from_numpy(outs[r].ravel()))
        b[s + lse_off:s + lse_off + rows * 4].view(torch.float32).copy_(torch.from_numpy(lses[r]))
        fl = b[flags_off:flags_off + 4 * world].view(torch.int32)
        for p in raise_flags_of:
            fl[p] = int(np.uint32(epoch).view(np.int32))
        bufs.append(b)
    bases = torch.tensor([x.data_ptr() for x in bufs], dtype=torch.int64, device="cuda:0")
    return bufs, bases, outs, lses


def run(bases, world, rank, rows, D, epoch, status=None):
    out = torch.empty((rows, D), dtype=torch.float32, device="cuda:0")
    lse = torch.empty(rows, dtype=torch.float32, device="cuda:0")
    _lib.check("merge", _lib.call("pa_merge_peer_partials", ptr(out), ptr(lse), ptr(bases), world,
                                  rank, rows, D, epoch, ptr(status), stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("world,D,epoch", [(1, 128, 1), (2, 128, 2), (3, 64, 7), (8, 128, 5),
                                           (8, 62, 0xFFFFFFFF), (32, 32, 12)])
def test_merge_matches_lse_rule(world, D, epoch):
    rows = 64
    bufs, bases, outs, lses = make_buffers(world, rows, D, epoch, seed=world * 100 + D)
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    got, got_lse = run(bases, world, world - 1, rows, D, epoch, status)
    want, want_lse = np_merge(outs.astype(np.float64), lses.astype(np.float64))
    assert int(status.item()) == 0
    assert max_abs(got, want) <= 1e-5
    assert max_abs(got_lse, want_lse) <= 1e-5
    assert np.isnan(got[2]).all() and np.isneginf(got_lse[2])


def test_every_rank_computes_identical_rows():
    world, rows, D, epoch = 4, 96, 128, 3
    bufs, bases, _, _ = make_buffers(world, rows, D, epoch, seed=5)
    res = [run(bases, world, r, rows, D, epoch)[0] for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(res[0], res[r], equal_nan=True)


def test_flags_raised_on_every_peer():
    world, rows, D, epoch = 4, 8, 64, 9
    bufs, bases, _, _ = make_buffers(world, rows, D, epoch, seed=6)
    _, _, flags_off, _ = layout(rows, D)
    for b in bufs:  # rank 1's flag cleared in every buffer ...
        b[flags_off + 4:flags_off + 8].zero_()
    # ... and every flag raised in rank 1's own buffer, so its wait passes
    bufs[1][flags_off:flags_off + 4 * world].view(torch.int32).fill_(epoch)
    run(bases, world, 1, rows, D, epoch)
    for b in bufs:
        assert int(b[flags_off + 4:flags_off + 8].view(torch.int32).item()) == epoch


def test_peer_one_epoch_ahead_counts_as_ready():
    # a faster peer may already have raised epoch + 1 when this rank waits
    world, rows, D, epoch = 2, 16, 128, 4
    bufs, bases, outs, lses = make_buffers(world, rows, D, epoch, seed=7)
    _, _, flags_off, _ = layout(rows, D)
    bufs[0][flags_off + 4:flags_off + 8].view(torch.int32).fill_(epoch + 1)
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    got, _ = run(bases, world, 0, rows, D, epoch, status)
    assert int(status.item()) == 0
    assert max_abs(got, np_merge(outs.astype(np.float64), lses.astype(np.float64))[0]) <= 1e-5


def test_missing_peer_times_out_and_reports():
    # rank 1 never raises its flag in rank 0's buffer: the bounded wait gives
    # up after ~1 s, the rows are NaN and the status word says so
    world, rows, D, epoch = 2, 32, 128, 1
    bufs, bases, _, _ = make_buffers(world, rows, D, epoch, seed=8, raise_flags_of=[0])
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    t0 = time.perf_counter()
    got, got_lse = run(bases, world, 0, rows, D, epoch, status)
    dt = time.perf_counter() - t0
    assert int(status.item()) & _lib.PA_DEVERR_TIMEOUT
    assert np.isnan(got).all() and np.isnan(got_lse).all()
    assert 0.9 < dt < 10
    # the context stays usable: the next epoch with every flag raised works
    bufs2, bases2, outs2, lses2 = make_buffers(world, rows, D, 2, seed=9)
    got2, _ = run(bases2, world, 0, rows, D, 2)
    assert max_abs(got2, np_merge(outs2.astype(np.float64), lses2.astype(np.float64))[0]) <= 1e-5
