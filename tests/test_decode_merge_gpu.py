"""The split merge of the decode kernel: bit-determinism and the bounded
arrival's failure path, through the C ABI.

A sequence cut over several CTAs is merged by whichever warp arrives last at
its counter -- a CTA still inside its loop or one past its last tile, which
varies from launch to launch.  Both merge paths apply the same arithmetic in
the same order, so repeated launches on the same inputs must agree to the bit
(a serving loop, or bench.py's end-to-end check, compares them exactly).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from abi_helpers import decode_ws, max_abs, ptr, stream, to_dev
from oracle import oracle as orc
from pa_b200 import _lib

pytestmark = pytest.mark.gpu


def _launch(qd, kd, vd, btd, ctxd, scale, dtype, status=None):
    B, H, D = qd.shape
    NB, BS, HKV, _ = kd.shape
    MB = btd.shape[1]
    pa_dt = {"float16": _lib.PA_DTYPE_F16, "bfloat16": _lib.PA_DTYPE_BF16}[dtype]
    wsb = decode_ws(B, H, HKV, D, dtype, BS, MB)
    ws = torch.empty(max(wsb, 1), device=qd.device, dtype=torch.uint8)
    out = torch.empty((B, H, D), device=qd.device, dtype=torch.float32)
    _lib.check("pa_paged_attention_v3",
               _lib.call("pa_paged_attention_v3", ptr(out), None, ptr(qd), ptr(kd), ptr(vd),
                         pa_dt, ptr(btd), ptr(ctxd), B, H, HKV, D, BS, NB, MB, float(scale), 0,
                         ptr(ws), wsb, ptr(status), stream()))
    return out


@pytest.mark.parametrize("shape", [
    # configs[1] geometry: 64 sequences over 148 CTAs, pieces of 2-4 CTAs
    dict(B=64, H=12, HKV=12, D=64, ctx=[2048] * 64, dtype="float16"),
    # GQA, ragged: long sequences cut into > 8 pieces (two-level merge)
    dict(B=6, H=32, HKV=8, D=128, ctx=[30000, 1200, 17000, 64, 9000, 25000],
         dtype="bfloat16"),
])
def test_repeated_launches_are_bit_identical(shape):
    B, H, HKV, D, dtype = shape["B"], shape["H"], shape["HKV"], shape["D"], shape["dtype"]
    q, k, v, bt, ctx = orc.make_decode_case(77, B, H, HKV, D, 16, shape["ctx"])
    qd, kd, vd = to_dev(q), to_dev(k, dtype), to_dev(v, dtype)
    btd, ctxd = to_dev(bt), to_dev(ctx)
    first = _launch(qd, kd, vd, btd, ctxd, D ** -0.5, dtype)
    outs = [_launch(qd, kd, vd, btd, ctxd, D ** -0.5, dtype) for _ in range(40)]
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, first)
    ref = orc.decode(q, orc.round_to(k, dtype), orc.round_to(v, dtype), bt, ctx, D ** -0.5,
                     threads=8)
    assert max_abs(first.cpu().numpy(), ref) <= 2e-3


def test_merge_arrival_give_up_reports_and_writes_nan():
    """With the arrival limit at 0 every split piece gives up: its rows are
    NaN and PA_DEVERR_MERGE is set; rows held whole by one CTA are still
    exact.  The default limit is restored and the same call is correct."""
    dtype = "bfloat16"
    ctx_list = [32768, 16, 3000, 16]
    q, k, v, bt, ctx = orc.make_decode_case(78, 4, 32, 8, 128, 16, ctx_list)
    qd, kd, vd = to_dev(q), to_dev(k, dtype), to_dev(v, dtype)
    btd, ctxd = to_dev(bt), to_dev(ctx)
    ref = orc.decode(q, orc.round_to(k, dtype), orc.round_to(v, dtype), bt, ctx, 128 ** -0.5,
                     threads=8)
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    prev = _lib.call("pa_set_merge_arrive_rounds", 0)
    try:
        out = _launch(qd, kd, vd, btd, ctxd, 128 ** -0.5, dtype, status).cpu().numpy()
    finally:
        _lib.call("pa_set_merge_arrive_rounds", prev)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PA_DEVERR_MERGE
    assert np.isnan(out[0]).all()  # 32768 tokens: cut over many CTAs
    whole = ~np.isnan(out).any(axis=(1, 2))
    assert whole.any()  # at least one 16-token sequence sits inside one CTA
    assert max_abs(out[whole], ref[whole]) <= 2e-3
    assert np.isnan(out[~whole]).all(axis=(1, 2)).all()  # no half-written rows

    status.zero_()
    again = _launch(qd, kd, vd, btd, ctxd, 128 ** -0.5, dtype, status).cpu().numpy()
    assert int(status.item()) == 0
    assert max_abs(again, ref) <= 2e-3
