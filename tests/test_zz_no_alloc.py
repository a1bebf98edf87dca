"""pa_paged_attention_v3_noalloc: the decode entry point for callers that
cannot allocate device memory when they decode (hosts that only receive
device pointers from elsewhere, or serving loops that reserve all device
memory up front).  Its scratch lives in a fixed 8 MiB array inside the library.

Checked through the C ABI against the regular entry point (which takes a
caller-allocated workspace), within the decode tolerance of the other tests
(max-abs 2e-3), on calls in a row with different inputs -- the array keeps
the previous call's contents, so the later calls show nothing stale leaks.
The third case has more than 1024 sequences, where the plan tables themselves
live in the array.
Named to be collected last; it passes alone in a fresh process as well."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from abi_helpers import PA_DT, abi_decode, max_abs, ptr, stream, to_dev
from oracle import oracle as orc
from pa_b200 import _lib

pytestmark = pytest.mark.gpu

LIMIT = 8 << 20  # PA_NOALLOC_SCRATCH_BYTES


def noalloc_decode(q, k, v, bt, ctx, scale, dtype, num_splits=0):
    qd, kd, vd = to_dev(q), to_dev(k, dtype), to_dev(v, dtype)
    btd, cd = to_dev(bt), to_dev(ctx)
    B, H, D = q.shape
    NB, BS, HKV, _ = k.shape
    out = torch.empty((B, H, D), device="cuda", dtype=torch.float32)
    lse = torch.empty((B, H), device="cuda", dtype=torch.float32)
    st = _lib.call("pa_paged_attention_v3_noalloc", ptr(out), ptr(lse), ptr(qd), ptr(kd),
                   ptr(vd), PA_DT[dtype], ptr(btd), ptr(cd), B, H, HKV, D, BS, NB,
                   bt.shape[1], float(scale), num_splits, None, stream())
    _lib.check("pa_paged_attention_v3_noalloc", st)
    torch.cuda.synchronize()
    return out.cpu().numpy(), lse.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    cases = [
        # GQA 32q/8kv, D=128, bf16, ragged contexts (one split over many CTAs)
        (orc.make_decode_case(71, 4, 32, 8, 128, 16, [5000, 17, 1200, 300]), "bfloat16", 128),
        # gpt2 geometry, fp16, different sizes for the second call
        (orc.make_decode_case(72, 16, 12, 12, 64, 16, 2048), "float16", 64),
        # more than 1024 short sequences: the plan kernel writes its tables
        # into the library's array (smaller batches plan in shared memory)
        (orc.make_decode_case(73, 1100, 12, 12, 64, 16,
                              np.random.default_rng(73).integers(1, 80, 1100)), "float16", 64),
    ]
    for (q, k, v, bt, ctx), dtype, D in cases:
        k, v = orc.round_to(k, dtype), orc.round_to(v, dtype)
        scale = D ** -0.5
        n = ctypes.c_size_t(0)
        _lib.check("ws", _lib.call("pa_decode_workspace_size", q.shape[0], q.shape[1],
                                   k.shape[2], D, PA_DT[dtype], 16, bt.shape[1], 0,
                                   ctypes.byref(n)))
        assert n.value <= LIMIT
        ref_out, ref_lse = abi_decode(q, k, v, bt, ctx, scale, dtype, want_lse=True)
        out, lse = noalloc_decode(q, k, v, bt, ctx, scale, dtype)
        assert max_abs(out, ref_out) <= 2e-3
        assert max_abs(lse, ref_lse) <= 2e-3
        assert max_abs(out, orc.decode(q, k, v, bt, ctx, scale, threads=8)) <= 2e-3


def test_noalloc_rejects_requests_beyond_its_scratch():
    # valid for the workspace entry point, but needs more than 8 MiB of scratch
    n = ctypes.c_size_t(0)
    _lib.check("ws", _lib.call("pa_decode_workspace_size", 512, 12, 12, 64, _lib.PA_DTYPE_F16,
                               16, 128, 8, ctypes.byref(n)))
    assert n.value > LIMIT
    st = _lib.call("pa_paged_attention_v3_noalloc", None, None, None, None, None,
                   _lib.PA_DTYPE_F16, None, None, 512, 12, 12, 64, 16, 8192, 128, 0.125, 8,
                   None, stream())
    assert st == _lib.PA_ERR_TOO_LARGE
