"""Generate the golden fixtures under tests/golden/ from the reference's own code.

Two sources, both compiled from the reference sources by oracle/build_ref.py
into oracle/_ref/ (the reference's repository has no committed golden values):

  --arm      (CPU) the reference's scalar CPU lane, arm_cpu/src/scalar.cpp:
             attention_scores + softmax_inplace on the inputs of its own bench
             (arm_cpu/src/bench.cpp:56-63: mt19937(2026), U(-0.25, 0.25)).
             -> arm_scalar.npz
  --kernels  (GPU) the reference's five CUDA kernels, kernels/*.cu compiled
             unchanged for sm_100a, on small seeded decode / prefill cases and
             on the HIP self-test fixture (rocm/hip/paged_attn_v1_hip.cpp:
             151-164).  -> ref_kernels.npz

The CPU tests compare the oracle with these outputs; the GPU tests compare
the B200 kernels with them.  Usage (from the repo root):

    python tests/golden/make_golden.py --arm
    python tests/golden/make_golden.py --kernels   # on a machine with a B200
"""
from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import oracle as orc  # noqa: E402

ARM_SHAPES = [(2048, 64), (64, 128), (257, 32)]


def make_arm() -> Path:
    lib = ctypes.CDLL(str(REPO / "oracle" / "_ref" / "libref_arm_scalar.so"))
    P, I64 = ctypes.c_void_p, ctypes.c_int64
    lib.ref_attention_scores.argtypes = [P, P, P, I64, I64]
    lib.ref_softmax_inplace.argtypes = [P, I64]
    data = {}
    for tokens, dim in ARM_SHAPES:
        query, keys = orc.fixture_arm_bench(tokens, dim)
        scores = np.empty(tokens, np.float32)
        lib.ref_attention_scores(query.ctypes.data, keys.ctypes.data, scores.ctypes.data,
                                 tokens, dim)
        raw = scores.copy()
        lib.ref_softmax_inplace(scores.ctypes.data, tokens)
        data[f"t{tokens}_d{dim}_scores"] = raw
        data[f"t{tokens}_d{dim}_softmax"] = scores
    out = HERE / "arm_scalar.npz"
    np.savez_compressed(out, **data)
    return out


# (name, seed, B, H, HKV, D, BS, ctx, dtype)
DECODE_CASES = [
    ("gpt2ish_f16", 11, 3, 4, 4, 64, 16, [1, 37, 150], "float16"),
    ("gqa_f16", 12, 2, 8, 2, 128, 16, [5, 200], "float16"),
    ("f32_bs8", 13, 2, 4, 2, 32, 8, [17, 64], "float32"),
    ("f64_d256", 14, 2, 2, 1, 256, 16, [3, 40], "float64"),
]
# (name, seed, B, Sq, H, HKV, D, ctx, dtype)
PREFILL_CASES = [
    ("prefill_f16", 21, 2, 24, 4, 2, 64, [24, 70], "float16"),
    ("prefill_pad_f16", 22, 2, 20, 2, 2, 32, [12, 45], "float16"),
]


def make_kernels() -> Path:
    import torch
    sys.path.insert(0, str(REPO / "oracle" / "_ref"))
    import gb10_ref_kernels as ref  # noqa: E402

    dev = torch.device("cuda:0")
    tdt = {"float16": torch.float16, "float32": torch.float32, "float64": torch.float64}
    data = {}

    def put(prefix, **arrs):
        for k, v in arrs.items():
            data[f"{prefix}/{k}"] = np.asarray(v)

    # the HIP self-test fixture (fp32 pool), scale 1/sqrt(D)
    q, k, v, bt, ctx = orc.fixture_hip_selftest()
    scale = 1.0 / np.sqrt(np.float32(32))
    args = [torch.from_numpy(x).to(dev) for x in (q, k, v, bt, ctx)]
    put("hip_selftest", q=q, k=k, v=v, bt=bt, ctx=ctx, scale=np.float64(scale),
        v1=ref.paged_attention(*args, float(scale)).cpu().numpy(),
        v2=ref.paged_attention_v2(*args, float(scale)).cpu().numpy(),
        v3=ref.paged_attention_v3(*args, float(scale), 0).cpu().numpy(),
        v3_s3=ref.paged_attention_v3(*args, float(scale), 3).cpu().numpy())

    for name, seed, B, H, HKV, D, BS, ctxs, dt in DECODE_CASES:
        q, k, v, bt, ctx = orc.make_decode_case(seed, B, H, HKV, D, BS, ctxs)
        k, v = orc.round_to(k, dt), orc.round_to(v, dt)
        scale = float(D) ** -0.5
        args = [torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev, tdt[dt]),
                torch.from_numpy(v).to(dev, tdt[dt]), torch.from_numpy(bt).to(dev),
                torch.from_numpy(ctx).to(dev)]
        put(name, q=q, k=k.astype(dt), v=v.astype(dt), bt=bt, ctx=ctx, scale=np.float64(scale),
            v1=ref.paged_attention(*args, scale).cpu().numpy(),
            v2=ref.paged_attention_v2(*args, scale).cpu().numpy(),
            v3=ref.paged_attention_v3(*args, scale, 0).cpu().numpy())

    for name, seed, B, Sq, H, HKV, D, ctxs, dt in PREFILL_CASES:
        _, k, v, bt, ctx = orc.make_decode_case(seed, B, H, HKV, D, 16, ctxs)
        k, v = orc.round_to(k, dt), orc.round_to(v, dt)
        q = np.random.default_rng(seed).standard_normal((B, Sq, H, D), dtype=np.float32)
        scale = float(D) ** -0.5
        args = [torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev, tdt[dt]),
                torch.from_numpy(v).to(dev, tdt[dt]), torch.from_numpy(bt).to(dev),
                torch.from_numpy(ctx).to(dev)]
        put(name, q=q, k=k.astype(dt), v=v.astype(dt), bt=bt, ctx=ctx, scale=np.float64(scale),
            prefill=ref.paged_attention_prefill(*args, scale).cpu().numpy(),
            wmma=ref.paged_attention_prefill_wmma(*args, scale).cpu().numpy())

    put("choose_num_splits", args=np.array([[64, 12, 2048], [4, 12, 2048], [1, 12, 512],
                                            [8, 32, 32768], [512, 12, 8192], [2, 4, 40]]),
        values=np.array([ref.choose_num_splits(a, b, c) for a, b, c in
                         [(64, 12, 2048), (4, 12, 2048), (1, 12, 512), (8, 32, 32768),
                          (512, 12, 8192), (2, 4, 40)]]),
        sms=np.int64(torch.cuda.get_device_properties(0).multi_processor_count))
    out = HERE / "ref_kernels.npz"
    np.savez_compressed(out, **data)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--arm", action="store_true")
    ap.add_argument("--kernels", action="store_true")
    ap.add_argument("--out", default=None, help="copy the kernels fixture here too")
    a = ap.parse_args()
    if a.arm:
        print(make_arm())
    if a.kernels:
        p = make_kernels()
        print(p)
        if a.out:
            import shutil
            shutil.copy(p, a.out)
