"""Call the kernels through the C ABI (ctypes over libpa_b200.so), the way a
non-torch host would.  torch only provides device memory and the stream."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from pa_b200 import _lib

TORCH_DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
            "float64": torch.float64}
PA_DT = {"float32": _lib.PA_DTYPE_F32, "float16": _lib.PA_DTYPE_F16,
         "bfloat16": _lib.PA_DTYPE_BF16, "float64": _lib.PA_DTYPE_F64}


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def to_dev(x, dtype: str | None = None, device="cuda:0") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.to(device, TORCH_DT[dtype]) if dtype else t.to(device)


def decode_ws(B, H, HKV, D, dtype, BS, MB, num_splits=0) -> int:
    n = ctypes.c_size_t(0)
    _lib.check("pa_decode_workspace_size",
               _lib.call("pa_decode_workspace_size", B, H, HKV, D, PA_DT[dtype], BS, MB,
                         num_splits, ctypes.byref(n)))
    return n.value


def abi_decode(q, k, v, bt, ctx, scale, dtype, num_splits=0, entry="pa_paged_attention_v3",
               want_lse=False, num_blocks=None, status=None, raise_on_error=True):
    """Decode through the C ABI.  k/v are numpy values (cast to `dtype` on the
    device) or device tensors already of that dtype.  Returns out (and lse)."""
    qd = to_dev(q) if not isinstance(q, torch.Tensor) else q
    kd = to_dev(k, dtype) if not isinstance(k, torch.Tensor) else k
    vd = to_dev(v, dtype) if not isinstance(v, torch.Tensor) else v
    btd = to_dev(np.asarray(bt, np.int32)) if not isinstance(bt, torch.Tensor) else bt
    ctxd = to_dev(np.asarray(ctx, np.int32)) if not isinstance(ctx, torch.Tensor) else ctx
    B, H, D = qd.shape
    NB, BS, HKV, _ = kd.shape
    MB = btd.shape[1]
    out = torch.empty((B, H, D), device=qd.device, dtype=torch.float32)
    lse = torch.empty((B, H), device=qd.device, dtype=torch.float32) if want_lse else None
    wsb = decode_ws(B, H, HKV, D, dtype, BS, MB, num_splits if entry.endswith("v3") else 0)
    ws = torch.empty(max(wsb, 1), device=qd.device, dtype=torch.uint8)
    nb = NB if num_blocks is None else num_blocks
    common = (PA_DT[dtype], ptr(btd), ptr(ctxd), B, H, HKV, D, BS, nb, MB, float(scale))
    if entry == "pa_paged_attention_v3":
        st = _lib.call(entry, ptr(out), ptr(lse), ptr(qd), ptr(kd), ptr(vd), *common,
                       num_splits, ptr(ws), wsb, ptr(status), stream())
    else:
        st = _lib.call(entry, ptr(out), ptr(qd), ptr(kd), ptr(vd), *common, ptr(ws), wsb,
                       ptr(status), stream())
    if raise_on_error:
        _lib.check(entry, st)
    torch.cuda.synchronize()
    if want_lse:
        return out.cpu().numpy(), lse.cpu().numpy()
    return out.cpu().numpy()


def abi_prefill(q, k, v, bt, ctx, scale, dtype, entry="pa_paged_attention_prefill",
                status=None):
    qd = to_dev(q)
    kd = to_dev(k, dtype) if not isinstance(k, torch.Tensor) else k
    vd = to_dev(v, dtype) if not isinstance(v, torch.Tensor) else v
    btd = to_dev(np.asarray(bt, np.int32))
    ctxd = to_dev(np.asarray(ctx, np.int32))
    B, Sq, H, D = qd.shape
    NB, BS, HKV, _ = kd.shape
    MB = btd.shape[1]
    n = ctypes.c_size_t(0)
    _lib.check("pa_prefill_workspace_size",
               _lib.call("pa_prefill_workspace_size", B, Sq, H, HKV, D, PA_DT[dtype], BS, MB,
                         ctypes.byref(n)))
    ws = torch.empty(max(n.value, 1), device=qd.device, dtype=torch.uint8)
    out = torch.empty((B, Sq, H, D), device=qd.device, dtype=torch.float32)
    st = _lib.call(entry, ptr(out), ptr(qd), ptr(kd), ptr(vd), PA_DT[dtype], ptr(btd),
                   ptr(ctxd), B, Sq, H, HKV, D, BS, NB, MB, float(scale), ptr(ws), n.value,
                   ptr(status), stream())
    _lib.check(entry, st)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def max_abs(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    same = (np.isnan(a) & np.isnan(b)) | (np.isinf(a) & (a == b))  # NaN/NaN, equal infinities
    d = np.abs(np.where(same, 0, a) - np.where(same, 0, b))
    return float(np.nan_to_num(d, nan=np.inf).max(initial=0.0))
