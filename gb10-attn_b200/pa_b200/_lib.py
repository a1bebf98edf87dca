"""ctypes binding of libpa_b200.so (the C ABI declared in include/pa_b200.h).

This is the FFI a non-torch host would write against the library; the tests
call the kernels through it.  It loads only the in-tree build and raises if
it is missing -- there is no fallback of any kind.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libpa_b200.so"
HEADER = PKG_DIR.parent.parent / "include" / "pa_b200.h"

PA_DTYPE_F32, PA_DTYPE_F16, PA_DTYPE_BF16, PA_DTYPE_F64, PA_DTYPE_E4M3 = 0, 1, 2, 3, 4
PA_OK = 0
PA_ERR_INVALID_ARGUMENT = 1
PA_ERR_NUM_HEADS = 2
PA_ERR_HEAD_DIM = 3
PA_ERR_DTYPE = 4
PA_ERR_BLOCK_SIZE = 5
PA_ERR_ALIGNMENT = 6
PA_ERR_WORKSPACE = 7
PA_ERR_CUDA = 8
PA_ERR_TOO_LARGE = 9
PA_ERR_NO_DEVICE = 10
PA_DEVERR_BLOCK_ID, PA_DEVERR_CONTEXT, PA_DEVERR_TIMEOUT, PA_DEVERR_MERGE = 1, 2, 4, 8
PA_DEVERR_RANGE = 0x10
PA_IPC_HANDLE_BYTES = 64

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_D = ctypes.c_double
_SZ = ctypes.c_size_t



class PaKvSeq(ctypes.Structure):
    """``pa_kv_seq`` of include/pa_b200.h: one sequence of pa_write_kv_batch."""
    _fields_ = [("k_src", _P), ("v_src", _P), ("src_layer_stride", _I64),
                ("src_head_stride", _I64), ("src_token_stride", _I64), ("block_ids", _P),
                ("num_block_ids", _I64), ("start", _I64), ("num_tokens", _I64)]


# name -> (restype, argtypes); mirrors include/pa_b200.h
_DECODE = [_P, _P, _I, _P, _P] + [_I64] * 7 + [_D]
SIGNATURES = {
    "pa_abi_version": (_I, []),
    "pa_strerror": (ctypes.c_char_p, [_I]),
    "pa_last_cuda_error": (_I, []),
    "pa_set_merge_arrive_rounds": (_I, [_I]),
    "pa_choose_num_splits": (_I64, [_I64, _I64, _I64]),
    "pa_decode_workspace_size": (_I, [_I64, _I64, _I64, _I64, _I, _I64, _I64, _I64,
                                      ctypes.POINTER(_SZ)]),
    "pa_paged_attention_v3": (_I, [_P, _P, _P, _P, _P, _I, _P, _P] + [_I64] * 7 +
                              [_D, _I64, _P, _SZ, _P, _P]),
    "pa_paged_attention_v3_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _P, _P] + [_I64] * 7 +
                                      [_D, _I64, _P, _P]),
    "pa_paged_attention_v3_fp8": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P] + [_I64] * 7 +
                                  [_D, _I64, _P, _SZ, _P, _P]),
    "pa_paged_attention": (_I, [_P, _P, _P, _P, _I, _P, _P] + [_I64] * 7 +
                           [_D, _P, _SZ, _P, _P]),
    "pa_paged_attention_v2": (_I, [_P, _P, _P, _P, _I, _P, _P] + [_I64] * 7 +
                              [_D, _P, _SZ, _P, _P]),
    "pa_merge_states": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "pa_peer_exchange_layout": (_I, [_I64, _I64] + [ctypes.POINTER(_SZ)] * 4),
    "pa_ipc_alloc": (_I, [_SZ, ctypes.POINTER(_P), _P]),
    "pa_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "pa_ipc_close": (_I, [_P]),
    "pa_ipc_free": (_I, [_P]),
    "pa_merge_peer_partials": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, ctypes.c_uint32, _P,
                                    _P]),
    "pa_prefill_workspace_size": (_I, [_I64, _I64, _I64, _I64, _I64, _I, _I64, _I64,
                                       ctypes.POINTER(_SZ)]),
    "pa_paged_attention_prefill": (_I, [_P, _P, _P, _P, _I, _P, _P] + [_I64] * 8 +
                                   [_D, _P, _SZ, _P, _P]),
    "pa_paged_attention_prefill_wmma": (_I, [_P, _P, _P, _P, _I, _P, _P] + [_I64] * 8 +
                                        [_D, _P, _SZ, _P, _P]),
    "pa_paged_attention_prefill_simt": (_I, [_P, _P, _P, _P, _I, _P, _P] + [_I64] * 8 +
                                        [_D, _P, _SZ, _P, _P]),
    "pa_write_kv": (_I, [_P, _P, _I, _P, _P, _I, _I64, _I64, _I64, _P] + [_I64] * 8 +
                    [_P, _P]),
    "pa_write_kv_scaled": (_I, [_P, _P, _I, _P, _P, _I, _I64, _I64, _I64, _P] + [_I64] * 8 +
                           [_P, _P, _P, _P]),
    "pa_write_kv_batch": (_I, [_P, _P, _I, _I, _P, _I64] + [_I64] * 5 + [_P, _P, _P, _P]),
    "pa_append_kv": (_I, [_P, _P, _I, _P, _P, _I, _P, _I64, _P] + [_I64] * 6 +
                     [_P, _P, _P, _P]),
    "pa_decode_layer_step": (_I, [_P, _P, _P, _I, _P, _P, _I, _P, _P, _P, _P] + [_I64] * 7 +
                             [_D, _I64, _P, _SZ, _P, _P]),
    "pa_validate_block_tables": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _P]),
}

_lib = None


def header_symbols() -> list[str]:
    """Entry points declared in include/pa_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^PA_API\s+[\w\s\*]+?\b(pa_\w+)\s*\(", text, re.M)))


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with "
                              "`python gb10-attn_b200/build.py` (or __graft_entry__.build())")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def strerror(status: int) -> str:
    return load().pa_strerror(status).decode()


class PaError(RuntimeError):
    def __init__(self, fn: str, status: int):
        msg = strerror(status)
        if status == PA_ERR_CUDA:
            msg += f" (cudaError {load().pa_last_cuda_error()})"
        super().__init__(f"{fn}: {msg}")
        self.status = status


def check(fn: str, status: int) -> None:
    if status != PA_OK:
        raise PaError(fn, status)


def call(name: str, *args) -> int:
    """Call an entry point; returns its status (does not raise)."""
    return getattr(load(), name)(*args)
