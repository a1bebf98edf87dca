"""The C ABI library on CPU: it loads, exports every entry point the header
declares, and rejects bad arguments before touching a device."""
from __future__ import annotations

import ctypes

import pytest

from pa_b200 import _lib


def test_library_loads_and_version():
    lib = _lib.load()
    assert lib.pa_abi_version() == 1


def test_exports_every_header_symbol():
    declared = _lib.header_symbols()
    assert len(declared) >= 15
    lib = _lib.load()
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # and the ctypes table covers every declared entry point
    assert set(declared) <= set(_lib.SIGNATURES), set(declared) - set(_lib.SIGNATURES)


def test_strerror_table():
    for code in range(0, 11):
        assert _lib.strerror(code) != "unknown status"
    assert _lib.strerror(999) == "unknown status"
    assert _lib.strerror(_lib.PA_ERR_NUM_HEADS) == "n_head must be divisible by n_kv_head"


@pytest.mark.parametrize("H,HKV,D,dt,want", [
    (12, 5, 64, _lib.PA_DTYPE_F16, _lib.PA_ERR_NUM_HEADS),
    (12, 12, 48, _lib.PA_DTYPE_F16, _lib.PA_ERR_HEAD_DIM),
    (12, 12, 64, 17, _lib.PA_ERR_DTYPE),
    (0, 12, 64, _lib.PA_DTYPE_F16, _lib.PA_ERR_INVALID_ARGUMENT),
])
def test_workspace_query_validates_before_device(H, HKV, D, dt, want):
    n = ctypes.c_size_t(0)
    st = _lib.call("pa_decode_workspace_size", 4, H, HKV, D, dt, 16, 128, 0, ctypes.byref(n))
    assert st == want


def test_no_device_is_reported_not_crashed():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    n = ctypes.c_size_t(0)
    st = _lib.call("pa_decode_workspace_size", 4, 12, 12, 64, _lib.PA_DTYPE_F16, 16, 128, 0,
                   ctypes.byref(n))
    assert st == _lib.PA_ERR_NO_DEVICE
    assert _lib.call("pa_choose_num_splits", 4, 12, 2048) == -1


def test_empty_batch_is_a_no_op():
    n = ctypes.c_size_t(123)
    assert _lib.call("pa_decode_workspace_size", 0, 12, 12, 64, _lib.PA_DTYPE_F16, 16, 128, 0,
                     ctypes.byref(n)) == 0
    assert n.value == 0
    # B = 0: no pointer is touched, nothing launched
    st = _lib.call("pa_paged_attention_v3", None, None, None, None, None, _lib.PA_DTYPE_F16,
                   None, None, 0, 12, 12, 64, 16, 10, 4, 0.125, 0, None, 0, None, None)
    assert st == 0


def test_peer_exchange_layout_and_argument_checks():
    f = [ctypes.c_size_t(0) for _ in range(4)]
    assert _lib.call("pa_peer_exchange_layout", 32, 128, *[ctypes.byref(x) for x in f]) == 0
    lse_off, slot, flags_off, total = (x.value for x in f)
    # out [32, 128] fp32, lse [32] fp32, each 256-byte aligned; two slots + flags
    assert lse_off == 32 * 128 * 4 and slot == lse_off + 256
    assert flags_off == 2 * slot and total == flags_off + 256  # 32 u32 flags, padded
    assert _lib.call("pa_peer_exchange_layout", 7, 62, *[ctypes.byref(x) for x in f]) == 0
    assert f[0].value % 256 == 0 and f[1].value % 256 == 0 and f[0].value >= 7 * 62 * 4
    assert _lib.call("pa_peer_exchange_layout", -1, 62,
                     *[ctypes.byref(x) for x in f]) == _lib.PA_ERR_INVALID_ARGUMENT
    bad = _lib.PA_ERR_INVALID_ARGUMENT
    dummy = ctypes.c_void_p(16)
    # world outside [1, 32], rank outside [0, world), null pointers: rejected
    # before any launch
    assert _lib.call("pa_merge_peer_partials", dummy, None, dummy, 0, 0, 4, 128, 1, None,
                     None) == bad
    assert _lib.call("pa_merge_peer_partials", dummy, None, dummy, 33, 0, 4, 128, 1, None,
                     None) == bad
    assert _lib.call("pa_merge_peer_partials", dummy, None, dummy, 2, 2, 4, 128, 1, None,
                     None) == bad
    assert _lib.call("pa_merge_peer_partials", None, None, dummy, 2, 0, 4, 128, 1, None,
                     None) == bad
    assert _lib.call("pa_merge_peer_partials", dummy, None, None, 2, 0, 4, 128, 1, None,
                     None) == bad
    # no rows: nothing to do
    assert _lib.call("pa_merge_peer_partials", dummy, None, dummy, 2, 1, 0, 128, 1, None,
                     None) == 0
    assert _lib.call("pa_ipc_alloc", 0, ctypes.byref(ctypes.c_void_p()), None) == bad
    assert _lib.call("pa_ipc_open", None, ctypes.byref(ctypes.c_void_p())) == bad


def test_append_kv_and_scaled_writer_argument_checks():
    bad = _lib.PA_ERR_INVALID_ARGUMENT
    one = (ctypes.c_void_p * 1)(16)
    d = ctypes.c_void_p(16)
    # negative sizes, null pointers with work to do: rejected before any launch
    assert _lib.call("pa_append_kv", one, one, _lib.PA_DTYPE_F16, d, d, _lib.PA_DTYPE_F32,
                     d, 4, d, -1, 1, 2, 64, 16, 8, None, None, None, None) == bad
    assert _lib.call("pa_append_kv", one, one, _lib.PA_DTYPE_F16, d, d, _lib.PA_DTYPE_F32,
                     None, 4, d, 3, 1, 2, 64, 16, 8, None, None, None, None) == bad
    assert _lib.call("pa_append_kv", one, one, _lib.PA_DTYPE_F16, d, d, _lib.PA_DTYPE_F32,
                     d, 4, None, 3, 1, 2, 64, 16, 8, None, None, None, None) == bad
    # a source dtype the writer does not read, a pool dtype it does not know
    assert _lib.call("pa_append_kv", one, one, _lib.PA_DTYPE_F16, d, d, _lib.PA_DTYPE_E4M3,
                     d, 4, d, 3, 1, 2, 64, 16, 8, None, None, None, None) == _lib.PA_ERR_DTYPE
    assert _lib.call("pa_append_kv", one, one, 17, d, d, _lib.PA_DTYPE_F32,
                     d, 4, d, 3, 1, 2, 64, 16, 8, None, None, None, None) == _lib.PA_ERR_DTYPE
    # no sequences: nothing to do
    assert _lib.call("pa_append_kv", None, None, _lib.PA_DTYPE_F16, None, None,
                     _lib.PA_DTYPE_F32, None, 4, None, 0, 1, 2, 64, 16, 8, None, None, None,
                     None) == 0
    assert _lib.call("pa_write_kv_scaled", None, None, _lib.PA_DTYPE_E4M3, None, None, 9, 0, 0, 0,
                     None, 4, 0, 10, 1, 12, 64, 16, 10, None, None, None, None) == bad


def test_write_kv_argument_checks():
    st = _lib.call("pa_write_kv", None, None, _lib.PA_DTYPE_F16, None, None, 9, 0, 0, 0, None,
                   4, 0, 10, 1, 12, 64, 16, 10, None, None)
    assert st == _lib.PA_ERR_INVALID_ARGUMENT  # null pointers with work to do
    st = _lib.call("pa_write_kv", None, None, _lib.PA_DTYPE_F16, None, None, 9, 0, 0, 0, None,
                   4, 0, 0, 1, 12, 64, 16, 10, None, None)
    assert st == 0  # zero tokens: nothing to do


def test_write_kv_batch_argument_checks():
    one = (ctypes.c_void_p * 1)(16)
    seqs = (_lib.PaKvSeq * 2)()
    bad = _lib.PA_ERR_INVALID_ARGUMENT
    args = (1, 2, 64, 16, 8, None, None, None, None)
    # null sequence array with sequences to write, negative counts
    assert _lib.call("pa_write_kv_batch", one, one, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32,
                     None, 2, *args) == bad
    assert _lib.call("pa_write_kv_batch", one, one, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32,
                     seqs, -1, *args) == bad
    seqs[1].num_tokens = -3
    assert _lib.call("pa_write_kv_batch", one, one, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32,
                     seqs, 2, *args) == bad
    # a sequence with tokens but no source
    seqs[1].num_tokens = 4
    assert _lib.call("pa_write_kv_batch", one, one, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32,
                     seqs, 2, *args) == bad
    # dtypes the writer does not handle
    assert _lib.call("pa_write_kv_batch", one, one, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_E4M3,
                     seqs, 2, *args) == _lib.PA_ERR_DTYPE
    assert _lib.call("pa_write_kv_batch", one, one, 17, _lib.PA_DTYPE_F32,
                     seqs, 2, *args) == _lib.PA_ERR_DTYPE
    # nothing to write: no sequences, or only empty ones
    assert _lib.call("pa_write_kv_batch", None, None, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32,
                     None, 0, *args) == 0
    seqs[1].num_tokens = 0
    assert _lib.call("pa_write_kv_batch", one, one, _lib.PA_DTYPE_F16, _lib.PA_DTYPE_F32,
                     seqs, 2, *args) == 0


def test_decode_layer_step_argument_checks():
    one = ctypes.c_void_p(16)
    args = (1, 8, 2, 64, 16, 8, 4, 0.125, 0, None, 0, None, None)
    # q / out in a type the step does not take
    assert _lib.call("pa_decode_layer_step", one, None, one, _lib.PA_DTYPE_F64, one, one,
                     _lib.PA_DTYPE_F16, None, None, one, one, *args) == _lib.PA_ERR_DTYPE
    # a new K row without its V row
    assert _lib.call("pa_decode_layer_step", one, None, one, _lib.PA_DTYPE_BF16, one, one,
                     _lib.PA_DTYPE_F16, one, None, one, one, *args) == _lib.PA_ERR_INVALID_ARGUMENT
    # an FP8 pool cannot take the append (its scales are not arguments here)
    assert _lib.call("pa_decode_layer_step", one, None, one, _lib.PA_DTYPE_BF16, one, one,
                     _lib.PA_DTYPE_E4M3, one, one, one, one, *args) == _lib.PA_ERR_DTYPE


def test_torch_shim_imports_on_cpu():
    from pa_b200 import ops
    assert ops.shim_path().exists()
    for name in ("paged_attention", "paged_attention_v2", "paged_attention_v3",
                 "choose_num_splits", "paged_attention_prefill", "paged_attention_prefill_wmma",
                 "write_kv"):
        assert callable(getattr(ops, name))


def test_shim_rejects_cpu_tensors_like_the_reference():
    import torch
    from pa_b200 import ops
    q = torch.zeros(1, 2, 32)
    k = torch.zeros(4, 16, 2, 32, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="q must be on CUDA"):
        ops.paged_attention_v3(q, k, k, torch.zeros(1, 1, dtype=torch.int32),
                               torch.ones(1, dtype=torch.int32), 0.1, 0)
