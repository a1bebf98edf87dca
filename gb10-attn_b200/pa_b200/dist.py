"""Multi-GPU decode: batch sharding and sequence-sharded long-context decode.

The reference is single-GPU (``docs/REPORT.md:274``); the B200 build adds the
two partitions of the decode path across the GPUs of one box, one process per
GPU (``torch.distributed``, NCCL over NVLink):

* batch sharding -- rank r decodes sequences ``shard_range(B, world, r)``
  against its own pool; no collective on the data path.
* sequence sharding -- one very long context is split into ``world`` token
  ranges, one per GPU, each with its local pages and block table.  Every rank
  computes the normalised partial ``out_r`` and ``lse_r`` of its range
  (``paged_attention_v3_lse``), the ranks exchange the small
  ``[B, H, D + 1]`` partials with one all-gather, and each merges them with the
  log-sum-exp rule of the reference's ``merge_splits_kernel``
  (``kernels/paged_attn_v3.cu:139-165``), here ``pa_merge_states``.

The compute and merge steps are injectable so the host logic (ranges, packing,
gather order, merge) is testable on CPU ranks with gloo.

``PeerMerge`` is the same sequence-sharded decode with the exchange on peer
memory instead of a collective: every rank's decode writes its partial into
an exchange buffer in its own HBM that every other rank has mapped (CUDA IPC),
and one small kernel of ours (``pa_merge_peer_partials``) raises this rank's
step flag on every peer, waits (bounded) for theirs and merges the peers'
partials with plain peer loads -- one launch instead of an all-gather plus a
merge launch.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous share [lo, hi) of n items for rank (sizes differ by <= 1)."""
    return n * rank // world, n * (rank + 1) // world


def pack_state(out: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    return torch.cat([out, lse.unsqueeze(-1)], dim=-1).contiguous()


def unpack_states(packed: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    return packed[..., :-1].contiguous(), packed[..., -1].contiguous()


def gather_states(out: torch.Tensor, lse: torch.Tensor, group=None
                  ) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather the (out [B,H,D], lse [B,H]) partials of every rank:
    returns outs [R,B,H,D], lses [R,B,H] in rank order (one collective)."""
    world = dist.get_world_size(group)
    packed = pack_state(out.float(), lse.float())
    # flat [world * B, ...] output: the layout every backend accepts
    buf = torch.empty((world * packed.shape[0], *packed.shape[1:]), dtype=packed.dtype,
                      device=packed.device)
    dist.all_gather_into_tensor(buf, packed, group=group)
    return unpack_states(buf.view(world, *packed.shape))


def sequence_sharded_decode(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                            block_tables_local: torch.Tensor, context_lens_local: torch.Tensor,
                            scale: float, group=None,
                            partial_fn: Callable | None = None,
                            merge_fn: Callable | None = None) -> torch.Tensor:
    """Decode of sequences whose KV is split across the ranks of `group`.

    Each rank passes the same q and its own slice of the context (local pages,
    block table and lengths; a rank holding no tokens of a sequence passes
    length 0).  Returns the merged [B, H, D] output on every rank."""
    if partial_fn is None or merge_fn is None:
        from . import ops
        partial_fn = partial_fn or (lambda *a: ops.paged_attention_v3_lse(*a, 0))
        merge_fn = merge_fn or ops.merge_states
    out, lse = partial_fn(q, k_local, v_local, block_tables_local, context_lens_local, scale)
    outs, lses = gather_states(out, lse, group)
    merged, _ = merge_fn(outs, lses)
    return merged


class PeerMerge:
    """Sequence-sharded decode with its exchange on peer memory.

    Collective to construct and to ``close()``: every rank of `group` builds
    one with the same (num_seqs, num_heads, head_dim).  ``decode`` is called
    once per step on every rank in the same order (each call is one epoch of
    the exchange protocol of ``include/pa_b200.h``); it returns the merged
    [B, H, D] output, identical on every rank.  ``status`` is the device
    word the kernels OR their PA_DEVERR_* bits into (a timed-out exchange
    wait sets PA_DEVERR_TIMEOUT and yields NaN rows)."""

    def __init__(self, num_seqs: int, num_heads: int, head_dim: int, group=None,
                 device: torch.device | None = None):
        from . import _lib
        self._lib = _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        self.B, self.H, self.D = num_seqs, num_heads, head_dim
        self.rows = num_seqs * num_heads
        f = [ctypes.c_size_t(0) for _ in range(4)]
        _lib.check("pa_peer_exchange_layout",
                   _lib.call("pa_peer_exchange_layout", self.rows, head_dim,
                             *[ctypes.byref(x) for x in f]))
        self.lse_offset, self.slot_bytes, self.flags_offset, total = (x.value for x in f)
        handle = ctypes.create_string_buffer(_lib.PA_IPC_HANDLE_BYTES)
        base = ctypes.c_void_p(0)
        with torch.cuda.device(self.dev):
            _lib.check("pa_ipc_alloc", _lib.call("pa_ipc_alloc", total, ctypes.byref(base),
                                                 handle))
        self.base = base.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        bases = []
        with torch.cuda.device(self.dev):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self.base)
                    continue
                p = ctypes.c_void_p(0)
                _lib.check("pa_ipc_open", _lib.call("pa_ipc_open", h, ctypes.byref(p)))
                self._opened.append(p.value)
                bases.append(p.value)
        as_i64 = [b - (1 << 64) if b >= (1 << 63) else b for b in bases]
        self.peer_bases = torch.tensor(as_i64, dtype=torch.int64, device=self.dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self._ws = None
        self.epoch = 0
        # every buffer is zeroed (pa_ipc_alloc synchronises) before any rank
        # can raise a flag in it
        dist.barrier(group)

    def slot(self, epoch: int) -> tuple[int, int]:
        """(out, lse) device addresses of this rank's slot for `epoch`."""
        s = self.base + (epoch & 1) * self.slot_bytes
        return s, s + self.lse_offset

    def decode(self, q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
               block_tables_local: torch.Tensor, context_lens_local: torch.Tensor,
               scale: float, out: torch.Tensor | None = None,
               num_splits: int = 0) -> torch.Tensor:
        L = self._lib
        B, H, D = q.shape
        if (B, H, D) != (self.B, self.H, self.D):
            raise ValueError(f"PeerMerge built for {(self.B, self.H, self.D)}, got {(B, H, D)}")
        NB, BS, HKV, _ = k_local.shape
        MB = block_tables_local.shape[1]
        dt = {torch.float32: L.PA_DTYPE_F32, torch.float16: L.PA_DTYPE_F16,
              torch.bfloat16: L.PA_DTYPE_BF16, torch.float64: L.PA_DTYPE_F64}[k_local.dtype]
        if self._ws is None or self._ws_key != (NB, BS, HKV, MB, dt, num_splits):
            n = ctypes.c_size_t(0)
            L.check("pa_decode_workspace_size",
                    L.call("pa_decode_workspace_size", B, H, HKV, D, dt, BS, MB, num_splits,
                           ctypes.byref(n)))
            self._ws = torch.empty(max(n.value, 1), dtype=torch.uint8, device=self.dev)
            self._ws_bytes = n.value
            self._ws_key = (NB, BS, HKV, MB, dt, num_splits)
        qf = q.float().contiguous()
        if out is None:
            out = torch.empty((B, H, D), dtype=torch.float32, device=self.dev)
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        # u32 serial numbers: after 2^32 - 1 comes 0, which still compares as
        # newer than the flags of the step before; the parity keeps alternating
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        o_ptr, l_ptr = self.slot(self.epoch)
        L.check("pa_paged_attention_v3",
                L.call("pa_paged_attention_v3", o_ptr, l_ptr, qf.data_ptr(), k_local.data_ptr(),
                       v_local.data_ptr(), dt, block_tables_local.data_ptr(),
                       context_lens_local.data_ptr(), B, H, HKV, D, BS, NB, MB, float(scale),
                       num_splits, self._ws.data_ptr(), self._ws_bytes,
                       self.status.data_ptr(), stream))
        L.check("pa_merge_peer_partials",
                L.call("pa_merge_peer_partials", out.data_ptr(), None,
                       self.peer_bases.data_ptr(), self.world, self.rank, self.rows, D,
                       self.epoch, self.status.data_ptr(), stream))
        return out

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self.base is None:
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(self.group)  # no rank still reads a peer buffer
        with torch.cuda.device(self.dev):
            for p in self._opened:
                self._lib.check("pa_ipc_close", self._lib.call("pa_ipc_close", p))
            self._opened = []
        dist.barrier(self.group)  # every mapping of this rank's buffer is gone
        with torch.cuda.device(self.dev):
            self._lib.check("pa_ipc_free", self._lib.call("pa_ipc_free", self.base))
        self.base = None
