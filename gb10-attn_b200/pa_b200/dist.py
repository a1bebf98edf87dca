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
"""
from __future__ import annotations

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
