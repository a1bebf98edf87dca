"""Paged KV pool: block allocator, per-layer pool proxy and the pool writer.

Mirrors the interface of hetero-serve's ``heteroserve/kv/torch_blocks.py``
(un-vendored by the reference; known from its call sites
``harness/repro_crash.py:39-58`` and ``harness/gb10_extended.sbatch:40-53``,
and from ``docs/REPORT.md:141-179``)::

    kv = KVConfig(block_size=16, num_blocks=N, dtype="float16")
    alloc = TorchBlockAllocator(kv, ModelConfig(), device="cuda:0")
    a = alloc.allocate(token_ids)          # a.block_ids
    alloc.write_kv(a.block_ids, 0, k, v)   # k, v: [n_layer, n_kv_head, n_tok, head_dim]
    alloc.pool[layer, 0]                   # K of one layer: [NB, BS, HKV, D]

Layout: ``[n_layer, 2, num_blocks, block_size, n_kv_head, head_dim]``
(gb10-attn ``README.md:114-117``).  By default each layer is its own tensor
behind ``LayeredPool`` (the reference's ``_LayeredPool`` fix); ``layered=False``
keeps one monolithic tensor, which the B200 kernels also address correctly
beyond 2^31 elements (all offsets are 64-bit).

The scatter itself is the ``pa_write_kv`` kernel (``csrc/write_kv.cu``); the
host side here only moves the source to the device (pinned, asynchronous), as
the reference's ``write_kv`` did with ``torch.as_tensor``.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

INT32_MAX = 2**31 - 1

_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
           "float64": torch.float64, "half": torch.float16, "bf16": torch.bfloat16,
           "float": torch.float32, "e4m3": torch.float8_e4m3fn,
           "float8_e4m3fn": torch.float8_e4m3fn}


@dataclass
class KVConfig:
    block_size: int = 16
    num_blocks: int = 1024
    dtype: str = "float16"


@dataclass
class ModelConfig:
    """Model geometry; defaults are GPT-2 small (the reference's ModelConfig())."""
    name: str = "gpt2"
    n_layer: int = 12
    n_head: int = 12
    head_dim: int = 64
    n_kv_head: int | None = None

    @property
    def kv_heads(self) -> int:
        return self.n_kv_head or self.n_head


@dataclass
class Allocation:
    block_ids: list[int]
    num_tokens: int
    token_ids: list[int] = field(default_factory=list)


class LayeredPool:
    """One tensor per layer, indexed like the monolithic
    ``[n_layer, 2, NB, BS, H, D]`` tensor: ``pool[l]``, ``pool[l, kv]``,
    ``pool[l, kv, ids]``, ``pool[:, :, ids]`` and assignment through the same
    keys.  Keeps every single tensor's element count n_layer times smaller."""

    def __init__(self, layers: list[torch.Tensor]):
        self.layers = layers

    @property
    def shape(self) -> tuple[int, ...]:
        return (len(self.layers), *self.layers[0].shape)

    @property
    def dtype(self) -> torch.dtype:
        return self.layers[0].dtype

    @property
    def device(self) -> torch.device:
        return self.layers[0].device

    def numel(self) -> int:
        return sum(t.numel() for t in self.layers)

    def __len__(self) -> int:
        return len(self.layers)

    def _split(self, key):
        if not isinstance(key, tuple):
            key = (key,)
        return key[0], key[1:]

    def __getitem__(self, key):
        first, rest = self._split(key)
        if isinstance(first, (int, np.integer)):
            t = self.layers[int(first)]
            return t[rest] if rest else t
        idx = range(len(self.layers))[first]
        return torch.stack([self.layers[i][rest] if rest else self.layers[i] for i in idx])

    def __setitem__(self, key, value):
        first, rest = self._split(key)
        if isinstance(first, (int, np.integer)):
            t = self.layers[int(first)]
            if rest:
                t[rest] = value
            else:
                t.copy_(value)
            return
        idx = list(range(len(self.layers))[first])
        for j, i in enumerate(idx):
            v = value[j] if isinstance(value, torch.Tensor) and value.dim() > 0 and \
                value.shape[0] == len(idx) else value
            if rest:
                self.layers[i][rest] = v
            else:
                self.layers[i].copy_(v)


class TorchBlockAllocator:
    """Block allocator over a paged KV pool on one device."""

    def __init__(self, kv_cfg: KVConfig, model_cfg: ModelConfig | None = None,
                 device: str | torch.device = "cuda:0", layered: bool = True,
                 zero: bool = True):
        self.kv_cfg = kv_cfg
        self.model_cfg = model_cfg or ModelConfig()
        self.device = torch.device(device)
        dt = _DTYPES[kv_cfg.dtype] if isinstance(kv_cfg.dtype, str) else kv_cfg.dtype
        m = self.model_cfg
        per_layer = (2, kv_cfg.num_blocks, kv_cfg.block_size, m.kv_heads, m.head_dim)
        self.fp8 = dt == torch.float8_e4m3fn

        def make(shape):
            if self.fp8:  # bytes, viewed as e4m3 (zero bytes are +0.0)
                t = (torch.zeros if zero else torch.empty)(shape, dtype=torch.uint8,
                                                           device=self.device)
                return t.view(dt)
            return (torch.zeros if zero else torch.empty)(shape, dtype=dt, device=self.device)

        self.layered = layered
        if layered:
            self.pool = LayeredPool([make(per_layer) for _ in range(m.n_layer)])
        else:
            self.pool = make((m.n_layer, *per_layer))
        # FP8 pools: per-(layer, kv head) scales, stored value = x / scale
        self.k_scales = self.v_scales = None
        if self.fp8:
            self.k_scales = torch.ones((m.n_layer, m.kv_heads), dtype=torch.float32,
                                       device=self.device)
            self.v_scales = torch.ones_like(self.k_scales)
        self._free = list(range(kv_cfg.num_blocks - 1, -1, -1))

    def set_scales(self, k_scales, v_scales) -> None:
        """FP8 pools: the [n_layer, n_kv_head] quantisation scales used by
        write_kv (and to be passed to the decode with ``layer_scales``)."""
        if not self.fp8:
            raise ValueError("scales apply to FP8 (e4m3) pools only")
        self.k_scales.copy_(torch.as_tensor(k_scales, dtype=torch.float32))
        self.v_scales.copy_(torch.as_tensor(v_scales, dtype=torch.float32))

    def layer_scales(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """FP8 pools: (k_scale, v_scale) [n_kv_head] of one layer."""
        return self.k_scales[layer], self.v_scales[layer]

    # -- block accounting --------------------------------------------------
    @property
    def num_free_blocks(self) -> int:
        return len(self._free)

    def blocks_for(self, num_tokens: int) -> int:
        return -(-num_tokens // self.kv_cfg.block_size)

    def allocate(self, token_ids) -> Allocation:
        ids = list(token_ids)
        n = self.blocks_for(len(ids))
        if n > len(self._free):
            raise MemoryError(f"KV pool exhausted: need {n} blocks, {len(self._free)} free")
        blocks = [self._free.pop() for _ in range(n)]
        return Allocation(blocks, len(ids), ids)

    def free(self, block_ids) -> None:
        self._free.extend(reversed(list(block_ids)))

    def capacity_headroom(self) -> dict:
        """Free blocks and the margin of the largest single pool tensor below
        2^31 elements (the reference's int32 wall, docs/REPORT.md:171-175).
        The B200 kernels index in 64 bits, so a negative margin is still
        served correctly; it is reported for callers that use torch indexing."""
        m, kv = self.model_cfg, self.kv_cfg
        per_layer = 2 * kv.num_blocks * kv.block_size * m.kv_heads * m.head_dim
        biggest = per_layer if self.layered else per_layer * m.n_layer
        per_block = 2 * kv.block_size * m.kv_heads * m.head_dim * (1 if self.layered else m.n_layer)
        return {"free_blocks": len(self._free), "used_blocks": kv.num_blocks - len(self._free),
                "largest_tensor_elements": biggest,
                "int32_margin_elements": INT32_MAX - biggest,
                "int32_margin_blocks": (INT32_MAX - biggest) // per_block}

    # -- views ---------------------------------------------------------------
    def layer_kv(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(K, V) of one layer as [NB, BS, HKV, D] views."""
        return self.pool[layer, 0], self.pool[layer, 1]

    def block_table(self, allocations, max_blocks: int | None = None) -> torch.Tensor:
        mb = max_blocks or max(len(a.block_ids) for a in allocations)
        bt = torch.zeros((len(allocations), mb), dtype=torch.int32)
        for i, a in enumerate(allocations):
            bt[i, :len(a.block_ids)] = torch.tensor(a.block_ids, dtype=torch.int32)
        return bt.to(self.device)

    # -- decode-step append -----------------------------------------------------
    def append_kv(self, block_tables, positions, k_new, v_new) -> None:
        """Write one new token per sequence for every layer (a decode step).

        k_new, v_new: [n_layer, B, n_kv_head, head_dim] (any device; fp32 /
        fp16 / bf16); sequence b's token lands at position positions[b]
        (< 0: none) through row b of block_tables."""
        from . import ops
        n_layer = self.model_cfg.n_layer
        ks = [self.pool[layer, 0] for layer in range(n_layer)]
        vs = [self.pool[layer, 1] for layer in range(n_layer)]
        empty = torch.empty(0)
        ops.append_kv(ks, vs, torch.as_tensor(block_tables), torch.as_tensor(positions),
                      torch.as_tensor(k_new), torch.as_tensor(v_new),
                      self.k_scales if self.fp8 else empty,
                      self.v_scales if self.fp8 else empty)

    def decode_step(self, q_layers, block_tables, context_lens, k_new=None, v_new=None,
                    scale: float | None = None):
        """One decode step of the engine: for every layer, the sequences' new
        K / V row appended at position context_lens[b] - 1 and the attention
        over the grown context, in one launch per layer (pa_decode_layer_step).

        q_layers: [n_layer, B, n_head, head_dim] (fp32 / fp16 / bf16; the
        outputs have the same dtype); k_new, v_new: [n_layer, B, n_kv_head,
        head_dim] or None (nothing appended); context_lens counts the new
        token.  Returns [n_layer, B, n_head, head_dim]."""
        from . import ops
        n_layer = self.model_cfg.n_layer
        d = q_layers.shape[-1]
        sc = d ** -0.5 if scale is None else float(scale)
        bt = torch.as_tensor(block_tables).to(self.device, torch.int32)
        ctx = torch.as_tensor(context_lens).to(self.device, torch.int32)
        empty = torch.empty(0, device=self.device)
        outs = []
        for layer in range(n_layer):
            kc, vc = self.pool[layer, 0], self.pool[layer, 1]
            kn = empty if k_new is None else k_new[layer]
            vn = empty if v_new is None else v_new[layer]
            outs.append(ops.decode_layer_step(q_layers[layer], kc, vc, bt, ctx, sc, kn, vn))
        return torch.stack(outs)

    # -- writer ----------------------------------------------------------------
    _IDS_CACHE_MAX = 4096

    def _device_ids(self, block_ids) -> torch.Tensor:
        """Device int32 copy of a block-id list, kept by content: a sequence
        written chunk by chunk (or re-written) reuses its copy, so the writer
        does not upload its block ids from pageable memory on every call (a
        synchronous copy that would stall the stream)."""
        arr = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32).reshape(-1))
        key = arr.tobytes()
        cache = self.__dict__.setdefault("_ids_cache", {})
        ids = cache.pop(key, None)
        if ids is None:
            ids = torch.from_numpy(arr.copy()).to(self.device)
            if len(cache) >= self._IDS_CACHE_MAX:
                cache.pop(next(iter(cache)))
        cache[key] = ids  # most recently used last
        return ids

    def write_kv_batch(self, block_id_lists, starts, ks, vs) -> None:
        """write_kv for several sequences in one call (one kernel launch for up
        to 32 sequences): entry i of each argument is one write_kv call's
        (block_ids, start, k, v).  Sequences must not share pool rows."""
        from . import ops

        def dev(x):
            t = torch.from_numpy(np.ascontiguousarray(x)) if isinstance(x, np.ndarray) else x
            if t.device.type == "cpu":
                t = t.pin_memory().to(self.device, non_blocking=True)
            return t

        ids = [b.to(device=self.device, dtype=torch.int32) if isinstance(b, torch.Tensor)
               else self._device_ids(b) for b in block_id_lists]
        n_layer = self.model_cfg.n_layer
        kl = [self.pool[layer, 0] for layer in range(n_layer)]
        vl = [self.pool[layer, 1] for layer in range(n_layer)]
        empty = torch.empty(0)
        ops.write_kv_batch(kl, vl, ids, [int(s) for s in starts], [dev(k) for k in ks],
                           [dev(v) for v in vs], self.k_scales if self.fp8 else empty,
                           self.v_scales if self.fp8 else empty)

    def write_kv(self, block_ids, start: int, k, v) -> None:
        """Write K/V of one sequence for every layer.

        k, v: [n_layer, n_kv_head, n_tok, head_dim] numpy arrays or tensors
        (any device; fp32/fp16/bf16).  Token t lands at sequence position
        start + t, i.e. row (start+t) % BS of block block_ids[(start+t)//BS]."""
        from . import ops

        def dev(x):
            t = torch.from_numpy(np.ascontiguousarray(x)) if isinstance(x, np.ndarray) else x
            if t.device.type == "cpu":
                t = t.pin_memory().to(self.device, non_blocking=True)
            return t

        if isinstance(block_ids, torch.Tensor):
            ids = block_ids.to(device=self.device, dtype=torch.int32)
        else:
            ids = self._device_ids(block_ids)
        n_layer = self.model_cfg.n_layer
        ks = [self.pool[layer, 0] for layer in range(n_layer)]
        vs = [self.pool[layer, 1] for layer in range(n_layer)]
        if self.fp8:
            ops.write_kv_scaled(ks, vs, ids, int(start), dev(k), dev(v), self.k_scales,
                                self.v_scales)
        else:
            ops.write_kv(ks, vs, ids, int(start), dev(k), dev(v))
