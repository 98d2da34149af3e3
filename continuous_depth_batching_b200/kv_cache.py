"""Looped paged-KV cache: slot arithmetic, the FIFO block pool and the device block table.

* Slot arithmetic restates ``looped_cdb/kv_cache_policy.py`` (``resolve_kv_slots_per_layer``
  ``:52-79``, ``kv_slot_for_step`` ``:82-103``, ``kv_layer_index`` ``:106-128``,
  ``LoopedKvLayout.exit_copy_layer_groups`` ``:235-258``) for the four policies.
* :class:`BlockPool` is the host owner of physical block ids with the reference's FIFO order
  (``continuous_batching/cache_manager.py:33-91``: allocate pops the left of a deque, free
  appends in the request's block order), so block ids - and every block table - come out
  bit-identical to the reference's for the same allocate/free sequence.
* :class:`PagedKVPool` holds the device side: one bf16 allocation
  ``[num_cache_layers, 2, (num_blocks+2)*block_size, Hkv, D]`` (each cache layer's K and V are
  exactly the reference's ``[(nb+2)*bs, Hkv, D]`` tensors, ``continuous_batching/cache.py:131-145``)
  and a device block table ``[resident slots, ceil(max_model_len/bs)]`` that the host updates by
  edits only (new block ids), never by re-uploading rows per launch.
"""

from __future__ import annotations

from collections import deque

import torch

from . import _lib

KV_CACHE_POLICIES = ("depth_indexed", "last_exited", "single", "first_then_shared")


def resolve_kv_slots_per_layer(policy: str, *, total_recurrent_steps: int, requested_slots: int | None = None) -> int:
    if policy not in KV_CACHE_POLICIES:
        raise ValueError(f"Unsupported KV cache policy {policy!r}; expected one of {KV_CACHE_POLICIES}")
    if total_recurrent_steps <= 0:
        raise ValueError(f"total_recurrent_steps must be positive, got {total_recurrent_steps}")
    fixed = {"depth_indexed": total_recurrent_steps, "last_exited": total_recurrent_steps, "single": 1}
    if policy in fixed:
        slots = fixed[policy]
        if requested_slots is not None and requested_slots != slots:
            raise ValueError(f"Policy {policy!r} uses exactly {slots} KV slot(s) per layer, got {requested_slots}")
        return slots
    slots = 2 if requested_slots is None else requested_slots
    if slots <= 0:
        raise ValueError(f"kv_slots_per_layer must be positive, got {slots}")
    if slots > total_recurrent_steps:
        raise ValueError(f"kv_slots_per_layer={slots} exceeds total_recurrent_steps={total_recurrent_steps}")
    return slots


def kv_slot_for_step(recurrent_step: int, *, policy: str, slots_per_layer: int) -> int:
    if policy in ("depth_indexed", "last_exited"):
        return recurrent_step
    if policy == "single":
        return 0
    return min(recurrent_step, slots_per_layer - 1)


def copies_exit_kv(policy: str) -> bool:
    return policy == "last_exited"


class BlockPool:
    """Physical block ids in FIFO order, per-request block lists, and pending device edits."""

    def __init__(self, num_blocks: int, block_size: int, width: int) -> None:
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.width = width
        self.reset()

    def reset(self) -> None:
        self.free: deque[int] = deque(range(self.num_blocks))
        self.tables: dict[int, list[int]] = {}
        self.edits: list[int] = []
        self.peak = 0

    @property
    def num_free(self) -> int:
        return len(self.free)

    def allocate(self, key: int, slot: int, n: int) -> bool:
        """Append ``n`` blocks to request ``key`` (resident slot ``slot``); False if short."""

        if n > len(self.free):
            return False
        blocks = self.tables.setdefault(key, [])
        if len(blocks) + n > self.width:
            raise ValueError(f"request needs {len(blocks) + n} blocks, above the block-table width {self.width}")
        for _ in range(n):
            b = self.free.popleft()
            self.edits.extend((slot, len(blocks), b))
            blocks.append(b)
        self.peak = max(self.peak, self.num_blocks - len(self.free))
        return True

    def release(self, key: int) -> None:
        self.free.extend(self.tables.pop(key, []))

    def take_edits(self) -> list[int]:
        edits, self.edits = self.edits, []
        return edits


class PagedKVPool:
    """Device KV storage plus the device block table, sized once per engine."""

    def __init__(
        self,
        *,
        num_cache_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        max_model_len: int,
        resident_slots: int,
        device: torch.device,
        dtype: torch.dtype = torch.bfloat16,
    ) -> None:
        self.num_cache_layers = num_cache_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.rows = (num_blocks + 2) * block_size
        self.width = -(-max_model_len // block_size)
        self.device = device
        self.kv = torch.zeros(
            (num_cache_layers, 2, self.rows, num_kv_heads, head_dim), dtype=dtype, device=device
        )
        self.block_table = torch.full((resident_slots, self.width), -1, dtype=torch.int32, device=device)
        self.pool = BlockPool(num_blocks, block_size, self.width)

    def key_cache(self, cache_layer: int) -> torch.Tensor:
        return self.kv[cache_layer, 0]

    def value_cache(self, cache_layer: int) -> torch.Tensor:
        return self.kv[cache_layer, 1]

    def flush_edits(self, upload, stream: torch.cuda.Stream) -> None:
        """Push pending block-table edits to the device table on ``stream``.

        ``upload(list[int]) -> device int32 tensor`` stages the edit triples asynchronously.
        """

        edits = self.pool.take_edits()
        if not edits:
            return
        dev = upload(edits)
        _lib.call(
            "cdb_block_table_update",
            _lib.ptr(self.block_table),
            self.block_table.stride(0),
            _lib.ptr(dev),
            len(edits) // 3,
            stream.cuda_stream,
        )
