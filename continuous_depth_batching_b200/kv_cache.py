"""Looped paged-KV cache: slot arithmetic, the FIFO block pool and the device block table.

* Slot arithmetic restates ``looped_cdb/kv_cache_policy.py`` (``resolve_kv_slots_per_layer``
  ``:52-79``, ``kv_slot_for_step`` ``:82-103``, ``kv_layer_index`` ``:106-128``,
  ``LoopedKvLayout`` ``:135-258``) for the four policies.
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


class LoopedKvLayout:
    """Cache-layer numbering of a looped model (``LoopedKvLayout``, ``kv_cache_policy.py:135-258``):
    prelude layers first (one slot each), then the core layers slot-major (slot s, layer l ->
    prelude + s * core + l), then the coda layers. Ouro is all core; Huginn has all three stages."""

    def __init__(self, *, num_prelude_layers: int, num_core_layers: int, num_coda_layers: int,
                 total_recurrent_steps: int, policy: str, requested_slots: int | None = None) -> None:
        if num_prelude_layers < 0 or num_coda_layers < 0:
            raise ValueError("prelude and coda layer counts must be non-negative")
        if num_core_layers <= 0:
            raise ValueError(f"num_core_layers must be positive, got {num_core_layers}")
        self.num_prelude_layers = num_prelude_layers
        self.num_core_layers = num_core_layers
        self.num_coda_layers = num_coda_layers
        self.total_recurrent_steps = total_recurrent_steps
        self.policy = policy
        self.slots_per_layer = resolve_kv_slots_per_layer(
            policy, total_recurrent_steps=total_recurrent_steps, requested_slots=requested_slots
        )

    @property
    def num_cache_layers(self) -> int:
        return self.num_prelude_layers + self.slots_per_layer * self.num_core_layers + self.num_coda_layers

    def slot_for_step(self, recurrent_step: int) -> int:
        if not 0 <= recurrent_step < self.total_recurrent_steps:
            raise ValueError(f"recurrent_step must be in [0, {self.total_recurrent_steps}), got {recurrent_step}")
        return kv_slot_for_step(recurrent_step, policy=self.policy, slots_per_layer=self.slots_per_layer)

    @staticmethod
    def _check(layer: int, count: int, stage: str) -> None:
        if not 0 <= layer < count:
            raise ValueError(f"{stage} layer must be in [0, {count}), got {layer}")

    def prelude_layer_index(self, layer: int) -> int:
        self._check(layer, self.num_prelude_layers, "prelude")
        return layer

    def core_slot_layer_index(self, slot: int, layer: int) -> int:
        """Cache layer of core layer ``layer`` in KV slot ``slot``."""

        self._check(layer, self.num_core_layers, "core")
        if not 0 <= slot < self.slots_per_layer:
            raise ValueError(f"slot must be in [0, {self.slots_per_layer}), got {slot}")
        return self.num_prelude_layers + slot * self.num_core_layers + layer

    def core_layer_index(self, layer: int, recurrent_step: int) -> int:
        return self.core_slot_layer_index(self.slot_for_step(recurrent_step), layer)

    def coda_layer_index(self, layer: int) -> int:
        self._check(layer, self.num_coda_layers, "coda")
        return self.num_prelude_layers + self.slots_per_layer * self.num_core_layers + layer

    def exit_copy_layer_groups(self, exit_step: int) -> list[tuple[int, list[int]]]:
        """Per core layer: (the cache layer the exit step wrote, the same layer in every deeper
        slot). Empty when no deeper slot exists; only ``last_exited`` copies."""

        src = self.slot_for_step(exit_step)
        return [
            (
                self.core_slot_layer_index(src, layer),
                [self.core_slot_layer_index(t, layer) for t in range(src + 1, self.slots_per_layer)],
            )
            for layer in range(self.num_core_layers)
            if src + 1 < self.slots_per_layer
        ]


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
        self.row_bytes = num_kv_heads * head_dim * self.kv.element_size()
        self.num_host_blocks = 0
        self.host_pool: torch.Tensor | None = None

    @property
    def block_bytes(self) -> int:
        """Bytes of one block over every cache layer, K and V (``OffloadingManager._bytes_per_block``,
        ``offloading_manager.py:146-157``)."""

        return 2 * self.num_cache_layers * self.block_size * self.row_bytes

    def attach_host_pool(self, num_host_blocks: int) -> None:
        """Pinned host swap pool of ``num_host_blocks`` blocks for offload preemption, laid out
        ``[host_blocks, cache_layers * 2, block_size * row_bytes]``."""

        self.num_host_blocks = max(0, int(num_host_blocks))
        self.host_pool = None
        if self.num_host_blocks:
            self.host_pool = torch.empty(
                (self.num_host_blocks, 2 * self.num_cache_layers, self.block_size * self.row_bytes),
                dtype=torch.uint8,
                pin_memory=True,
            )

    def host_copy(self, device_blocks: list[int], host_blocks: list[int], to_host: bool, stream) -> None:
        """Copy whole blocks (every cache layer, K and V) between the device pool and the host pool
        on ``stream`` (``cdb_kv_blocks_host_copy``)."""

        if len(device_blocks) != len(host_blocks):
            raise ValueError("device_blocks and host_blocks must pair up")
        if not device_blocks:
            return
        if self.host_pool is None:
            raise RuntimeError("no host swap pool is attached")
        dev = torch.tensor(device_blocks, dtype=torch.int32)
        host = torch.tensor(host_blocks, dtype=torch.int32)
        _lib.call(
            "cdb_kv_blocks_host_copy", _lib.ptr(self.kv), self.num_cache_layers, self.rows, self.row_bytes,
            self.block_size, self.num_blocks, dev.data_ptr(), self.host_pool.data_ptr(), self.num_host_blocks,
            host.data_ptr(), len(device_blocks), int(to_host), stream.cuda_stream,
        )

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
