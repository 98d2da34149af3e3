"""The reference's inner attention seam on the B200 kernels.

The reference's models reach attention through HF transformers' registry key
``"paged|flash_attention_3"`` (``transformers/integrations/flash_paged.py:8-122``): the model
applies its projections and RoPE, then calls ``paged_attention_forward(module, q, k, v,
attention_mask, cache, cu_seq_lens_q, cu_seq_lens_k, max_seqlen_q, max_seqlen_k, block_table,
read_index=..., write_index=...)`` and gets ``(out [T, H, D], None)`` back. This module provides
a function with that signature on this library's kernels, so the reference's own models and
engine (``OuroAttention.forward`` ``modeling_ouro.py:377-432``, ``HuginnAttention.forward``
``modeling_huginn.py:244-302``) run their attention here after ``register()``:

* ``block_table`` given (decode): append k/v at ``cache_seqlens[b] = cu_seq_lens_k[b+1] -
  cu_seq_lens_k[b] - 1`` and attend over positions ``0 .. cache_seqlens[b]`` through
  ``block_table[group][b]``; rows with ``cache_seqlens[b] < 0`` are padding. One launch of the
  fused append + ragged paged decode kernel (``cdb_paged_decode_attn_append``, append 2 with no
  rotation - the model has rotated q and k already), plus its per-launch work plan.
* ``block_table`` absent (varlen prefill): ``cache.update`` writes the new rows (the reference's
  own cache code), then causal attention of every query chunk over its sequence's cached keys
  with the mask aligned bottom-right, on the tiled prefill kernel (``cdb_prefill_attention``),
  which reads the keys through block tables built from ``read_index``.

The kernels address K and V of every cache layer through one pool ``[layers, 2, rows, H, D]``.
The reference cache (``PagedAttentionCache``, ``continuous_batching/cache.py``) keeps two
separate ``[rows, H, D]`` tensors per layer, so ``bind_paged_cache`` moves them once into one pool
of that shape and puts views of it back into ``cache.key_cache`` / ``cache.value_cache``; every
reference code path (``update``, block copies, offloading) then works on the pool unchanged. The
first call binds a cache that is not bound yet; that call allocates, so it must not run while a
stream is being captured (it raises there). Serves MHA (``num_key_value_heads == num_heads``),
block size 16, full attention (no sliding window), head_dim 64, 96 or 128, bf16.
"""

from __future__ import annotations

import torch

from . import _lib
from . import ops as _ops

ATTENTION_KEY = "paged|flash_attention_3"
BLOCK = 16
PREFILL_TILE_ROWS = 64


def bind_paged_cache(cache) -> torch.Tensor:
    """Move ``cache``'s per-layer K/V tensors into one ``[layers, 2, rows, H, D]`` pool (contents
    kept) and make ``cache.key_cache[j]`` / ``cache.value_cache[j]`` views of it. Returns the pool;
    a cache already bound returns its pool."""

    pool = getattr(cache, "_cdb_pool", None)
    if pool is not None:
        return pool
    keys, values = list(cache.key_cache), list(cache.value_cache)
    if not keys or len(keys) != len(values):
        raise ValueError("the cache has no per-layer key/value tensors to bind")
    shape, dtype, dev = keys[0].shape, keys[0].dtype, keys[0].device
    if any(t.shape != shape or t.dtype != dtype or t.device != dev for t in keys + values):
        raise ValueError("every cache layer must hold K and V tensors of one shape, dtype and device")
    if dtype != torch.bfloat16 or dev.type != "cuda" or len(shape) != 3:
        raise NotImplementedError("the B200 attention kernels serve bf16 CUDA caches of shape [rows, heads, head_dim]")
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("bind_paged_cache allocates the pool: call it (or the first attention call) before capture")
    pool = torch.empty((len(keys), 2, *shape), dtype=dtype, device=dev)
    for j, (k, v) in enumerate(zip(keys, values, strict=True)):
        pool[j, 0].copy_(k)
        pool[j, 1].copy_(v)
        cache.key_cache[j] = pool[j, 0]
        cache.value_cache[j] = pool[j, 1]
    cache._cdb_pool = pool
    return pool


def _check_cache(cache, module, q: torch.Tensor, k: torch.Tensor) -> tuple[int, int, int, int]:
    heads, head_dim = q.shape[1], q.shape[3]
    if k.shape[1] != heads:
        raise NotImplementedError("the B200 paged decode kernel serves MHA (num_key_value_heads == num_heads)")
    if int(cache.block_size) != BLOCK:
        raise NotImplementedError(f"the B200 paged kernels use block size {BLOCK}, got {cache.block_size}")
    sliding = getattr(cache, "sliding_windows", {}).get(module.layer_idx, 1)
    if sliding not in (1, None) or getattr(module, "sliding_window", None):
        raise NotImplementedError("sliding-window attention is not served by the B200 paged kernels")
    group_idx, layer_in_group = cache.layer_index_to_group_indices[module.layer_idx]
    return heads, head_dim, group_idx, layer_in_group


_ROWS: dict[int, torch.Tensor] = {}


def _arange(dev: torch.device, n: int) -> torch.Tensor:
    idx = dev.index
    cur = _ROWS.get(idx)
    if cur is None or cur.numel() < n:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("paged_attention_forward: make one call with the largest batch before capture")
        cur = torch.arange(max(n, 1024), dtype=torch.int32, device=dev)
        _ROWS[idx] = cur
    return cur[:n]


def paged_attention_forward(
    module: torch.nn.Module,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    attention_mask: torch.Tensor | None,
    cache,
    cu_seq_lens_q: torch.Tensor,
    cu_seq_lens_k: torch.Tensor | dict,
    max_seqlen_q: int,
    max_seqlen_k: int | dict,
    block_table: torch.Tensor | None = None,
    **kwargs,
) -> tuple[torch.Tensor, None]:
    """``paged|flash_attention_3`` on the B200 kernels: ``q [1,H,T,D]``, ``k/v [1,H,T,D]`` in,
    ``(out [T,H,D], None)`` out, the cache updated in place (signature of ``flash_paged.py:8-21``)."""

    del attention_mask, max_seqlen_q, max_seqlen_k
    if isinstance(cu_seq_lens_k, dict):
        cu_seq_lens_k = cu_seq_lens_k["full_attention"]
    heads, head_dim, group_idx, layer_in_group = _check_cache(cache, module, q, k)
    pool = bind_paged_cache(cache)
    scale = float(module.scaling)
    tokens = q.shape[2]
    hd = heads * head_dim
    # [1, H, T, D] -> [T, H*D] rows, as the kernels read them
    q_rows = q[0].transpose(0, 1).reshape(tokens, hd)

    if block_table is not None:
        k_rows = k[0].transpose(0, 1).reshape(tokens, hd)
        v_rows = v[0].transpose(0, 1).reshape(tokens, hd)
        qkv = torch.cat([q_rows, k_rows, v_rows], dim=1).contiguous()
        item_pos = (cu_seq_lens_k[1 : tokens + 1] - cu_seq_lens_k[:tokens] - 1).to(torch.int32).contiguous()
        table = block_table[group_idx]
        if table.dtype != torch.int32:
            table = table.to(torch.int32)
        table = table.contiguous()
        out = torch.zeros(tokens, hd, dtype=q.dtype, device=q.device)
        torch.ops.cdb.paged_decode_attention(
            qkv, out, pool, layer_in_group, table, _arange(q.device, tokens), item_pos, None, None, None, 0, heads,
            head_dim, scale,
        )
        return out.view(tokens, heads, head_dim), None

    # Varlen prefill: the reference's cache write, then tiled causal attention over the pool.
    cache.update(
        key_states=k, value_states=v, layer_idx=module.layer_idx, read_index=kwargs["read_index"],
        write_index=kwargs["write_index"],
    )
    read = kwargs["read_index"][group_idx].tolist()
    cu_q = [int(x) for x in cu_seq_lens_q.tolist()]
    cu_k = [int(x) for x in cu_seq_lens_k.tolist()]
    tiles: list[tuple[int, int, int, int]] = []
    tables: list[list[int]] = []
    for b in range(len(cu_q) - 1):
        q0, q1, k0, k1 = cu_q[b], cu_q[b + 1], cu_k[b], cu_k[b + 1]
        rows = read[k0:k1]
        blocks = [r // BLOCK for r in rows[::BLOCK]]
        if any(r != blocks[i // BLOCK] * BLOCK + i % BLOCK for i, r in enumerate(rows)):
            raise NotImplementedError("the prefill read index is not whole cache blocks in position order")
        seq = len(tables)
        tables.append(blocks)
        first = (k1 - k0) - (q1 - q0)  # bottom-right aligned causal mask
        for s in range(q0, q1, PREFILL_TILE_ROWS):
            n = min(PREFILL_TILE_ROWS, q1 - s)
            tiles.append((s, n, seq, first + (s - q0)))
    out = torch.zeros(tokens, hd, dtype=q.dtype, device=q.device)
    if not tiles:
        return out.view(tokens, heads, head_dim), None
    width = max(1, max(len(t) for t in tables))
    table = torch.full((len(tables), width), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        table[i, : len(t)] = torch.tensor(t, dtype=torch.int32)
    table = table.to(q.device)
    tile_t = torch.tensor(tiles, dtype=torch.int32).to(q.device)
    q_rows = q_rows.contiguous()
    status = _ops._status(q)
    _lib.call(
        "cdb_prefill_attention", _lib.ptr(q_rows), q_rows.stride(0), 0, 0, _lib.ptr(out), out.stride(0),
        _lib.ptr(pool), pool.shape[0], pool.shape[2], layer_in_group, _lib.ptr(table), table.stride(0),
        _lib.ptr(tile_t), len(tiles), heads, head_dim, BLOCK, scale, _lib.ptr(status),
        torch.cuda.current_stream(q.device).cuda_stream,
    )
    return out.view(tokens, heads, head_dim), None


def register(key: str = ATTENTION_KEY) -> None:
    """Install ``paged_attention_forward`` in transformers' attention registry under ``key``.

    A model whose ``config._attn_implementation`` is ``key`` (the reference sets
    ``"paged|flash_attention_3"`` for its CDB engine) then runs its paged attention here."""

    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    ALL_ATTENTION_FUNCTIONS[key] = paged_attention_forward
