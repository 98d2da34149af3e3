"""CPU restatement of the paged FlashAttention contract the reference decode path calls.

TEST INFRASTRUCTURE ONLY. This module is the checker: only ``tests/``, the golden
fixture generator, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline may use
it. The product path never imports it.

The reference reaches attention through HF transformers' ``paged_attention_forward``
(``transformers/integrations/flash_paged.py:8-123``, transformers 5.5.0 here, 5.9.0
pinned by the reference ``uv.lock:1973-1974``), which forwards to the FlashAttention-3
binary (``flash-attn-3==3.0.0``, ``uv.lock:429-431``; not present in this image). Its
two branches are restated from that published contract:

* ``block_table is None`` (varlen prefill, ``flash_paged.py:50-81``): write the new k/v
  rows through ``cache.update`` (``continuous_batching/cache.py:284-318``), then causal
  attention per sequence with the mask aligned bottom-right (query ``i`` of a length-``Lq``
  chunk sees keys ``0 .. Lk-Lq+i``).
* ``block_table`` given (decode, ``flash_paged.py:84-122``): ``seqlen_b =
  cu_seq_lens_k[b+1]-cu_seq_lens_k[b]-1``; rows with ``seqlen_b < 0`` are padding and
  are skipped; write k/v at block ``block_table[b][seqlen_b // bs]`` offset
  ``seqlen_b % bs``, then attend over positions ``0 .. seqlen_b`` gathered through the
  block table.

Scores and softmax are computed in fp32 (FlashAttention accumulates in fp32); the output
is rounded once to the query dtype.
"""

from __future__ import annotations

import torch


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal_offset: int | None) -> torch.Tensor:
    """Softmax attention for one sequence. q [Lq,H,D], k/v [Lk,Hkv,D] -> [Lq,H,D] fp32."""

    h, hkv = q.shape[1], k.shape[1]
    if hkv != h:
        k = k.repeat_interleave(h // hkv, dim=1)
        v = v.repeat_interleave(h // hkv, dim=1)
    qf, kf, vf = q.float(), k.float(), v.float()
    scores = torch.einsum("qhd,khd->hqk", qf, kf) * scale
    if causal_offset is not None:
        lq, lk = q.shape[0], k.shape[0]
        qi = torch.arange(lq).unsqueeze(1)
        kj = torch.arange(lk).unsqueeze(0)
        scores = scores.masked_fill((kj > qi + causal_offset).unsqueeze(0), float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("hqk,khd->qhd", probs, vf)


def cpu_paged_attention_forward(
    module,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    attention_mask,
    cache,
    cu_seq_lens_q: torch.Tensor,
    cu_seq_lens_k,
    max_seqlen_q: int,
    max_seqlen_k,
    block_table: torch.Tensor | None = None,
    **kwargs,
):
    """Drop-in for ``ALL_ATTENTION_FUNCTIONS["paged|flash_attention_3"]`` on CPU.

    Same signature and return convention as ``flash_paged.paged_attention_forward``:
    ``q [1,H,T,D]``, ``k/v [1,Hkv,T,D]`` in, ``(out [T,H,D], None)`` out.
    """

    del attention_mask, max_seqlen_q
    if isinstance(cu_seq_lens_k, dict):
        cu_seq_lens_k = cu_seq_lens_k["full_attention"]
        max_seqlen_k = max_seqlen_k["full_attention"] if isinstance(max_seqlen_k, dict) else max_seqlen_k
    scale = float(module.scaling)
    cu_q = [int(x) for x in cu_seq_lens_q.tolist()]
    cu_k = [int(x) for x in cu_seq_lens_k.tolist()]
    q_rows = q[0].transpose(0, 1)  # [T, H, D]

    if block_table is None:
        k_all, v_all = cache.update(
            key_states=k,
            value_states=v,
            layer_idx=module.layer_idx,
            read_index=kwargs["read_index"],
            write_index=kwargs["write_index"],
        )
        out = torch.zeros(q_rows.shape, dtype=torch.float32)
        for b in range(len(cu_q) - 1):
            q0, q1, k0, k1 = cu_q[b], cu_q[b + 1], cu_k[b], cu_k[b + 1]
            if q1 <= q0:
                continue
            out[q0:q1] = _attend(q_rows[q0:q1], k_all[k0:k1], v_all[k0:k1], scale, (k1 - k0) - (q1 - q0))
        return out.to(q.dtype), None

    group_idx, layer_in_group = cache.layer_index_to_group_indices[module.layer_idx]
    bs = cache.block_size
    k_cache = cache.key_cache[layer_in_group].view(-1, bs, cache.num_key_value_heads, cache.head_dim)
    v_cache = cache.value_cache[layer_in_group].view(-1, bs, cache.num_key_value_heads, cache.head_dim)
    table = block_table[group_idx]
    k_new = k[0].transpose(0, 1)  # [B, Hkv, D]
    v_new = v[0].transpose(0, 1)
    batch = k_new.shape[0]
    out = torch.zeros(q_rows.shape, dtype=torch.float32)
    for b in range(batch):
        seqlen = cu_k[b + 1] - cu_k[b] - 1
        if seqlen < 0:
            continue
        blk = int(table[b, seqlen // bs])
        k_cache[blk, seqlen % bs] = k_new[b]
        v_cache[blk, seqlen % bs] = v_new[b]
        n_blocks = seqlen // bs + 1
        ids = table[b, :n_blocks].long()
        keys = k_cache[ids].reshape(-1, k_cache.shape[2], k_cache.shape[3])[: seqlen + 1]
        vals = v_cache[ids].reshape(-1, v_cache.shape[2], v_cache.shape[3])[: seqlen + 1]
        out[b : b + 1] = _attend(q_rows[b : b + 1], keys, vals, scale, None)
    return out.to(q.dtype), None
