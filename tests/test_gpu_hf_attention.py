"""The ``paged|flash_attention_3`` hook (``hf_attention.paged_attention_forward``) against the CPU
restatement of the same contract (``oracle/paged_attention.py``), both called with the
reference's own argument layout: ``q/k/v [1, H, T, D]``, ``cu_seq_lens``, ``block_table
[groups, B, W]`` with ``seqlen = -1`` padding rows (decode), ``read_index`` / ``write_index`` per
layer group (prefill), and a cache object with the ``PagedAttentionCache`` attributes the hook
uses (``key_cache``/``value_cache`` per layer, ``layer_index_to_group_indices``, ``update``).

Tolerance: 2e-2 max-abs on the bf16 attention output (the attention kernel tests' bound); the
cache rows written by the call must equal the oracle's exactly.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from continuous_depth_batching_b200 import hf_attention
from oracle.paged_attention import cpu_paged_attention_forward

pytestmark = pytest.mark.gpu
BS = 16


class Cache:
    """The attributes and ``update`` (full-attention branch) of transformers' PagedAttentionCache."""

    def __init__(self, layers: int, rows: int, heads: int, d: int, device, gen):
        self.block_size = BS
        self.num_key_value_heads = heads
        self.head_dim = d
        self.layer_index_to_group_indices = {j: (0, j) for j in range(layers)}
        self.sliding_windows = {j: 1 for j in range(layers)}
        self.key_cache = [torch.randn(rows, heads, d, generator=gen).to(torch.bfloat16).to(device) for _ in range(layers)]
        self.value_cache = [torch.randn(rows, heads, d, generator=gen).to(torch.bfloat16).to(device) for _ in range(layers)]

    def copy_to(self, device):
        c = Cache.__new__(Cache)
        c.__dict__.update({k: v for k, v in self.__dict__.items() if k not in ("key_cache", "value_cache", "_cdb_pool")})
        c.key_cache = [t.to(device).clone() for t in self.key_cache]
        c.value_cache = [t.to(device).clone() for t in self.value_cache]
        return c

    def update(self, key_states, value_states, layer_idx, read_index, write_index):
        group, j = self.layer_index_to_group_indices[layer_idx]
        k = key_states.transpose(1, 2).squeeze(0)
        v = value_states.transpose(1, 2).squeeze(0)
        self.key_cache[j][write_index[group]] = k
        self.value_cache[j][write_index[group]] = v
        return self.key_cache[j][read_index[group]], self.value_cache[j][read_index[group]]


def _module(layer: int, d: int):
    return SimpleNamespace(layer_idx=layer, scaling=d**-0.5, config=SimpleNamespace(_attn_implementation="paged|flash_attention_3"))


@pytest.mark.parametrize("heads,d", [(16, 128), (4, 64), (5, 96)])
def test_decode_branch_matches_cpu_contract(heads, d):
    gen = torch.Generator().manual_seed(heads * d)
    nb, b, width = 160, 20, 6
    cache = Cache(3, (nb + 2) * BS, heads, d, "cpu", gen)
    gpu_cache = cache.copy_to("cuda")
    seqlen = torch.randint(0, width * BS, (b,), generator=gen)
    seqlen[0], seqlen[1], seqlen[2] = 0, BS - 1, -1  # first row, page edge, padding row
    cu_k = torch.zeros(b + 1, dtype=torch.int32)
    cu_k[1:] = torch.cumsum(seqlen + 1, 0).to(torch.int32)
    cu_q = torch.arange(b + 1, dtype=torch.int32)
    table = torch.randperm(nb, generator=gen)[: b * width].view(1, b, width).to(torch.int32)
    q = torch.randn(1, heads, b, d, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, heads, b, d, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, heads, b, d, generator=gen).to(torch.bfloat16)
    module = _module(1, d)
    ref, _ = cpu_paged_attention_forward(module, q, k, v, None, cache, cu_q, cu_k, 1, int(seqlen.max()) + 1, table)
    for call in range(2):  # the second call binds a fresh cache copy and reuses the op scratch
        c = gpu_cache.copy_to("cuda") if call else gpu_cache
        out, none = hf_attention.paged_attention_forward(
            module, q.cuda(), k.cuda(), v.cuda(), None, c, cu_q.cuda(), cu_k.cuda(), 1, int(seqlen.max()) + 1,
            table.cuda(),
        )
        torch.cuda.synchronize()
        assert none is None and out.shape == (b, heads, d)
        live = seqlen >= 0
        err = (out.cpu().float()[live] - ref.float()[live]).abs().max().item()
        assert err < 2e-2, err
        for j in range(3):
            assert torch.equal(c.key_cache[j].cpu(), cache.key_cache[j]), j
            assert torch.equal(c.value_cache[j].cpu(), cache.value_cache[j]), j
        assert hasattr(c, "_cdb_pool")


def test_prefill_branch_matches_cpu_contract():
    heads, d = 16, 128
    gen = torch.Generator().manual_seed(5)
    nb = 64
    cache = Cache(2, (nb + 2) * BS, heads, d, "cpu", gen)
    gpu_cache = cache.copy_to("cuda")
    # three sequences: a fresh prompt, a chunk after 23 cached tokens, a long chunk after 30
    q_lens, past = [5, 17, 70], [0, 23, 30]
    perm = torch.randperm(nb, generator=gen).tolist()
    read, write, cu_q, cu_k, used = [], [], [0], [0], 0
    for ql, pl in zip(q_lens, past, strict=True):
        n = ql + pl
        blocks = perm[used : used + (n + BS - 1) // BS]
        used += len(blocks)
        rows = [blocks[i // BS] * BS + i % BS for i in range(n)]
        read += rows
        write += rows[pl:]
        cu_q.append(cu_q[-1] + ql)
        cu_k.append(cu_k[-1] + n)
    t = sum(q_lens)
    q = torch.randn(1, heads, t, d, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, heads, t, d, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, heads, t, d, generator=gen).to(torch.bfloat16)
    module = _module(1, d)
    ri, wi = [torch.tensor(read)], [torch.tensor(write)]
    cq, ck = torch.tensor(cu_q, dtype=torch.int32), torch.tensor(cu_k, dtype=torch.int32)
    ref, _ = cpu_paged_attention_forward(module, q, k, v, None, cache, cq, ck, 70, 100, None, read_index=ri, write_index=wi)
    out, _ = hf_attention.paged_attention_forward(
        module, q.cuda(), k.cuda(), v.cuda(), None, gpu_cache, cq.cuda(), ck.cuda(), 70, 100, None,
        read_index=[x.cuda() for x in ri], write_index=[x.cuda() for x in wi],
    )
    torch.cuda.synchronize()
    err = (out.cpu().float() - ref.float()).abs().max().item()
    assert err < 2e-2, err
    for j in range(2):
        assert torch.equal(gpu_cache.key_cache[j].cpu(), cache.key_cache[j])
        assert torch.equal(gpu_cache.value_cache[j].cpu(), cache.value_cache[j])
