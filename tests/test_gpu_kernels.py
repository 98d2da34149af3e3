"""Kernel-level parity of libcdb_b200 against plain PyTorch fp32 references on the GPU.

Every call goes through the C ABI (ctypes). Tolerances: exact where the op is integer or a
pure copy (argmax, embed, block-table edits, KV copy, appended K/V rows); bf16 rounding of an
identical fp32 formula otherwise (one bf16 ulp at the output scale); attention is compared with
fp32 softmax at 2e-2 max-abs (bf16 output of values of order 1).
"""

from __future__ import annotations

import math

import pytest
import torch

from continuous_depth_batching_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda"
BS = 16


def _rot_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _rope_tables(max_pos: int, d: int, theta: float = 10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).to(torch.float32) / d))
    freqs = torch.arange(max_pos, dtype=torch.float32, device=DEV)[:, None] * inv.to(DEV)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()


class AttnHarness:
    """Buffers for one attention call through the C ABI."""

    def __init__(self, n_items, heads, d, layers=2, num_blocks=512, scratch=256):
        self.h, self.d = heads, d
        self.layers = layers
        self.rows = (num_blocks + 2) * BS
        self.kv = torch.randn(layers, 2, self.rows, heads, d, device=DEV).to(torch.bfloat16)
        self.hg = 5 if d == 96 else 4
        self.cap = max(scratch * (heads // self.hg) * 64, n_items * (heads // self.hg))
        self.hdr = torch.zeros(_lib.ATTN_PLAN_HEADER_INTS, dtype=torch.int32, device=DEV)
        self.units = torch.zeros(self.cap, 4, dtype=torch.int32, device=DEV)
        self.part_o = torch.zeros(scratch * heads * 64 * d, device=DEV)
        self.part_ml = torch.zeros(scratch * heads * 64 * 2, device=DEV)
        self.counters = torch.zeros(scratch * heads, dtype=torch.int32, device=DEV)
        self.status = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.scratch = scratch
        self.num_blocks = num_blocks

    def run(self, qkv, out, layer, block_table, item_slot, item_pos, append, rope_mode, cos, sin, qk_bias=None):
        n = item_pos.numel()
        sp = torch.cuda.current_stream().cuda_stream
        _lib.call(
            "cdb_attn_plan", _lib.ptr(item_pos), n, append, self.h, self.d, BS, self.cap, self.scratch, 148,
            _lib.ptr(self.hdr), _lib.ptr(self.units), sp,
        )
        hd = self.h * self.d
        _lib.call(
            "cdb_paged_decode_attn_append", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, _lib.ptr(out), out.stride(0),
            _lib.ptr(self.kv), self.layers, self.rows, layer, _lib.ptr(block_table), block_table.stride(0),
            _lib.ptr(item_slot), _lib.ptr(item_pos), rope_mode, _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(qk_bias), append,
            _lib.ptr(self.hdr), _lib.ptr(self.units), _lib.ptr(self.part_o), _lib.ptr(self.part_ml),
            _lib.ptr(self.counters), self.scratch, n, self.h, self.d, BS, self.d**-0.5, 296, _lib.ptr(self.status), sp,
        )
        torch.cuda.synchronize()
        assert int(self.status.item()) == 0


def _make_tables(n_req, max_blocks, num_blocks, gen):
    perm = torch.randperm(num_blocks, generator=gen)
    table = torch.full((n_req, max_blocks), -1, dtype=torch.int32)
    k = 0
    for r in range(n_req):
        table[r] = perm[k : k + max_blocks].to(torch.int32)
        k += max_blocks
    return table.to(DEV)


def _reference_decode(h, qkv, kv, layer, table, slots, pos, cos, sin, append, rope=True):
    """fp32 attention over the paged cache (+ the roped new token when appending)."""

    heads, d = h.h, h.d
    hd = heads * d
    out = torch.zeros(len(pos), hd, device=DEV)
    new_k = {}
    for i, (s, p) in enumerate(zip(slots.tolist(), pos.tolist(), strict=True)):
        if p < 0:
            continue
        q = qkv[i, :hd].view(heads, d)
        k = qkv[i, hd : 2 * hd].view(heads, d)
        v = qkv[i, 2 * hd :].view(heads, d)
        if append:
            if rope:
                q = q * cos[p] + _rot_half(q) * sin[p]
                k = k * cos[p] + _rot_half(k) * sin[p]
            n_cached = p
        else:
            n_cached = p + 1
        rows = [int(table[s, t // BS]) * BS + t % BS for t in range(n_cached)]
        kc = kv[layer, 0, rows].float()
        vc = kv[layer, 1, rows].float()
        if append:
            kc = torch.cat([kc, k.float()[None]], 0)
            vc = torch.cat([vc, v.float()[None]], 0)
            new_k[i] = (k, v, int(table[s, p // BS]) * BS + p % BS)
        sc = torch.einsum("hd,thd->ht", q.float(), kc) * d**-0.5
        pr = torch.softmax(sc, -1)
        out[i] = torch.einsum("ht,thd->hd", pr, vc).reshape(-1)
    return out, new_k


@pytest.mark.parametrize("append", [1, 2])
@pytest.mark.parametrize(
    "heads,d,n_items,max_pos",
    [(16, 128, 37, 700), (16, 128, 256, 300), (4, 64, 16, 120), (16, 128, 3, 3000), (55, 96, 9, 200)],
)
def test_decode_attention_append_matches_fp32(heads, d, n_items, max_pos, append):
    gen = torch.Generator().manual_seed(heads * 1000 + n_items)
    h = AttnHarness(n_items, heads, d, num_blocks=max(512, n_items * (max_pos // BS + 2)))
    max_blocks = max_pos // BS + 2
    table = _make_tables(n_items, max_blocks, h.num_blocks, gen)
    pos = torch.randint(0, max_pos, (n_items,), generator=gen).to(torch.int32)
    pos[0] = 0  # first token of a sequence: nothing cached
    if n_items > 4:
        pos[3] = -1  # padding row
        pos[1] = 15  # page boundary
        pos[2] = 16
    pos = pos.to(DEV)
    slots = torch.arange(n_items, dtype=torch.int32, device=DEV)
    qkv = (torch.randn(n_items, 3 * heads * d, device=DEV)).to(torch.bfloat16)
    cos, sin = _rope_tables(max_pos + 1, d)
    out = torch.zeros(n_items, heads * d, device=DEV, dtype=torch.bfloat16)
    # head_dim 96 is the Huginn shape, whose interleaved RoPE is not the Ouro table: run it unrotated.
    rope_mode = 1 if d != 96 else 0
    ref, new_k = _reference_decode(h, qkv, h.kv.clone(), 1, table, slots, pos, cos, sin, append=1, rope=rope_mode == 1)
    qkv_in = qkv.clone()
    h.run(qkv, out, 1, table, slots, pos, append, rope_mode, cos, sin)
    if append == 2:  # fused: q is rotated in registers, qkv is left as it was
        assert torch.equal(qkv, qkv_in)
    valid = pos >= 0
    err = (out.float()[valid] - ref[valid]).abs().max().item()
    assert err < 2e-2, err
    for i, (k, v, row) in new_k.items():
        assert torch.equal(h.kv[1, 0, row], k.to(torch.bfloat16)), i
        assert torch.equal(h.kv[1, 1, row], v), i
    # padding row untouched
    if n_items > 4:
        assert out[3].abs().sum().item() == 0.0


@pytest.mark.parametrize(
    "heads,d,rope_mode,bias,n_items,max_pos,scratch",
    [
        (16, 128, 1, False, 37, 700, 256),  # split-KV pieces; the last piece appends
        (16, 128, 1, False, 300, 200, 256),  # rows > scratch rows: whole segments, round-robin
        (16, 128, 1, True, 5, 3000, 256),  # long contexts: many pieces per segment
        (4, 64, 1, False, 33, 90, 256),
        (5, 96, 2, True, 21, 400, 256),  # Huginn: qk_bias + interleaved fp32 RoPE
        (55, 96, 2, True, 4, 150, 256),
        (16, 128, 0, True, 12, 100, 256),  # bias without rotation
    ],
)
def test_fused_append_bit_exact_vs_two_kernels(heads, d, rope_mode, bias, n_items, max_pos, scratch):
    """append=2 (one launch) against append=1 (rope_append kernel, then attention): the same
    output bits and the same cache contents, at every position within a page (both token halves
    of the page own the new row somewhere in the batch) and with padding rows."""

    gen = torch.Generator().manual_seed(heads + 17 * n_items + rope_mode)
    max_blocks = max_pos // BS + 2
    h = AttnHarness(n_items, heads, d, num_blocks=max(512, n_items * max_blocks), scratch=scratch)
    table = _make_tables(n_items, max_blocks, h.num_blocks, gen)
    pos = torch.randint(0, max_pos, (n_items,), generator=gen).to(torch.int32)
    for i in range(min(n_items, 16)):
        pos[i] = (pos[i] // BS) * BS + i  # every offset within a page
    if n_items > 4:
        pos[4] = -1
    pos = pos.to(DEV)
    slots = torch.arange(n_items, dtype=torch.int32, device=DEV)
    qkv = torch.randn(n_items, 3 * heads * d, device=DEV).to(torch.bfloat16)
    qk_bias = (0.1 * torch.randn(2, heads, d, device=DEV)).to(torch.bfloat16) if bias else None
    if rope_mode == 2:
        inv = 1.0 / (50000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        freqs = torch.arange(max_pos + BS, device=DEV).float().unsqueeze(-1) * inv.to(DEV)
        cos, sin = freqs.cos().contiguous(), freqs.sin().contiguous()
    else:
        cos, sin = _rope_tables(max_pos + BS, d)  # positions reach max_pos + 14
    kv0 = h.kv.clone()
    out1 = torch.zeros(n_items, heads * d, device=DEV, dtype=torch.bfloat16)
    out2 = torch.zeros_like(out1)
    qkv1 = qkv.clone()
    h.run(qkv1, out1, 1, table, slots, pos, 1, rope_mode, cos, sin, qk_bias=qk_bias)
    kv1 = h.kv.clone()
    h.kv.copy_(kv0)
    qkv2 = qkv.clone()
    h.run(qkv2, out2, 1, table, slots, pos, 2, rope_mode, cos, sin, qk_bias=qk_bias)
    assert torch.equal(qkv2, qkv)
    assert torch.equal(h.kv, kv1)
    assert torch.equal(out2, out1)
    assert int(h.counters.abs().sum().item()) == 0


@pytest.mark.parametrize("heads,d", [(16, 128), (4, 64), (55, 96)])
def test_cache_only_attention_matches_fp32(heads, d):
    n_items = 40
    gen = torch.Generator().manual_seed(7)
    h = AttnHarness(n_items, heads, d)
    table = _make_tables(4, 12, h.num_blocks, gen)
    slots = torch.randint(0, 4, (n_items,), generator=gen).to(torch.int32).to(DEV)
    pos = torch.randint(0, 12 * BS, (n_items,), generator=gen).to(torch.int32).to(DEV)
    qkv = torch.randn(n_items, 3 * heads * d, device=DEV).to(torch.bfloat16)
    cos, sin = _rope_tables(8, d)
    out = torch.zeros(n_items, heads * d, device=DEV, dtype=torch.bfloat16)
    ref, _ = _reference_decode(h, qkv, h.kv, 0, table, slots, pos, cos, sin, append=0)
    h.run(qkv, out, 0, table, slots, pos, 0, 0, cos, sin)
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err


def test_split_scratch_counters_return_to_zero():
    h = AttnHarness(8, 16, 128, num_blocks=2048)
    gen = torch.Generator().manual_seed(3)
    table = _make_tables(8, 200, h.num_blocks, gen)
    pos = torch.full((8,), 3000, dtype=torch.int32, device=DEV)
    slots = torch.arange(8, dtype=torch.int32, device=DEV)
    qkv = torch.randn(8, 3 * 16 * 128, device=DEV).to(torch.bfloat16)
    cos, sin = _rope_tables(3001, 128)
    out = torch.zeros(8, 16 * 128, device=DEV, dtype=torch.bfloat16)
    for _ in range(3):
        h.run(qkv, out, 0, table, slots, pos, 0, 0, cos, sin)
        assert int(h.hdr[0].item()) > 8 * 4  # split-KV was used
        assert int(h.counters.abs().sum().item()) == 0


def _torch_rmsnorm(x, w, eps):
    xf = x.float()
    return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


@pytest.mark.parametrize("hidden", [256, 2048, 5280])
def test_rmsnorm_and_sandwich_add(hidden):
    torch.manual_seed(hidden)
    n = 33
    eps = 1e-6
    x = torch.randn(n, hidden, device=DEV).to(torch.bfloat16)
    a = (3 * torch.randn(n, hidden, device=DEV)).to(torch.bfloat16)
    w1 = (1 + 0.1 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    w2 = (1 + 0.1 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    gw = (0.05 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    gb = torch.tensor([0.25], device=DEV).to(torch.bfloat16)
    y = torch.empty_like(x)
    xc = torch.empty_like(x)
    sp = torch.cuda.current_stream().cuda_stream
    rows = torch.arange(n - 1, -1, -1, dtype=torch.int32, device=DEV)
    _lib.call("cdb_rmsnorm", _lib.ptr(x), hidden, _lib.ptr(rows), _lib.ptr(w1), _lib.ptr(y), hidden, _lib.ptr(xc), hidden, n, hidden, eps, sp)
    torch.cuda.synchronize()
    ref = _torch_rmsnorm(x.flip(0), w1, eps)
    assert torch.equal(xc, x.flip(0))
    assert (y.float() - ref.float()).abs().max().item() <= 2 ** -7 * ref.float().abs().max().item()
    x2 = x.clone()
    g = torch.zeros(n, device=DEV, dtype=torch.bfloat16)
    _lib.call(
        "cdb_add_rmsnorm", _lib.ptr(x2), hidden, _lib.ptr(a), hidden, _lib.ptr(w1), _lib.ptr(w2), _lib.ptr(y), hidden,
        None, _lib.ptr(gw), _lib.ptr(gb), _lib.ptr(g), n, hidden, eps, sp,
    )
    torch.cuda.synchronize()
    xr = x + _torch_rmsnorm(a, w1, eps)
    yr = _torch_rmsnorm(xr, w2, eps)
    gr = torch.nn.functional.linear(yr, gw[None], gb)[:, 0]
    assert (x2.float() - xr.float()).abs().max().item() <= 2 ** -6 * xr.float().abs().max().item()
    assert (y.float() - yr.float()).abs().max().item() <= 2 ** -6 * yr.float().abs().max().item()
    # the gate logit is one bf16 rounding of an fp32 dot product: within 2^-7 of its magnitude
    # (one ulp), plus summation-order noise near zero
    assert ((g.float() - gr.float()).abs() <= 2**-7 * gr.float().abs() + 1e-2).all()


def test_silu_mul_matches_torch():
    n, inter = 19, 5632
    gu = (2 * torch.randn(n, 2 * inter, device=DEV)).to(torch.bfloat16)
    act = torch.empty(n, inter, device=DEV, dtype=torch.bfloat16)
    _lib.call("cdb_silu_mul", _lib.ptr(gu), gu.stride(0), _lib.ptr(act), act.stride(0), n, inter, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    diff = (act.float() - ref.float()).abs()
    assert diff.max().item() <= 2 ** -7 * ref.float().abs().max().item()


@pytest.mark.parametrize("vocab", [1024, 49152, 1000])
def test_argmax_first_index_and_scatter(vocab):
    n = 23
    logits = torch.randn(n, vocab, device=DEV).to(torch.bfloat16)
    logits[0, 5] = 9.0
    logits[0, 700] = 9.0  # tie: first index wins
    logits[1] = 0.0
    out = torch.full((64,), -7, dtype=torch.int64, device=DEV)
    out_rows = torch.arange(n, dtype=torch.int32, device=DEV) * 2
    tok_rows = torch.arange(n, dtype=torch.int32, device=DEV)
    table = torch.zeros(n, dtype=torch.int32, device=DEV)
    _lib.call(
        "cdb_argmax", _lib.ptr(logits), logits.stride(0), n, vocab, _lib.ptr(out), _lib.ptr(out_rows), _lib.ptr(tok_rows),
        _lib.ptr(table), torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    ref = torch.argmax(logits.float(), dim=-1)
    assert torch.equal(out[::2][:n], ref)
    assert torch.equal(table.long(), ref)
    assert int(out[0]) == 5 and int(out[2]) == 0


def test_embed_gathers_host_and_device_ids():
    vocab, hidden, n = 1000, 256, 10
    table = torch.randn(vocab, hidden, device=DEV).to(torch.bfloat16)
    ids = torch.tensor([3, -1, 999, -1, 0, 5, -1, 7, 8, 9], dtype=torch.int32, device=DEV)
    src = torch.arange(n, dtype=torch.int32, device=DEV)
    tok = torch.tensor([0, 42, 0, 17, 0, 0, 500, 0, 0, 0], dtype=torch.int32, device=DEV)
    out = torch.zeros(2 * n, hidden, device=DEV, dtype=torch.bfloat16)
    rows = torch.arange(n, dtype=torch.int32, device=DEV) * 2
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.call(
        "cdb_embed", _lib.ptr(table), hidden, vocab, _lib.ptr(ids), _lib.ptr(src), _lib.ptr(tok), _lib.ptr(out), hidden,
        _lib.ptr(rows), n, 1.0, _lib.ptr(status), torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    want = torch.where(ids >= 0, ids, tok).long()
    assert torch.equal(out[::2], table[want])
    assert int(status.item()) == 0
    # Huginn's scaled embedding: bf16(table[id] * sqrt(n_embd)), one rounding (torch's bf16 * float)
    scale = math.sqrt(5280)
    _lib.call(
        "cdb_embed", _lib.ptr(table), hidden, vocab, _lib.ptr(ids), _lib.ptr(src), _lib.ptr(tok), _lib.ptr(out), hidden,
        _lib.ptr(rows), n, scale, _lib.ptr(status), torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    assert torch.equal(out[::2], table[want] * scale)


def test_block_table_edits_and_exit_copy():
    table = torch.full((4, 8), -1, dtype=torch.int32, device=DEV)
    edits = torch.tensor([0, 0, 5, 0, 1, 9, 3, 7, 2], dtype=torch.int32, device=DEV)
    _lib.call("cdb_block_table_update", _lib.ptr(table), 8, _lib.ptr(edits), 3, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert table[0, :2].tolist() == [5, 9] and int(table[3, 7]) == 2
    kv = torch.randn(4, 2, 64, 4, 64, device=DEV).to(torch.bfloat16)
    before = kv.clone()
    rows = torch.tensor([3, 17, 40], dtype=torch.int32, device=DEV)
    src = torch.tensor([0, 0], dtype=torch.int32, device=DEV)
    dst = torch.tensor([2, 3], dtype=torch.int32, device=DEV)
    _lib.call(
        "cdb_exit_kv_copy", _lib.ptr(kv), 4, 64, 4, 64, _lib.ptr(rows), 3, _lib.ptr(src), _lib.ptr(dst), 2,
        torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    for layer in (2, 3):
        assert torch.equal(kv[layer][:, rows.long()], before[0][:, rows.long()])
    untouched = [r for r in range(64) if r not in (3, 17, 40)]
    assert torch.equal(kv[2][:, untouched], before[2][:, untouched])


def test_kv_blocks_host_copy_round_trip():
    """Offload swap (``cdb_kv_blocks_host_copy``): whole blocks (every cache layer, K and V) go out
    to a pinned host pool and come back into other blocks bit for bit; block ids out of range are
    refused before anything is queued."""

    from continuous_depth_batching_b200.kv_cache import PagedKVPool

    pool = PagedKVPool(
        num_cache_layers=3, num_blocks=12, block_size=16, num_kv_heads=4, head_dim=64, max_model_len=256,
        resident_slots=4, device=torch.device(DEV),
    )
    pool.kv.copy_(torch.randn(pool.kv.shape, device=DEV).to(torch.bfloat16))
    before = pool.kv.clone()
    pool.attach_host_pool(8)
    assert pool.host_pool.is_pinned() and pool.block_bytes == 2 * 3 * 16 * 4 * 64 * 2
    stream = torch.cuda.current_stream()
    pool.host_copy([5, 2, 9], [3, 0, 7], True, stream)
    torch.cuda.synchronize()
    host = pool.host_pool.view(torch.bfloat16).view(8, 3, 2, 16, 4, 64)

    def blk(t, b):
        return t[:, :, b * 16 : (b + 1) * 16]

    for d, h in ((5, 3), (2, 0), (9, 7)):
        assert torch.equal(host[h], blk(before, d).cpu())
    pool.kv.zero_()
    pool.host_copy([1, 11, 4], [3, 0, 7], False, stream)
    torch.cuda.synchronize()
    for d, src in ((1, 5), (11, 2), (4, 9)):
        assert torch.equal(blk(pool.kv, d), blk(before, src))
    others = [b for b in range(14) if b not in (1, 11, 4)]
    assert all(int(blk(pool.kv, b).abs().sum()) == 0 for b in others)
    snapshot = pool.kv.clone()
    with pytest.raises(_lib.CDBError):
        pool.host_copy([3, 12], [0, 1], True, stream)
    with pytest.raises(_lib.CDBError):
        pool.host_copy([3], [8], False, stream)
    torch.cuda.synchronize()
    assert torch.equal(pool.kv, snapshot)


def test_exit_hazard_matches_host_policy():
    n = 6
    logits = torch.tensor([0.3, -2.0, 4.0, 0.0, -0.1, 1.5], device=DEV).to(torch.bfloat16)
    slots = torch.arange(n, dtype=torch.int32, device=DEV)
    steps = torch.tensor([0, 0, 1, 2, 0, 0], dtype=torch.int32, device=DEV)
    reset = torch.ones(n, dtype=torch.int8, device=DEV)
    cdf = torch.zeros(n, dtype=torch.float64, device=DEV)
    surv = torch.ones(n, dtype=torch.float64, device=DEV)
    flags = torch.zeros(n, dtype=torch.int8, device=DEV)
    _lib.call(
        "cdb_exit_hazard", _lib.ptr(logits), 1, _lib.ptr(slots), _lib.ptr(steps), _lib.ptr(reset), _lib.ptr(cdf),
        _lib.ptr(surv), _lib.ptr(flags), n, 2, 0.5, torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    for i in range(n):
        hz = float(torch.sigmoid(logits[i].cpu()).float().item())
        assert math.isclose(float(cdf[i]), hz, rel_tol=0, abs_tol=1e-12)
        want = (int(steps[i]) + 1 >= 2) and hz >= 0.5
        assert bool(flags[i]) == want


@pytest.mark.parametrize("heads,d", [(16, 128), (4, 64), (5, 96)])
def test_prefill_attention_tiles_match_fp32(heads, d):
    """Tiled causal prefill attention == per-row fp32 attention over [0, position]."""

    from continuous_depth_batching_b200.runner import OuroRunner

    gen = torch.Generator().manual_seed(21)
    h = AttnHarness(8, heads, d, num_blocks=600)
    table = _make_tables(5, 40, h.num_blocks, gen)
    # chunks: (slot, past, rows) - cached prefixes, ragged lengths, a 1-row chunk, > 64-row chunks
    chunks = [(0, 0, 150), (1, 37, 5), (2, 100, 64), (3, 0, 1), (4, 250, 129)]
    slots, pos = [], []
    for s, past, rows in chunks:
        slots += [s] * rows
        pos += list(range(past, past + rows))
    n = len(pos)
    tiles = OuroRunner.prefill_tiles(slots, pos)
    assert all(t[1] <= 64 for t in tiles) and sum(t[1] for t in tiles) == n
    tiles_d = torch.tensor(tiles, dtype=torch.int32, device=DEV).reshape(-1)
    qkv = torch.randn(n, 3 * heads * d, device=DEV).to(torch.bfloat16)
    out = torch.zeros(n, heads * d, device=DEV, dtype=torch.bfloat16)
    slots_d = torch.tensor(slots, dtype=torch.int32, device=DEV)
    pos_d = torch.tensor(pos, dtype=torch.int32, device=DEV)
    cos, sin = _rope_tables(8, d)
    ref, _ = _reference_decode(h, qkv, h.kv, 1, table, slots_d, pos_d, cos, sin, append=0)
    hd = heads * d
    _lib.call(
        "cdb_prefill_attention", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, _lib.ptr(out), out.stride(0), _lib.ptr(h.kv),
        h.layers, h.rows, 1, _lib.ptr(table), table.stride(0), _lib.ptr(tiles_d), len(tiles), heads, d, BS, d**-0.5,
        _lib.ptr(h.status), torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    assert int(h.status.item()) == 0
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("hidden", [2048, 1000])
def test_gather_rows_exact(hidden):
    src = torch.randn(20, hidden + 8, device=DEV).to(torch.bfloat16)[:, :hidden]
    rows = torch.tensor([3, -1, 19, 0, 3], dtype=torch.int32, device=DEV)
    dst = torch.full((5, hidden), 7.0, device=DEV, dtype=torch.bfloat16)
    _lib.call(
        "cdb_gather_rows", _lib.ptr(src), src.stride(0), _lib.ptr(rows), 5, hidden, _lib.ptr(dst), dst.stride(0),
        torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    for i, r in enumerate(rows.tolist()):
        if r < 0:
            assert dst[i].abs().sum().item() == 0
        else:
            assert torch.equal(dst[i], src[r])


# ----------------------------------------------------------------------------- Huginn kernels
def _huginn_rotate(x, cos, sin):
    """apply_rotary_emb_complex_like (modeling_huginn.py:175-197) on [T, H, D] bf16."""

    x2 = x.unflatten(-1, (-1, 2)).float()
    c, s_ = cos[:, None, :], sin[:, None, :]
    return torch.stack([x2[..., 0] * c - x2[..., 1] * s_, x2[..., 1] * c + x2[..., 0] * s_], dim=-1).flatten(2).type_as(x)


def test_huginn_rope_bias_append_exact():
    """rope_mode 2 + qk_bias: q rotated in place and k/v appended equal the reference's op sequence
    bit for bit (bf16 bias add, fp32 products and sums each rounded, one cast back)."""

    heads, d, n = 5, 96, 7
    gen = torch.Generator().manual_seed(5)
    h = AttnHarness(n, heads, d, num_blocks=64)
    table = _make_tables(n, 4, h.num_blocks, gen)
    pos = torch.tensor([0, 3, 15, 16, 40, 17, 2], dtype=torch.int32, device=DEV)
    slots = torch.arange(n, dtype=torch.int32, device=DEV)
    qkv = torch.randn(n, 3 * heads * d, device=DEV).to(torch.bfloat16)
    bias = (0.1 * torch.randn(2, heads, d, device=DEV)).to(torch.bfloat16)
    inv = 1.0 / (50000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    freqs = torch.arange(64, device=DEV).float().unsqueeze(-1) * inv.to(DEV)
    cos, sin = freqs.cos().contiguous(), freqs.sin().contiguous()
    hd = heads * d
    q0 = qkv[:, :hd].reshape(n, heads, d).clone()
    k0 = qkv[:, hd : 2 * hd].reshape(n, heads, d).clone()
    v0 = qkv[:, 2 * hd :].reshape(n, heads, d).clone()
    p = pos.long()
    q_ref = _huginn_rotate((q0 + bias[0]).to(torch.bfloat16), cos[p], sin[p])
    k_ref = _huginn_rotate((k0 + bias[1]).to(torch.bfloat16), cos[p], sin[p])
    out = torch.zeros(n, hd, device=DEV, dtype=torch.bfloat16)
    h.run(qkv, out, 1, table, slots, pos, 1, 2, cos, sin, qk_bias=bias)
    assert torch.equal(qkv[:, :hd].reshape(n, heads, d), q_ref)
    for i in range(n):
        pi = int(pos[i])
        row = int(table[i, pi // BS]) * BS + pi % BS
        assert torch.equal(h.kv[1, 0, row], k_ref[i]), i
        assert torch.equal(h.kv[1, 1, row], v0[i]), i
    # the attention output over the cache (now holding the appended rows) against fp32
    ref, _ = _reference_decode(h, qkv, h.kv, 1, table, slots, pos, cos, sin, append=0)
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("hidden", [480, 5280])
def test_sandwich_norm_matches_torch(hidden):
    n, eps = 9, 1e-6
    x = (4 * torch.randn(12, hidden, device=DEV)).to(torch.bfloat16)
    a = torch.randn(n, hidden, device=DEV).to(torch.bfloat16)
    w1 = (1 + 0.1 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    w2 = (1 + 0.1 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    rows = torch.tensor([3, 0, -1, 11, 5, 6, 7, 8, 2], dtype=torch.int32, device=DEV)
    drows = torch.tensor([1, -1, 0, 2, 3, 4, 5, 6, 7], dtype=torch.int32, device=DEV)
    xd = torch.zeros(8, hidden, device=DEV, dtype=torch.bfloat16)
    y = torch.zeros(n, hidden, device=DEV, dtype=torch.bfloat16)
    _lib.call(
        "cdb_sandwich_norm", _lib.ptr(x), x.stride(0), _lib.ptr(rows), _lib.ptr(a), a.stride(0), _lib.ptr(w1),
        _lib.ptr(xd), xd.stride(0), _lib.ptr(drows), _lib.ptr(w2), _lib.ptr(y), y.stride(0), n, hidden, eps,
        torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    for r in range(n):
        src, dst = int(rows[r]), int(drows[r])
        if src < 0:
            continue
        v = _torch_rmsnorm(a[r] + x[src], w1, eps)  # norm_2(attn + x)
        yr = _torch_rmsnorm(v, w2, eps)  # norm_3(x)
        if dst >= 0:
            assert (xd[dst].float() - v.float()).abs().max().item() <= 2**-7 * v.float().abs().max().item()
        assert (y[r].float() - yr.float()).abs().max().item() <= 2**-7 * yr.float().abs().max().item()
    # no add, no first norm: a pure gather + norm (coda entry is ln_f of the gathered state)
    y2 = torch.zeros_like(y)
    _lib.call(
        "cdb_sandwich_norm", _lib.ptr(x), x.stride(0), _lib.ptr(rows), None, 0, None, None, 0, None, _lib.ptr(w2),
        _lib.ptr(y2), y2.stride(0), n, hidden, eps, torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    r = 0
    ref = _torch_rmsnorm(x[int(rows[r])], w2, eps)
    assert (y2[r].float() - ref.float()).abs().max().item() <= 2**-7 * ref.float().abs().max().item()


def test_latent_diff_matches_torch():
    n, hidden = 11, 5280
    new = torch.randn(n, hidden, device=DEV).to(torch.bfloat16)
    old = (new.float() + 0.3 * torch.randn(n, hidden, device=DEV)).to(torch.bfloat16)
    old[3] = new[3]  # converged row: exactly zero
    rows = torch.arange(n, dtype=torch.int32, device=DEV)
    rows[5] = -1
    out = torch.full((n,), 7.0, device=DEV, dtype=torch.bfloat16)
    _lib.call(
        "cdb_latent_diff", _lib.ptr(new), new.stride(0), _lib.ptr(old), old.stride(0), _lib.ptr(rows), n, hidden,
        _lib.ptr(out), torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    ref = ((new - old).norm(dim=-1) / new.norm(dim=-1).clamp_min(1e-9)).to(torch.bfloat16)
    keep = rows >= 0
    assert ((out.float() - ref.float()).abs()[keep] <= 2**-7 * ref.float().abs()[keep]).all()
    assert float(out[3]) == 0.0 and float(out[5]) == 7.0
