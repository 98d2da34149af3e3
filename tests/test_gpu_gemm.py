"""tcgen05/TMEM GEMM (cdb_gemm_bf16) against a plain PyTorch fp32 reference on the GPU.

c = x @ w^T with bf16 x, w; the reference multiplies the same bf16 values in fp32. The GEMM
accumulates in fp32 and rounds once, so every element is within one bf16 rounding of the
reference plus fp32 summation-order noise: |c - ref| <= 2^-8 |ref| + 2^-12 * ||x_row|| ||w_row||.
Shapes cover the Ouro-1.4B projections (N 6144/2048/11264/2048, K 2048/5632, LM head 49152),
token counts from 1 to prefill sizes, M/N/K tails (odd output widths take the scalar store
path), persistent CTA counts from one CTA (every tile in one range) to one per SM (tiles split
over CTAs and combined through the workspace), and repeated calls (the combine sums pieces in k
order, so results are bit-identical and the tile counters come back zeroed). Problems with fewer
tiles than SMs take the split mode (K split over a thread-block cluster, reduced through
distributed shared memory) unless a CTA count is forced; problems above 256 token rows with at
least two 256 x 256 tiles per SM pair take the CTA-pair mode (cta_group::2 MMAs) unless a CTA
count is forced.
"""

from __future__ import annotations

import pytest
import torch

from continuous_depth_batching_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


class Gemm:
    def __init__(self):
        self.work = _lib.GemmWorkspace(torch.device(DEV), 2048, 65536, 148)
        self.status = torch.zeros(1, dtype=torch.int32, device=DEV)

    def __call__(self, x, w, ctas=0, out=None):
        m, k = x.shape
        n = w.shape[0]
        c = torch.empty(m, n, dtype=torch.bfloat16, device=DEV) if out is None else out
        _lib.call(
            "cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(c), c.stride(0), m, n, k,
            ctas, *self.work.args(), 148, _lib.ptr(self.status), torch.cuda.current_stream().cuda_stream,
        )
        return c


@pytest.fixture(scope="module")
def gemm():
    return Gemm()


def _check(c, x, w):
    ref = x.float() @ w.float().t()
    bound = 2**-8 * ref.abs() + 2**-12 * (x.float().norm(dim=1)[:, None] * w.float().norm(dim=1)[None, :])
    bad = (c.float() - ref).abs() > bound
    assert not bad.any(), f"{int(bad.sum())} elements out of bound; max err {(c.float() - ref).abs().max().item():.3e}"


@pytest.mark.parametrize(
    "m,n,k",
    [
        (1, 6144, 2048), (7, 2048, 2048), (33, 11264, 2048), (64, 2048, 5632), (100, 6144, 2048),
        (256, 6144, 2048), (256, 2048, 2048), (256, 11264, 2048), (256, 2048, 5632), (96, 49152, 2048),
        (300, 768, 256), (1024, 1408, 256), (2048, 6144, 2048), (16, 256, 704), (130, 1000, 520),
        (5, 1001, 512), (40, 130, 4096), (24, 2048, 5632), (700, 1000, 520), (513, 11264, 2048),
        (4096, 2048, 5632),
    ],
)
def test_gemm_matches_fp32_reference(gemm, m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    c = gemm(x, w)
    torch.cuda.synchronize()
    assert int(gemm.status.item()) == 0
    _check(c, x, w)


@pytest.mark.parametrize("m", [200, 24, 60, 600])
@pytest.mark.parametrize("ctas", [1, 7, 74, 148])
def test_gemm_cta_counts_and_repeat(gemm, ctas, m):
    g = torch.Generator(device=DEV).manual_seed(ctas)
    x = torch.randn(m, 2048, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(2048, 2048, device=DEV, generator=g)).to(torch.bfloat16)
    first = gemm(x, w, ctas=ctas)
    for _ in range(3):
        again = gemm(x, w, ctas=ctas)
        torch.cuda.synchronize()
        assert torch.equal(first, again)  # deterministic across calls
    assert int(gemm.status.item()) == 0
    assert int(gemm.work.ctr.abs().sum().item()) == 0  # counters left zeroed
    _check(first, x, w)


@pytest.mark.parametrize("m,n,k", [(2048, 6144, 2048), (8192, 2048, 5632), (4000, 5000, 520), (2304, 4352, 1024)])
def test_pair_tiles_repeat_and_counters(gemm, m, n, k):
    """Above 256 token rows, with at least two 256 x 256 pair tiles per SM pair, the library's
    choice is the CTA-pair mode (tcgen05.mma.cta_group::2, stream-K over pairs with the split tiles
    combined per half; ragged M and N included): within the fp32 bound, bit-identical across
    calls, tile counters left zeroed."""

    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    first = gemm(x, w)
    for _ in range(2):
        again = gemm(x, w)
        torch.cuda.synchronize()
        assert torch.equal(first, again)
    assert int(gemm.status.item()) == 0
    assert int(gemm.work.ctr.abs().sum().item()) == 0
    _check(first, x, w)


def test_gemm_strided_operands_and_output(gemm):
    g = torch.Generator(device=DEV).manual_seed(3)
    big = torch.randn(64, 3000, device=DEV, generator=g).to(torch.bfloat16)
    x = big[:, 8:2056]  # ld 3000, 16-byte aligned start
    w = (0.05 * torch.randn(512, 2048, device=DEV, generator=g)).to(torch.bfloat16)
    out = torch.zeros(64, 700, dtype=torch.bfloat16, device=DEV)
    gemm(x, w, out=out[:, :512])
    torch.cuda.synchronize()
    _check(out[:, :512], x, w)
    assert out[:, 512:].abs().sum().item() == 0


@pytest.mark.parametrize(
    "m,inter,k",
    [(1, 5632, 2048), (80, 5632, 2048), (256, 5632, 2048), (700, 704, 256), (33, 504, 520), (8192, 5632, 2048),
     (3000, 2000, 520)],
)
def test_gateup_silu_gemm(gemm, m, inter, k):
    """cdb_mlp_gateup_silu_gemm == plain GEMM on the same interleaved weight + cdb_silu_mul
    (bit-exact: same tiles and stream-K pieces), and within one bf16 rounding of gate/up of the fp32
    reference act_fn(x Wg^T) * (x Wu^T) with the reference's bf16 rounding points."""

    g = torch.Generator(device=DEV).manual_seed(m + inter + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    wg = (0.05 * torch.randn(inter, k, device=DEV, generator=g)).to(torch.bfloat16)
    wu = (0.05 * torch.randn(inter, k, device=DEV, generator=g)).to(torch.bfloat16)
    w_il = torch.stack([wg, wu], dim=1).reshape(2 * inter, k).contiguous()
    act = torch.zeros(m, inter, dtype=torch.bfloat16, device=DEV)
    sp = torch.cuda.current_stream().cuda_stream
    _lib.call(
        "cdb_mlp_gateup_silu_gemm", _lib.ptr(x), x.stride(0), _lib.ptr(w_il), w_il.stride(0), _lib.ptr(act),
        act.stride(0), m, inter, k, 0, *gemm.work.args(), 148, _lib.ptr(gemm.status), sp,
    )
    gu_il = gemm(x, w_il)
    gu = torch.cat([gu_il[:, 0::2], gu_il[:, 1::2]], dim=1).contiguous()
    act2 = torch.zeros_like(act)
    _lib.call("cdb_silu_mul", _lib.ptr(gu), gu.stride(0), _lib.ptr(act2), act2.stride(0), m, inter, sp)
    torch.cuda.synchronize()
    assert int(gemm.status.item()) == 0
    assert torch.equal(act, act2)
    gf = x.float() @ wg.float().t()
    uf = x.float() @ wu.float().t()
    gb, ub = gf.to(torch.bfloat16), uf.to(torch.bfloat16)
    ref = (torch.nn.functional.silu(gb.float()).to(torch.bfloat16).float() * ub.float()).to(torch.bfloat16).float()
    # gate and up each carry the plain GEMM's error bound (one bf16 rounding plus fp32
    # summation-order noise, as in _check): E = 2^-7 |v| + 2^-12 ||x_row|| ||w_row||. Through
    # silu(g)*u (|silu'| <= 1.1, |silu(g)| <= |g|) that moves act by at most
    # 1.1 E_g (|u| + E_u) + (|g| + E_g) E_u, plus the product's own rounding 2^-7 |ref|.
    # A mis-paired gate/up row is off by O(|ref|).
    xn = x.float().norm(dim=1)[:, None]
    e_g = 2**-7 * gf.abs() + 2**-12 * xn * wg.float().norm(dim=1)[None, :]
    e_u = 2**-7 * uf.abs() + 2**-12 * xn * wu.float().norm(dim=1)[None, :]
    bound = 1.1 * e_g * (uf.abs() + e_u) + (gf.abs() + e_g) * e_u + 2**-7 * ref.abs() + 1e-6
    bad = (act.float() - ref).abs() > bound
    assert not bad.any(), f"{int(bad.sum())} out of bound; max err {(act.float() - ref).abs().max().item():.3e}"


@pytest.mark.parametrize("m,vocab,k", [(1, 49152, 2048), (7, 1000, 512), (80, 49152, 2048), (130, 65536, 480), (300, 4096, 256),
                                          (600, 49152, 2048)])
def test_lm_head_argmax_matches_logits_argmax(gemm, m, vocab, k):
    """cdb_lm_head_argmax == torch.argmax (first maximum) of the plain GEMM's bf16 logits, exactly
    (same tiles, same stream-K pieces, same accumulation), with the output-row and token-table
    scatters, twice in a row (the key/counter scratch must come back zeroed)."""

    g = torch.Generator(device=DEV).manual_seed(m + vocab)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(vocab, k, device=DEV, generator=g)).to(torch.bfloat16)
    keys = torch.zeros(m, dtype=torch.int64, device=DEV)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full((2 * m + 1,), -7, dtype=torch.int64, device=DEV)
    out_rows = (torch.arange(m, dtype=torch.int32, device=DEV) * 2 + 1)
    out_rows[0] = -1  # skipped row
    table = torch.full((m + 3,), -5, dtype=torch.int32, device=DEV)
    token_rows = torch.arange(m, dtype=torch.int32, device=DEV) + 3
    sp = torch.cuda.current_stream().cuda_stream
    logits = gemm(x, w, ctas=148)  # the LM head's own stream-K decomposition (one CTA per SM)
    ref = logits.float().argmax(dim=-1)
    for _ in range(2):
        _lib.call(
            "cdb_lm_head_argmax", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), m, vocab, k, _lib.ptr(out),
            _lib.ptr(out_rows), _lib.ptr(token_rows), _lib.ptr(table), _lib.ptr(keys), _lib.ptr(done),
            *gemm.work.args(), 148, _lib.ptr(gemm.status), sp,
        )
        torch.cuda.synchronize()
        assert int(gemm.status.item()) == 0
        assert torch.equal(out[out_rows[1:].long()], ref[1:])
        assert int(out[1]) == -7  # row 0 was skipped
        assert torch.equal(table[3:].long(), ref)
        assert int(keys.abs().sum()) == 0 and int(done.item()) == 0
        assert int(gemm.work.ctr.abs().sum().item()) == 0


def _sp():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("m,hidden,k,last", [(80, 2048, 2048, False), (37, 2048, 5632, True), (256, 512, 1408, True)])
def test_residual_norm_gemms_match_separate_calls(gemm, m, hidden, k, last):
    """cdb_o_proj_residual_norm_gemm / cdb_down_residual_norm_gemm equal cdb_gemm_bf16 followed by
    cdb_add_rmsnorm bit for bit (projection, residual stream, normed output, gate logit)."""

    torch.manual_seed(m + hidden)
    a = torch.randn(m, k, device=DEV).to(torch.bfloat16)
    w = (torch.randn(hidden, k, device=DEV) * k**-0.5).to(torch.bfloat16)
    x0 = torch.randn(m, hidden, device=DEV).to(torch.bfloat16)
    wa = (1 + 0.1 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    wn = (1 + 0.1 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    gw = (0.05 * torch.randn(hidden, device=DEV)).to(torch.bfloat16)
    gb = torch.tensor([0.25], device=DEV).to(torch.bfloat16)
    rows = torch.randperm(2 * m, device=DEV)[:m].to(torch.int32) if last else None
    if last:
        rows[m // 3] = -1
    out_rows = 2 * m if last else m
    results = []
    for fused in (False, True):
        x = x0.clone()
        proj = torch.zeros(m, hidden, dtype=torch.bfloat16, device=DEV)
        y = torch.zeros(out_rows, hidden, dtype=torch.bfloat16, device=DEV)
        gout = torch.zeros(m, dtype=torch.bfloat16, device=DEV)
        g = (_lib.ptr(gw), _lib.ptr(gb), _lib.ptr(gout)) if last else (None, None, None)
        if fused and last:
            _lib.call(
                "cdb_down_residual_norm_gemm", _lib.ptr(a), a.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(proj),
                proj.stride(0), _lib.ptr(x), x.stride(0), _lib.ptr(wa), _lib.ptr(wn), _lib.ptr(y), y.stride(0),
                _lib.ptr(rows), *g, m, hidden, k, 1e-6, *gemm.work.args(), 148, _lib.ptr(gemm.status), _sp(),
            )
        elif fused:
            _lib.call(
                "cdb_o_proj_residual_norm_gemm", _lib.ptr(a), a.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(proj),
                proj.stride(0), _lib.ptr(x), x.stride(0), _lib.ptr(wa), _lib.ptr(wn), _lib.ptr(y), y.stride(0), m,
                hidden, k, 1e-6, *gemm.work.args(), 148, _lib.ptr(gemm.status), _sp(),
            )
        else:
            gemm(a, w, out=proj)
            _lib.call(
                "cdb_add_rmsnorm", _lib.ptr(x), x.stride(0), _lib.ptr(proj), proj.stride(0), _lib.ptr(wa), _lib.ptr(wn),
                _lib.ptr(y), y.stride(0), _lib.ptr(rows), *g, m, hidden, 1e-6, _sp(),
            )
        torch.cuda.synchronize()
        assert int(gemm.status.item()) == 0
        results.append((proj, x, y, gout))
    for ref, got in zip(results[0], results[1], strict=True):
        assert torch.equal(ref, got)
    assert results[1][1].abs().sum().item() > 0


@pytest.mark.parametrize("heads,d,rope_mode,bias", [(16, 128, 1, False), (5, 96, 2, True)])
def test_qkv_rope_append_gemm_matches_separate_calls(gemm, heads, d, rope_mode, bias):
    """cdb_qkv_rope_append_gemm equals cdb_gemm_bf16 followed by cdb_rope_append_kv bit for bit
    (rotated q in the qkv buffer, rotated k and v in the cache rows)."""

    torch.manual_seed(heads)
    n, k, bs, nb = 21, 512, 16, 64
    hd = heads * d
    x = torch.randn(n, k, device=DEV).to(torch.bfloat16)
    w = (torch.randn(3 * hd, k, device=DEV) * k**-0.5).to(torch.bfloat16)
    kv0 = torch.randn(2, 2, (nb + 2) * bs, heads, d, device=DEV).to(torch.bfloat16)
    table = torch.randperm(nb, device=DEV)[: n * 3].view(n, 3).to(torch.int32)
    slots = torch.arange(n, dtype=torch.int32, device=DEV)
    pos = torch.randint(0, 3 * bs, (n,), device=DEV).to(torch.int32)
    pos[2] = -1  # padding row: nothing written
    qk_bias = (0.1 * torch.randn(2, heads, d, device=DEV)).to(torch.bfloat16) if bias else None
    if rope_mode == 2:
        inv = 1.0 / (50000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        f = torch.arange(3 * bs, device=DEV).float().unsqueeze(-1) * inv.to(DEV)
        cos, sin = f.cos().contiguous(), f.sin().contiguous()
    else:
        inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        f = torch.arange(3 * bs, device=DEV).float().unsqueeze(-1) * inv.to(DEV)
        emb = torch.cat((f, f), dim=-1)
        cos, sin = emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()
    outs = []
    for fused in (False, True):
        qkv = torch.zeros(n, 3 * hd, dtype=torch.bfloat16, device=DEV)
        kv = kv0.clone()
        common = (
            _lib.ptr(kv), 2, (nb + 2) * bs, 1, _lib.ptr(table), table.stride(0), _lib.ptr(slots), _lib.ptr(pos),
            rope_mode, _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(qk_bias),
        )
        if fused:
            _lib.call(
                "cdb_qkv_rope_append_gemm", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(qkv),
                qkv.stride(0), hd, 2 * hd, n, k, *common, heads, d, bs, *gemm.work.args(), 148,
                _lib.ptr(gemm.status), _sp(),
            )
        else:
            gemm(x, w, out=qkv)
            _lib.call("cdb_rope_append_kv", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, *common, n, heads, d, bs, _sp())
        torch.cuda.synchronize()
        assert int(gemm.status.item()) == 0
        outs.append((qkv, kv))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    assert not torch.equal(outs[1][1], kv0)


@pytest.mark.parametrize("m,n,k", [(1, 2048, 2048), (37, 2048, 5632), (80, 2048, 2048), (80, 2048, 5632),
                                   (200, 2048, 2048), (256, 512, 1408), (16, 1000, 520)])
def test_unreduced_split_planes_and_norm(gemm, m, n, k):
    """cdb_gemm_bf16_partials leaves one fp32 plane per K split: the planes sum (in split order) to
    the fp32 reference within the GEMM bound, and cdb_add_rmsnorm_parts on them equals
    cdb_add_rmsnorm on a = bf16(that sum) bit for bit (residual stream, normed output, gate)."""

    torch.manual_seed(m * 3 + n + k)
    a = torch.randn(m, k, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV) * k**-0.5).to(torch.bfloat16)
    splits = _lib.load().cdb_gemm_partial_splits(m, n, k, 148)
    kb = -(-k // 64)
    assert 1 <= splits <= 16 and splits <= kb
    stride = m * n + 4  # planes need not be packed
    stride += (-stride) % 4
    parts = torch.full((splits * stride,), float("nan"), dtype=torch.float32, device=DEV)
    for _ in range(2):  # the second call rewrites every plane element with the same values
        _lib.call(
            "cdb_gemm_bf16_partials", _lib.ptr(a), a.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(parts), stride,
            m, n, k, splits, _lib.ptr(gemm.status), _sp(),
        )
        torch.cuda.synchronize()
    assert int(gemm.status.item()) == 0
    planes = [parts[z * stride: z * stride + m * n].view(m, n) for z in range(splits)]
    total = planes[0].clone()
    for z in range(1, splits):
        total += planes[z]
    assert not torch.isnan(total).any()
    # each plane is the product over its own k blocks
    per = -(-kb // splits) * 64
    for z in (0, splits - 1):
        ref_z = a[:, z * per: (z + 1) * per].float() @ w[:, z * per: (z + 1) * per].float().t()
        assert (planes[z] - ref_z).abs().max().item() <= 1e-3 * (1 + ref_z.abs().max().item())
    _check(total.to(torch.bfloat16), a, w)
    if n % 8:
        return
    x0 = torch.randn(m, n, device=DEV).to(torch.bfloat16)
    wa = (1 + 0.1 * torch.randn(n, device=DEV)).to(torch.bfloat16)
    wn = (1 + 0.1 * torch.randn(n, device=DEV)).to(torch.bfloat16)
    gw = (0.05 * torch.randn(n, device=DEV)).to(torch.bfloat16)
    gb = torch.tensor([0.25], device=DEV).to(torch.bfloat16)
    results = []
    for from_parts in (False, True):
        x = x0.clone()
        y = torch.zeros(m, n, dtype=torch.bfloat16, device=DEV)
        gout = torch.zeros(m, dtype=torch.bfloat16, device=DEV)
        if from_parts:
            _lib.call(
                "cdb_add_rmsnorm_parts", _lib.ptr(x), x.stride(0), _lib.ptr(parts), splits, stride, _lib.ptr(wa),
                _lib.ptr(wn), _lib.ptr(y), y.stride(0), None, _lib.ptr(gw), _lib.ptr(gb), _lib.ptr(gout), m, n,
                1e-6, _sp(),
            )
        else:
            proj = total.to(torch.bfloat16)
            _lib.call(
                "cdb_add_rmsnorm", _lib.ptr(x), x.stride(0), _lib.ptr(proj), proj.stride(0), _lib.ptr(wa),
                _lib.ptr(wn), _lib.ptr(y), y.stride(0), None, _lib.ptr(gw), _lib.ptr(gb), _lib.ptr(gout), m, n,
                1e-6, _sp(),
            )
        torch.cuda.synchronize()
        results.append((x, y, gout))
    for ref, got in zip(results[0], results[1], strict=True):
        assert torch.equal(ref, got)
