"""torch.ops.cdb on the GPU: each op gives exactly what its C-ABI entry point gives, and the ops
can be captured in a CUDA graph and replayed."""

from __future__ import annotations

import pytest
import torch

import continuous_depth_batching_b200.ops as ops
from continuous_depth_batching_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _sp():
    return torch.cuda.current_stream().cuda_stream


def test_gemm_op_matches_abi_and_replays_in_graph():
    torch.manual_seed(0)
    x = torch.randn(80, 2048, device=DEV).to(torch.bfloat16)
    w = (torch.randn(2048, 2048, device=DEV) * 0.02).to(torch.bfloat16)
    ref = torch.empty(80, 2048, dtype=torch.bfloat16, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    work = _lib.GemmWorkspace(torch.device(DEV), 80, 2048, 148)
    _lib.call("cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(ref), ref.stride(0), 80,
              2048, 2048, 0, *work.args(), 148, _lib.ptr(st), _sp())
    out = torch.empty_like(ref)
    torch.ops.cdb.gemm_bf16(x, w, out)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    out.zero_()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        torch.ops.cdb.gemm_bf16(x, w, out)  # warm up on the capture stream
    s.synchronize()
    with torch.cuda.graph(g, stream=s):
        torch.ops.cdb.gemm_bf16(x, w, out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert ops.status_code() == 0


def test_lm_head_argmax_op_matches_abi():
    torch.manual_seed(1)
    x = torch.randn(37, 2048, device=DEV).to(torch.bfloat16)
    w = (torch.randn(49152, 2048, device=DEV) * 0.02).to(torch.bfloat16)
    ids = torch.ops.cdb.lm_head_argmax(x, w)
    ref = torch.zeros(37, dtype=torch.int64, device=DEV)
    keys = torch.zeros(256, dtype=torch.int64, device=DEV)
    done = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    work = _lib.GemmWorkspace(torch.device(DEV), 37, 49152, 148)
    _lib.call("cdb_lm_head_argmax", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), 37, 49152, 2048, _lib.ptr(ref),
              None, None, None, _lib.ptr(keys), _lib.ptr(done), *work.args(), 148, _lib.ptr(st), _sp())
    torch.cuda.synchronize()
    assert torch.equal(ids, ref)


class _AttnCase:
    """A paged pool with two cache layers, rows at ragged positions, RoPE tables."""

    def __init__(self, seed: int, n: int = 24, heads: int = 16, d: int = 128, nb: int = 256, bs: int = 16):
        torch.manual_seed(seed)
        self.heads, self.d, self.n, self.bs = heads, d, n, bs
        self.hd = heads * d
        self.kv0 = torch.randn(2, 2, (nb + 2) * bs, heads, d, device=DEV).to(torch.bfloat16)
        self.table = torch.randperm(nb, device=DEV)[: n * 8].view(n, 8).to(torch.int32)
        self.slots = torch.arange(n, dtype=torch.int32, device=DEV)
        self.pos = torch.randint(0, 8 * bs, (n,), device=DEV).to(torch.int32)
        self.qkv = torch.randn(n, 3 * self.hd, device=DEV).to(torch.bfloat16)
        inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        f = torch.arange(8 * bs, device=DEV).float().unsqueeze(-1) * inv.to(DEV)
        emb = torch.cat((f, f), dim=-1)
        self.cos, self.sin = emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()

    def abi(self, qkv, pos, kv, out):
        """cdb_attn_plan + cdb_paged_decode_attn_append with caller buffers sized as the op sizes its own."""

        hg = 4
        items = 4096 // self.heads
        cap = max(items * (self.heads // hg) * 64, self.n * (self.heads // hg)) + _lib.ATTN_PLAN_MAX_CHUNKS
        hdr = torch.zeros(_lib.ATTN_PLAN_HEADER_INTS, dtype=torch.int32, device=DEV)
        units = torch.zeros(cap, 4, dtype=torch.int32, device=DEV)
        part_o = torch.zeros(items * self.heads * 64 * self.d, device=DEV)
        part_ml = torch.zeros(items * self.heads * 64 * 2, device=DEV)
        ctr = torch.zeros(items * self.heads, dtype=torch.int32, device=DEV)
        st = torch.zeros(1, dtype=torch.int32, device=DEV)
        sms = torch.cuda.get_device_properties(DEV).multi_processor_count
        _lib.call("cdb_attn_plan", _lib.ptr(pos), self.n, 2, self.heads, self.d, self.bs, cap, items, sms,
                  _lib.ptr(hdr), _lib.ptr(units), _sp())
        _lib.call("cdb_paged_decode_attn_append", _lib.ptr(qkv), qkv.stride(0), self.hd, 2 * self.hd, _lib.ptr(out),
                  out.stride(0), _lib.ptr(kv), 2, kv.shape[2], 1, _lib.ptr(self.table), self.table.stride(0),
                  _lib.ptr(self.slots), _lib.ptr(pos), 1, _lib.ptr(self.cos), _lib.ptr(self.sin), None, 2,
                  _lib.ptr(hdr), _lib.ptr(units), _lib.ptr(part_o), _lib.ptr(part_ml), _lib.ptr(ctr), items, self.n,
                  self.heads, self.d, self.bs, self.d**-0.5, 2 * sms, _lib.ptr(st), _sp())
        torch.cuda.synchronize()
        assert int(st.item()) == 0

    def op(self, qkv, pos, kv, out):
        torch.ops.cdb.paged_decode_attention(qkv, out, kv, 1, self.table, self.slots, pos, self.cos, self.sin, None, 1,
                                             self.heads, self.d, self.d**-0.5)


def test_attention_and_route_ops_match_abi():
    c = _AttnCase(2)
    outs = []
    for use_op in (False, True):
        kv = c.kv0.clone()
        out = torch.zeros(c.n, c.hd, dtype=torch.bfloat16, device=DEV)
        (c.op if use_op else c.abi)(c.qkv, c.pos, kv, out)
        torch.cuda.synchronize()
        outs.append((out, kv))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    assert ops.status_code() == 0

    sig = torch.tensor([0.5, -2.0, 3.0, 0.0], device=DEV).to(torch.bfloat16)
    hidden = torch.arange(4, dtype=torch.int32, device=DEV)
    step = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device=DEV)
    reset = torch.ones(4, dtype=torch.int8, device=DEV)
    cdf = torch.zeros(4, dtype=torch.float64, device=DEV)
    surv = torch.ones(4, dtype=torch.float64, device=DEV)
    flags, srows, erows, counts = torch.ops.cdb.exit_gate_route(sig, hidden, step, None, reset, cdf, surv, None, 1,
                                                                 False, 1, 4, 0.5)
    torch.cuda.synchronize()
    # sigmoid(0.5) ~ 0.62 >= 0.5 exits; sigmoid(-2) ~ 0.12 stays; sigmoid(3) ~ 0.95 exits; step 3 is forced
    assert flags.tolist() == [1, 0, 1, 1]
    assert counts.tolist() == [1, 3]
    assert srows[:1].tolist() == [1] and erows[:3].tolist() == [0, 2, 3]


def test_attention_op_captured_and_replayed():
    """One eager call (allocates the op's scratch), capture in a graph, then two replays after
    rewriting qkv and item_pos in place; each replay equals the ABI call on the same inputs."""

    c = _AttnCase(3)
    qkv = c.qkv.clone()
    pos = c.pos.clone()
    kv = c.kv0.clone()
    out = torch.zeros(c.n, c.hd, dtype=torch.bfloat16, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        c.op(qkv, pos, kv, out)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        c.op(qkv, pos, kv, out)
    gen = torch.Generator(device=DEV).manual_seed(7)
    for rep in range(2):
        qkv.copy_(torch.randn(qkv.shape, device=DEV, generator=gen).to(torch.bfloat16))
        pos.copy_(torch.randint(0, 8 * c.bs, (c.n,), device=DEV, generator=gen).to(torch.int32))
        kv.copy_(c.kv0)
        ref_kv = c.kv0.clone()
        ref_out = torch.zeros_like(out)
        c.abi(qkv, pos, ref_kv, ref_out)
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), rep
        assert torch.equal(kv, ref_kv), rep
    assert ops.status_code() == 0


def test_attention_op_first_call_inside_capture_raises(monkeypatch):
    """The op's first call on a device allocates; inside a capture it raises before launching."""

    c = _AttnCase(4)
    monkeypatch.setattr(ops, "_ATTN", {})
    out = torch.zeros(c.n, c.hd, dtype=torch.bfloat16, device=DEV)
    kv = c.kv0.clone()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="before capturing"):
        with torch.cuda.graph(g, stream=s):
            c.op(c.qkv, c.pos, kv, out)
