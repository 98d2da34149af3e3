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
    _lib.call("cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(ref), ref.stride(0), 80,
              2048, 2048, 0, None, 0, None, 0, 148, _lib.ptr(st), _sp())
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
    _lib.call("cdb_lm_head_argmax", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), 37, 49152, 2048, _lib.ptr(ref),
              None, None, None, _lib.ptr(keys), _lib.ptr(done), 148, _lib.ptr(st), _sp())
    torch.cuda.synchronize()
    assert torch.equal(ids, ref)


def test_attention_and_route_ops_match_abi():
    torch.manual_seed(2)
    heads, d, n, nb, bs = 16, 128, 24, 256, 16
    hd = heads * d
    kv0 = torch.randn(2, 2, (nb + 2) * bs, heads, d, device=DEV).to(torch.bfloat16)
    table = torch.randperm(nb, device=DEV)[: n * 8].view(n, 8).to(torch.int32)
    slots = torch.arange(n, dtype=torch.int32, device=DEV)
    pos = torch.randint(0, 8 * bs, (n,), device=DEV).to(torch.int32)
    qkv = torch.randn(n, 3 * hd, device=DEV).to(torch.bfloat16)
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    f = torch.arange(8 * bs, device=DEV).float().unsqueeze(-1) * inv.to(DEV)
    emb = torch.cat((f, f), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()
    outs = []
    for use_op in (False, True):
        kv = kv0.clone()
        out = torch.zeros(n, hd, dtype=torch.bfloat16, device=DEV)
        if use_op:
            torch.ops.cdb.paged_decode_attention(qkv, out, kv, 1, table, slots, pos, cos, sin, None, 1, heads, d, d**-0.5)
        else:
            st = torch.zeros(1, dtype=torch.int32, device=DEV)
            _lib.call("cdb_paged_decode_attn_append_static", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, _lib.ptr(out),
                      out.stride(0), _lib.ptr(kv), 2, kv.shape[2], 1, _lib.ptr(table), table.stride(0), _lib.ptr(slots),
                      _lib.ptr(pos), 1, _lib.ptr(cos), _lib.ptr(sin), None, 2, n, heads, d, bs, d**-0.5, 296,
                      _lib.ptr(st), _sp())
        torch.cuda.synchronize()
        outs.append((out, kv))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])

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
