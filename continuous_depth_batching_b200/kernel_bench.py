"""Single-kernel timing on synthetic inputs, through the C ABI, for roofline and profiler runs.

    python -m continuous_depth_batching_b200.kernel_bench attention --rows 128 --context 1024
    python -m continuous_depth_batching_b200.kernel_bench gemm --m 80 --n 2048 --k 2048
    python -m continuous_depth_batching_b200.kernel_bench lm_head --m 32 --vocab 49152 --k 2048
    python -m continuous_depth_batching_b200.kernel_bench gemm_chain --m 80 --n 6144 --k 2048
    python -m continuous_depth_batching_b200.kernel_bench prefill_rows --rows 8192

``attention`` builds a one-cache-layer paged KV pool with the Ouro-1.4B head shape (16 heads x
128), gives each row a context drawn uniformly from [context/2, 3*context/2), and times the
decode attention with CUDA events on the launching stream: cache-only (``--append 0``, the
default), the rope/append kernel followed by the attention kernel (``--append 1``), or the fused
single launch the engine uses (``--append 2``, split-half RoPE). Algorithmic bytes per launch are
``attention_bytes`` below. ``gemm`` times ``cdb_gemm_bf16`` against ``torch.mm`` (cuBLAS) on one
shape, flushing L2 between launches so weights stream from HBM as they do in a decode step.
``prefill_rows`` times, each alone, the row-parallel kernels of one prefill layer at ``--rows``
tokens (Ouro-1.4B widths): the SwiGLU GEMM (against cuBLAS + ``cdb_silu_mul``), the RoPE + KV
append and the residual + sandwich norm. Each prints one JSON line.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _lib

BLOCK = 16


def attention_bytes(positions, num_heads: int, head_dim: int, append: bool) -> int:
    """Algorithmic HBM bytes of one decode-attention launch over rows at ``positions``.

    Per row at position p: K and V rows 0..p read (2*(p+1)*H*D*2 bytes), q read and o written
    (2*H*D*2), the block-table entries (4 bytes per page), and when appending the new k and v
    rows written (2*H*D*2). Padding rows (p < 0) cost nothing.
    """
    row = num_heads * head_dim * 2
    total = 0
    for p in positions:
        if p < 0:
            continue
        total += 2 * (p + 1) * row + 2 * row + 4 * (-(-(p + 1) // BLOCK))
        if append:
            total += 2 * row
    return total


def _events_ms(fn, reps: int, stream, flush: torch.Tensor | None = None) -> float:
    """Median device time of ``fn`` in ms over ``reps`` launches (CUDA events on ``stream``)."""
    times = []
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def run_attention(args) -> dict:
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(args.seed)
    heads, dim = args.heads, args.head_dim
    ctx = torch.randint(args.context // 2, args.context * 3 // 2, (args.rows,), generator=gen)
    pos = (ctx - 1).to(torch.int32)
    nb = (ctx + BLOCK - 1) // BLOCK
    width = int(nb.max())
    num_blocks = int(nb.sum())
    perm = torch.randperm(num_blocks, generator=gen).to(torch.int32)
    table = torch.zeros(args.rows, width, dtype=torch.int32)
    k = 0
    for r in range(args.rows):
        n = int(nb[r])
        table[r, :n] = perm[k : k + n]
        k += n
    kv_rows = (num_blocks + 2) * BLOCK
    kv = torch.empty(1, 2, kv_rows, heads, dim, device=dev, dtype=torch.bfloat16).normal_()
    table = table.to(dev)
    pos_d = pos.to(dev)
    slots = torch.arange(args.rows, dtype=torch.int32, device=dev)
    hd = heads * dim
    qkv = torch.randn(args.rows, 3 * hd, device=dev).to(torch.bfloat16)
    out = torch.empty(args.rows, hd, device=dev, dtype=torch.bfloat16)
    hg = 5 if dim == 96 else 4
    scratch_items = args.scratch_items
    cap = max(scratch_items * (heads // hg) * 64, args.rows * (heads // hg))
    hdr = torch.zeros(_lib.ATTN_PLAN_HEADER_INTS, dtype=torch.int32, device=dev)
    units = torch.zeros(cap, 4, dtype=torch.int32, device=dev)
    part_o = torch.zeros(scratch_items * heads * 64 * dim, device=dev)
    part_ml = torch.zeros(scratch_items * heads * 64 * 2, device=dev)
    counters = torch.zeros(scratch_items * heads, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    append = args.append
    rope_mode = 1 if append else 0
    tab = torch.arange(int(pos.max()) + 1, device=dev, dtype=torch.float32)[:, None] * torch.linspace(
        1.0, 1e-4, dim, device=dev
    )[None, :]
    cos, sin = tab.cos().to(torch.bfloat16).contiguous(), tab.sin().to(torch.bfloat16).contiguous()
    # the plan cuts the work into 2 * num_sms chunks, one per attention CTA: size it for --ctas
    if args.ctas < 2 or args.ctas % 2:
        raise SystemExit("--ctas must be an even number >= 2 (the plan makes two chunks per SM)")
    _lib.call(
        "cdb_attn_plan", _lib.ptr(pos_d), args.rows, append, heads, dim, BLOCK, cap, scratch_items, args.ctas // 2,
        _lib.ptr(hdr), _lib.ptr(units), sp,
    )

    def launch():
        _lib.call(
            "cdb_paged_decode_attn_append", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, _lib.ptr(out), out.stride(0),
            _lib.ptr(kv), 1, kv_rows, 0, _lib.ptr(table), table.stride(0), _lib.ptr(slots), _lib.ptr(pos_d), rope_mode,
            _lib.ptr(cos), _lib.ptr(sin), None, append, _lib.ptr(hdr), _lib.ptr(units), _lib.ptr(part_o),
            _lib.ptr(part_ml), _lib.ptr(counters), scratch_items, args.rows, heads, dim, BLOCK, dim**-0.5, args.ctas,
            _lib.ptr(status), sp,
        )

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    ms = _events_ms(launch, args.iters, stream)
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    algo = attention_bytes(pos.tolist(), heads, dim, append=bool(append))
    return {
        "kernel": f"cdb::decode_attn_kernel<{dim},{hg}>",
        "append": append,
        "rows": args.rows,
        "mean_context": float(ctx.float().mean()),
        "kv_pool_bytes": kv.numel() * 2,
        "plan": [int(x) for x in hdr[:4].tolist()],
        "launch_us": round(ms * 1e3, 2),
        "algorithmic_bytes": algo,
        "achieved_gbs": round(algo / (ms * 1e-3) / 1e9, 1),
    }


def run_gemm(args) -> dict:
    dev = torch.device("cuda")
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    m, n, k = args.m, args.n, args.k
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=dev)).to(torch.bfloat16)
    c = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    ws = _lib.GemmWorkspace(dev, m, n, 148)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def tc():
        _lib.call(
            "cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(c), c.stride(0), m, n, k,
            args.ctas, *ws.args(), 148, _lib.ptr(status), stream.cuda_stream,
        )

    def cublas():
        torch.mm(x, w.t(), out=c)

    res = {"m": m, "n": n, "k": k, "weight_bytes": 2 * n * k}
    for name, fn in (("tcgen05", tc), ("cublas", cublas)):
        if args.only and name != args.only:
            continue
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ms = _events_ms(fn, args.iters, stream, flush)
        byts = 2 * (n * k + m * k + m * n)
        res[name] = {"us": round(ms * 1e3, 2), "gbs": round(byts / (ms * 1e-3) / 1e9, 1),
                     "tflops": round(2 * m * n * k / (ms * 1e-3) / 1e12, 1)}
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    return res


def run_gemm_chain(args) -> dict:
    """Per-GEMM time inside a CUDA graph of ``--layers`` GEMMs of one shape on different weights
    (the shape of a decode step's projections, launch gaps and PDL overlap included), for cuBLAS
    and for cdb_gemm_bf16 at several persistent CTA counts (0 = one per SM)."""

    dev = torch.device("cuda")
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    m, n, k, layers = args.m, args.n, args.k, args.layers
    w = (0.02 * torch.randn(layers, n, k, device=dev)).to(torch.bfloat16)
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _lib.GemmWorkspace(dev, m, n, 148)
    stream = torch.cuda.Stream()
    res = {"m": m, "n": n, "k": k, "layers": layers, "us_per_gemm": {}}
    for ctas in ["cublas", *[int(c) for c in args.ctas_list.split(",")]]:
        def body(ctas=ctas):
            for layer in range(layers):
                if ctas == "cublas":
                    torch.mm(x, w[layer].t(), out=out)
                else:
                    _lib.call(
                        "cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w[layer]), w.stride(1), _lib.ptr(out),
                        out.stride(0), m, n, k, ctas, *ws.args(), 148, _lib.ptr(status), stream.cuda_stream,
                    )

        with torch.cuda.stream(stream):
            body()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
        with torch.cuda.stream(stream):  # replays run on the current stream: make it the timed one
            for _ in range(args.warmup):
                graph.replay()
            ms = _events_ms(graph.replay, args.iters, stream)
        res["us_per_gemm"][str(ctas)] = round(ms * 1e3 / layers, 2)
        del graph
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    return res


def run_proj_norm_chain(args) -> dict:
    """Per-layer time of a projection followed by the residual sandwich norm, inside a CUDA graph
    of ``--layers`` such pairs on different weights: cdb_gemm_bf16 (split-K reduced in the
    GEMM) + cdb_add_rmsnorm, against cdb_gemm_bf16_partials (planes left unreduced) +
    cdb_add_rmsnorm_parts at each split count of ``--splits-list`` (0 = the library's choice)."""

    dev = torch.device("cuda")
    m, n, k, layers = args.m, args.n, args.k, args.layers
    w = (0.02 * torch.randn(layers, n, k, device=dev)).to(torch.bfloat16)
    a = torch.randn(m, k, device=dev).to(torch.bfloat16)
    proj = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    x = torch.randn(m, n, device=dev).to(torch.bfloat16)
    y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    wn = torch.ones(n, device=dev, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _lib.GemmWorkspace(dev, m, n, 148)
    parts = torch.zeros(16 * m * n + 16, dtype=torch.float32, device=dev)
    stride = m * n + (-(m * n)) % 4
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    auto = _lib.load().cdb_gemm_partial_splits(m, n, k, 148)
    res = {"m": m, "n": n, "k": k, "layers": layers, "library_splits": auto, "us_per_layer": {}}
    kb = -(-k // 64)
    for mode in ["reduced", *[int(v) for v in args.splits_list.split(",")]]:
        splits = auto if mode == 0 else mode
        if mode != "reduced" and -(-kb // -(-kb // splits)) != splits:
            continue  # a split would be empty

        def body(mode=mode, splits=splits):
            for layer in range(layers):
                if mode == "reduced":
                    _lib.call(
                        "cdb_gemm_bf16", _lib.ptr(a), k, _lib.ptr(w[layer]), k, _lib.ptr(proj), n, m, n, k, 0,
                        *ws.args(), 148, _lib.ptr(status), sp,
                    )
                    _lib.call(
                        "cdb_add_rmsnorm", _lib.ptr(x), n, _lib.ptr(proj), n, _lib.ptr(wn), _lib.ptr(wn), _lib.ptr(y), n,
                        None, None, None, None, m, n, 1e-6, sp,
                    )
                else:
                    _lib.call(
                        "cdb_gemm_bf16_partials", _lib.ptr(a), k, _lib.ptr(w[layer]), k, _lib.ptr(parts), stride, m, n,
                        k, splits, _lib.ptr(status), sp,
                    )
                    _lib.call(
                        "cdb_add_rmsnorm_parts", _lib.ptr(x), n, _lib.ptr(parts), splits, stride, _lib.ptr(wn),
                        _lib.ptr(wn), _lib.ptr(y), n, None, None, None, None, m, n, 1e-6, sp,
                    )

        with torch.cuda.stream(stream):
            body()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                graph.replay()
            ms = _events_ms(graph.replay, args.iters, stream)
        res["us_per_layer"][str(mode if mode == "reduced" else splits)] = round(ms * 1e3 / layers, 2)
        del graph
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    return res


def run_prefill_attention(args) -> dict:
    """cdb_prefill_attention over ``--prompts`` fresh prompts of ``--length`` tokens each (causal,
    the chunk's K/V already in the paged cache), L2 flushed before every launch. FLOPs count the
    causal QK^T and PV products: 4 * heads * head_dim * L (L + 1) / 2 per prompt."""

    from .runner import OuroRunner

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(args.seed)
    heads, d, n_p, length = args.heads, args.head_dim, args.prompts, args.length
    t = n_p * length
    nb = (length + BLOCK - 1) // BLOCK
    kv_rows = (n_p * nb + 2) * BLOCK
    kv = torch.randn(1, 2, kv_rows, heads, d, device=dev, generator=g).to(torch.bfloat16)
    table = torch.randperm(n_p * nb, device=dev, generator=g).to(torch.int32).view(n_p, nb)
    hd = heads * d
    qkv = torch.randn(t, 3 * hd, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(t, hd, device=dev, dtype=torch.bfloat16)
    item_slot = [r for r in range(n_p) for _ in range(length)]
    item_pos = [i for _ in range(n_p) for i in range(length)]
    tiles = torch.tensor(OuroRunner.prefill_tiles(item_slot, item_pos), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def launch():
        _lib.call(
            "cdb_prefill_attention", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, _lib.ptr(out), out.stride(0),
            _lib.ptr(kv), 1, kv_rows, 0, _lib.ptr(table), table.stride(0), _lib.ptr(tiles), tiles.shape[0], heads,
            d, BLOCK, d**-0.5, _lib.ptr(status), stream.cuda_stream,
        )

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    ms = _events_ms(launch, args.iters, stream, flush)
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    flops = n_p * 4 * heads * d * length * (length + 1) / 2
    return {"kernel": f"cdb::prefill::prefill_attn_kernel<{d}>", "prompts": n_p, "length": length, "tokens": t,
            "tiles": int(tiles.shape[0]), "us": round(ms * 1e3, 2), "tflops": round(flops / (ms * 1e-3) / 1e12, 1)}


def run_lm_head(args) -> dict:
    """cdb_lm_head_argmax against torch.mm (cuBLAS) + cdb_argmax on the same rows."""

    dev = torch.device("cuda")
    m, v, k = args.m, args.vocab, args.k
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    w = (0.02 * torch.randn(v, k, device=dev)).to(torch.bfloat16)
    logits = torch.empty(m, v, device=dev, dtype=torch.bfloat16)
    ids = torch.zeros(m, dtype=torch.int64, device=dev)
    keys = torch.zeros(m, dtype=torch.int64, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _lib.GemmWorkspace(dev, m, v, 148)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def fused():
        _lib.call(
            "cdb_lm_head_argmax", _lib.ptr(x), k, _lib.ptr(w), k, m, v, k, _lib.ptr(ids), None, None, None,
            _lib.ptr(keys), _lib.ptr(done), *ws.args(), 148, _lib.ptr(status), sp,
        )

    def unfused():
        torch.mm(x, w.t(), out=logits)
        _lib.call("cdb_argmax", _lib.ptr(logits), v, m, v, _lib.ptr(ids), None, None, None, sp)

    res = {"m": m, "vocab": v, "k": k, "weight_bytes": 2 * v * k}
    for name, fn in (("fused_tcgen05", fused), ("cublas_plus_argmax", unfused)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ms = _events_ms(fn, args.iters, stream, flush)
        res[name] = {"us": round(ms * 1e3, 2), "gbs": round(2 * v * k / (ms * 1e-3) / 1e9, 1)}
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    return res


def run_prefill_rows(args) -> dict:
    """Prefill-width row kernels, each timed alone with an L2 flush before every launch."""

    dev = torch.device("cuda")
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    t, hidden, inter, heads, d = args.rows, 2048, 5632, 16, 128
    g = torch.Generator(device=dev).manual_seed(args.seed)
    x = torch.randn(t, hidden, device=dev, generator=g).to(torch.bfloat16)
    w_gu = (0.02 * torch.randn(2 * inter, hidden, device=dev, generator=g)).to(torch.bfloat16)
    act = torch.empty(t, inter, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(t, 2 * inter, device=dev, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = _lib.GemmWorkspace(dev, t, 2 * inter, 148)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    # RoPE + append: every row its own position in a fresh request, blocks laid out in order
    hs = heads * d
    qkv = torch.randn(t, 3 * hs, device=dev, generator=g).to(torch.bfloat16)
    nblk = (t + BLOCK - 1) // BLOCK
    pool = torch.zeros(2, nblk * BLOCK, heads, d, device=dev, dtype=torch.bfloat16)
    table = torch.arange(nblk, device=dev, dtype=torch.int32).view(1, nblk)
    slot = torch.zeros(t, device=dev, dtype=torch.int32)
    pos = torch.arange(t, device=dev, dtype=torch.int32)
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float32, device=dev) / d))
    emb = torch.arange(t + 1, dtype=torch.float32, device=dev)[:, None] * inv[None, :]
    emb = torch.cat((emb, emb), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()
    # residual + sandwich norm
    res_x = torch.randn(t, hidden, device=dev, generator=g).to(torch.bfloat16)
    a = torch.randn(t, hidden, device=dev, generator=g).to(torch.bfloat16)
    wn = torch.ones(hidden, device=dev, dtype=torch.bfloat16)
    y = torch.empty(t, hidden, device=dev, dtype=torch.bfloat16)

    def gateup():
        _lib.call(
            "cdb_mlp_gateup_silu_gemm", _lib.ptr(x), hidden, _lib.ptr(w_gu), hidden, _lib.ptr(act), inter, t, inter,
            hidden, 0, *ws.args(), 148, _lib.ptr(status), sp,
        )

    def gateup_cublas():
        torch.mm(x, w_gu.t(), out=gu)
        _lib.call("cdb_silu_mul", _lib.ptr(gu), 2 * inter, _lib.ptr(act), inter, t, inter, sp)

    def rope():
        _lib.call(
            "cdb_rope_append_kv", _lib.ptr(qkv), 3 * hs, hs, 2 * hs, _lib.ptr(pool), 1, nblk * BLOCK, 0,
            _lib.ptr(table), nblk, _lib.ptr(slot), _lib.ptr(pos), 1, _lib.ptr(cos), _lib.ptr(sin), None, t, heads,
            d, BLOCK, sp,
        )

    def norm():
        _lib.call(
            "cdb_add_rmsnorm", _lib.ptr(res_x), hidden, _lib.ptr(a), hidden, _lib.ptr(wn), _lib.ptr(wn), _lib.ptr(y),
            hidden, None, None, None, None, t, hidden, 1e-6, sp,
        )

    res = {"rows": t}
    for name, fn, byts, flops in (
        ("gateup_silu_tcgen05", gateup, 2 * (2 * inter * hidden + t * hidden + t * inter), 2 * t * 2 * inter * hidden),
        ("gateup_cublas_plus_silu_mul", gateup_cublas, 2 * (2 * inter * hidden + t * hidden + t * inter),
         2 * t * 2 * inter * hidden),
        ("rope_append", rope, 2 * 6 * t * hs, 0),
        ("add_rmsnorm", norm, 2 * 4 * t * hidden, 0),
    ):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ms = _events_ms(fn, args.iters, stream, flush)
        res[name] = {"us": round(ms * 1e3, 2), "gbs": round(byts / (ms * 1e-3) / 1e9, 1)}
        if flops:
            res[name]["tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
    if int(status.item()) != 0:
        raise RuntimeError(_lib.load().cdb_status_string(int(status.item())).decode())
    return res


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = p.add_subparsers(dest="kernel", required=True)
    a = sub.add_parser("attention")
    a.add_argument("--rows", type=int, default=128)
    a.add_argument("--context", type=int, default=1024)
    a.add_argument("--heads", type=int, default=16)
    a.add_argument("--head-dim", type=int, default=128)
    a.add_argument("--scratch-items", type=int, default=256)
    a.add_argument("--ctas", type=int, default=296)
    a.add_argument("--append", type=int, choices=[0, 1, 2], default=0)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=80)
    g.add_argument("--n", type=int, default=2048)
    g.add_argument("--k", type=int, default=2048)
    g.add_argument("--ctas", type=int, default=0, help="persistent CTAs (0 = one per SM)")
    g.add_argument("--only", choices=["tcgen05", "cublas"], default=None)
    lm = sub.add_parser("lm_head")
    lm.add_argument("--m", type=int, default=32)
    lm.add_argument("--vocab", type=int, default=49152)
    lm.add_argument("--k", type=int, default=2048)
    gc = sub.add_parser("gemm_chain")
    gc.add_argument("--m", type=int, default=80)
    gc.add_argument("--n", type=int, default=2048)
    gc.add_argument("--k", type=int, default=2048)
    gc.add_argument("--layers", type=int, default=24)
    gc.add_argument("--ctas-list", default="0,148,120,96,74",
                    help="comma-separated CTA counts (0 = the library's choice; > 0 forces stream-K)")
    pa = sub.add_parser("prefill_attention")
    pa.add_argument("--prompts", type=int, default=32)
    pa.add_argument("--length", type=int, default=256)
    pa.add_argument("--heads", type=int, default=16)
    pa.add_argument("--head-dim", type=int, default=128)
    pn = sub.add_parser("proj_norm_chain")
    pn.add_argument("--m", type=int, default=80)
    pn.add_argument("--n", type=int, default=2048)
    pn.add_argument("--k", type=int, default=2048)
    pn.add_argument("--layers", type=int, default=24)
    pn.add_argument("--splits-list", default="0,4,6,8,12,16")
    pr = sub.add_parser("prefill_rows")
    pr.add_argument("--rows", type=int, default=8192)
    for s in (a, g, lm, gc, pr, pn, pa):
        s.add_argument("--warmup", type=int, default=3)
        s.add_argument("--iters", type=int, default=20)
        s.add_argument("--seed", type=int, default=0)
    args = p.parse_args(argv)
    res = {"attention": run_attention, "gemm": run_gemm, "lm_head": run_lm_head, "gemm_chain": run_gemm_chain,
           "prefill_rows": run_prefill_rows, "proj_norm_chain": run_proj_norm_chain,
           "prefill_attention": run_prefill_attention}[
        args.kernel
    ](args)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
