"""``torch.ops.cdb.*``: the library's hot-path entry points as PyTorch custom operators.

A model adapter written against PyTorch (the reference's ``CDBModelAdapter`` seam,
``model_adapter.py:14-102``) can call these instead of ``ctypes``: they take tensors, run on the
current CUDA stream, and raise on CPU tensors (there is no CPU path). Persistent scratch (the
shared status word, the attention plan, the GEMM split workspace) is allocated on an op's first
call on a device, and that call raises instead if the stream is being captured; returned tensors
come from PyTorch's caching allocator. Each wraps one ``include/cdb_b200.h`` entry point:

* ``cdb::gemm_bf16(x, w, out)``: ``out = x @ w.T`` (``cdb_gemm_bf16``);
* ``cdb::mlp_gateup_silu(x, w_gate_up, act)``: SwiGLU of interleaved gate/up rows
  (``cdb_mlp_gateup_silu_gemm``);
* ``cdb::lm_head_argmax(x, w) -> ids``: greedy next tokens without logits (``cdb_lm_head_argmax``);
* ``cdb::add_rmsnorm(x, a, w_a, w_next, y)``: ``x += norm_a(a)``, ``y = norm_next(x)``
  (``cdb_add_rmsnorm``);
* ``cdb::paged_decode_attention(...)``: RoPE, KV append and paged decode attention in one
  launch (``cdb_attn_plan`` + ``cdb_paged_decode_attn_append``). Its work plan and split-combine
  scratch are allocated once per device, on the first call; that first call allocates and so must
  not run while a stream is being captured (the op raises if it does); later calls allocate
  nothing. The scratch is shared by the op's calls on one device, so those calls must be ordered
  (one stream);
* ``cdb::exit_gate_route(...)``: exit decision, routing and compaction of one recurrent launch
  (``cdb_exit_gate_route``).
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["gemm_bf16", "mlp_gateup_silu", "lm_head_argmax", "add_rmsnorm", "paged_decode_attention", "exit_gate_route"]


def _cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("torch.ops.cdb kernels run on CUDA tensors only (sm_100a); there is no CPU path")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _sms(t: torch.Tensor) -> int:
    return torch.cuda.get_device_properties(t.device).multi_processor_count


_STATUS: dict[int, torch.Tensor] = {}
_LM_SCRATCH: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}


def _capturing(t: torch.Tensor) -> bool:
    return torch.cuda.is_current_stream_capturing()


def _status(t: torch.Tensor) -> torch.Tensor:
    idx = t.device.index
    if idx not in _STATUS:
        if _capturing(t):
            raise RuntimeError(
                "torch.ops.cdb: the first call on a device allocates the shared status word; make one call "
                "before capturing a CUDA graph"
            )
        _STATUS[idx] = torch.zeros(1, dtype=torch.int32, device=t.device)
    return _STATUS[idx]


# Decode-attention work plan and split-combine scratch, per device: rows x heads the split
# scratch covers, and the plan's unit capacity, grown (outside capture) when a call needs more.
_ATTN_SCRATCH_ROWHEADS = 4096
_ATTN: dict[int, dict[str, torch.Tensor | int]] = {}


def _attn_scratch(t: torch.Tensor, n_items: int, num_heads: int, head_dim: int) -> dict:
    idx = t.device.index
    hg = 5 if head_dim == 96 else 4
    scratch_items = max(1, _ATTN_SCRATCH_ROWHEADS // num_heads)
    cap = max(scratch_items * (num_heads // hg) * 64, n_items * (num_heads // hg)) + _lib.ATTN_PLAN_MAX_CHUNKS
    cur = _ATTN.get(idx)
    if cur is None or cur["cap"] < cap or cur["head_dim"] < head_dim or cur["scratch_items"] != scratch_items:
        if _capturing(t):
            raise RuntimeError(
                "torch.ops.cdb.paged_decode_attention: the scratch for this shape is not allocated yet; make one "
                "call with the largest batch before capturing a CUDA graph"
            )
        dev = t.device
        cur = {
            "cap": cap,
            "head_dim": head_dim,
            "scratch_items": scratch_items,
            "hdr": torch.zeros(_lib.ATTN_PLAN_HEADER_INTS, dtype=torch.int32, device=dev),
            "units": torch.zeros(cap, 4, dtype=torch.int32, device=dev),
            "part_o": torch.zeros(scratch_items * num_heads * 64 * head_dim, dtype=torch.float32, device=dev),
            "part_ml": torch.zeros(scratch_items * num_heads * 64 * 2, dtype=torch.float32, device=dev),
            "counters": torch.zeros(scratch_items * num_heads, dtype=torch.int32, device=dev),
        }
        _ATTN[idx] = cur
    return cur


# Stream-K GEMM split workspace and tile counters, per device, grown (outside capture) on demand.
_GEMM: dict[int, tuple[int, int, _lib.GemmWorkspace]] = {}


def _gemm_ws(t: torch.Tensor, m: int, n: int) -> tuple:
    idx = t.device.index
    cur = _GEMM.get(idx)
    if cur is None or cur[0] < m or cur[1] < n:
        if _capturing(t):
            raise RuntimeError(
                "torch.ops.cdb: the GEMM workspace for this shape is not allocated yet; make one call with the "
                "largest shape before capturing a CUDA graph"
            )
        m2, n2 = max(m, 256, cur[0] if cur else 0), max(n, 65536, cur[1] if cur else 0)
        cur = (m2, n2, _lib.GemmWorkspace(t.device, m2, n2, _sms(t)))
        _GEMM[idx] = cur
    return cur[2].args()


def _check_index(name: str, t: torch.Tensor | None) -> None:
    if t is not None and (t.dtype != torch.int32 or not t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous int32 tensor, got {t.dtype} (contiguous={t.is_contiguous()})")


def _check_rows(name: str, t: torch.Tensor) -> None:
    if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D bf16 tensor with unit column stride, got {t.dtype} {tuple(t.shape)}")


def status_code(device: torch.device | str | int | None = None) -> int:
    """The device-side status word the ops share on ``device`` (0 = ok); reading it synchronises."""

    dev = torch.device("cuda") if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    s = _STATUS.get(idx)
    return 0 if s is None else int(s.item())


@torch.library.custom_op("cdb::gemm_bf16", mutates_args=("out",))
def gemm_bf16(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
    """``out[M, N] = x[M, K] @ w[N, K].T`` in bf16 with fp32 accumulation (tcgen05)."""

    _cuda(x, w, out)
    m, k = x.shape
    status = _status(x)
    ws = _gemm_ws(x, m, w.shape[0])
    _lib.call(
        "cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(out), out.stride(0), m,
        w.shape[0], k, 0, *ws, _sms(x), _lib.ptr(status), _stream(x),
    )


@torch.library.custom_op("cdb::mlp_gateup_silu", mutates_args=("act",))
def mlp_gateup_silu(x: torch.Tensor, w_gate_up: torch.Tensor, act: torch.Tensor) -> None:
    """``act = silu(x @ Wg.T) * (x @ Wu.T)`` with ``w_gate_up`` rows interleaved (gate j, up j)."""

    _cuda(x, w_gate_up, act)
    m, k = x.shape
    status = _status(x)
    ws = _gemm_ws(x, m, w_gate_up.shape[0])
    _lib.call(
        "cdb_mlp_gateup_silu_gemm", _lib.ptr(x), x.stride(0), _lib.ptr(w_gate_up), w_gate_up.stride(0),
        _lib.ptr(act), act.stride(0), m, w_gate_up.shape[0] // 2, k, 0, *ws, _sms(x), _lib.ptr(status), _stream(x),
    )


@torch.library.custom_op("cdb::lm_head_argmax", mutates_args=())
def lm_head_argmax(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Greedy next token of every row of ``x`` under the LM head ``w [vocab, K]`` (int64 [M])."""

    _cuda(x, w)
    m, k = x.shape
    idx = x.device.index
    if idx not in _LM_SCRATCH or _LM_SCRATCH[idx][0].numel() < m:
        if _capturing(x):
            raise RuntimeError("torch.ops.cdb.lm_head_argmax: make one call with the largest batch before capture")
        _LM_SCRATCH[idx] = (
            torch.zeros(max(m, 256), dtype=torch.int64, device=x.device),
            torch.zeros(1, dtype=torch.int32, device=x.device),
        )
    keys, done = _LM_SCRATCH[idx]
    status = _status(x)
    ws = _gemm_ws(x, m, w.shape[0])
    ids = torch.empty(m, dtype=torch.int64, device=x.device)
    _lib.call(
        "cdb_lm_head_argmax", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), m, w.shape[0], k, _lib.ptr(ids),
        None, None, None, _lib.ptr(keys), _lib.ptr(done), *ws, _sms(x), _lib.ptr(status), _stream(x),
    )
    return ids


@lm_head_argmax.register_fake
def _(x, w):
    return x.new_empty(x.shape[0], dtype=torch.int64)


@torch.library.custom_op("cdb::add_rmsnorm", mutates_args=("x", "y"))
def add_rmsnorm(x: torch.Tensor, a: torch.Tensor, w_a: torch.Tensor, w_next: torch.Tensor, y: torch.Tensor,
                eps: float) -> None:
    """Ouro's sandwich step: ``x = bf16(x + norm_a(a))``, ``y = norm_next(x)`` (bf16 rounding as
    OuroRMSNorm rounds)."""

    _cuda(x, a, w_a, w_next, y)
    _lib.call(
        "cdb_add_rmsnorm", _lib.ptr(x), x.stride(0), _lib.ptr(a), a.stride(0), _lib.ptr(w_a), _lib.ptr(w_next),
        _lib.ptr(y), y.stride(0), None, None, None, None, x.shape[0], x.shape[1], eps, _stream(x),
    )


@torch.library.custom_op("cdb::paged_decode_attention", mutates_args=("out", "kv_pool"))
def paged_decode_attention(
    qkv: torch.Tensor, out: torch.Tensor, kv_pool: torch.Tensor, cache_layer: int, block_table: torch.Tensor,
    item_slot: torch.Tensor, item_pos: torch.Tensor, rope_cos: torch.Tensor | None, rope_sin: torch.Tensor | None,
    qk_bias: torch.Tensor | None, rope_mode: int, num_heads: int, head_dim: int, scale: float,
) -> None:
    """Decode attention of rows at ``item_pos`` over the paged pool ``kv_pool [layers, 2, rows, H, D]``
    with RoPE and the KV append fused (``qkv`` rows hold q | k | v; q is not modified)."""

    _cuda(qkv, out, kv_pool, block_table, item_slot, item_pos, rope_cos, rope_sin, qk_bias)
    if kv_pool.dtype != torch.bfloat16 or kv_pool.dim() != 5 or not kv_pool.is_contiguous():
        raise ValueError("kv_pool must be a contiguous bf16 tensor [layers, 2, rows, heads, head_dim]")
    if kv_pool.shape[1] != 2 or kv_pool.shape[3] != num_heads or kv_pool.shape[4] != head_dim:
        raise ValueError(f"kv_pool shape {tuple(kv_pool.shape)} does not match {num_heads} heads of {head_dim}")
    _check_rows("qkv", qkv)
    _check_rows("out", out)
    for name, t in (("item_slot", item_slot), ("item_pos", item_pos)):
        _check_index(name, t)
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be a 2-D int32 tensor with unit column stride")
    n = item_pos.numel()
    if item_slot.numel() < n or qkv.shape[0] < n or out.shape[0] < n:
        raise ValueError("item_slot, qkv and out need a row per item_pos entry")
    hd = num_heads * head_dim
    if qkv.shape[1] < 3 * hd or out.shape[1] < hd:
        raise ValueError("qkv rows must hold q | k | v and out rows num_heads * head_dim values")
    status = _status(qkv)
    sc = _attn_scratch(qkv, n, num_heads, head_dim)
    stream = _stream(qkv)
    _lib.call(
        "cdb_attn_plan", _lib.ptr(item_pos), n, 2, num_heads, head_dim, 16, sc["cap"], sc["scratch_items"],
        _sms(qkv), _lib.ptr(sc["hdr"]), _lib.ptr(sc["units"]), stream,
    )
    _lib.call(
        "cdb_paged_decode_attn_append", _lib.ptr(qkv), qkv.stride(0), hd, 2 * hd, _lib.ptr(out), out.stride(0),
        _lib.ptr(kv_pool), kv_pool.shape[0], kv_pool.shape[2], cache_layer, _lib.ptr(block_table),
        block_table.stride(0), _lib.ptr(item_slot), _lib.ptr(item_pos), rope_mode, _lib.ptr(rope_cos),
        _lib.ptr(rope_sin), _lib.ptr(qk_bias), 2, _lib.ptr(sc["hdr"]), _lib.ptr(sc["units"]),
        _lib.ptr(sc["part_o"]), _lib.ptr(sc["part_ml"]), _lib.ptr(sc["counters"]), sc["scratch_items"], n,
        num_heads, head_dim, 16, scale, 2 * _sms(qkv), _lib.ptr(status), stream,
    )


@torch.library.custom_op("cdb::exit_gate_route", mutates_args=("cdf", "surv", "pending"))
def exit_gate_route(
    signal: torch.Tensor, hidden: torch.Tensor, step: torch.Tensor, depth: torch.Tensor | None,
    reset: torch.Tensor | None, cdf: torch.Tensor, surv: torch.Tensor, pending: torch.Tensor | None, policy: int,
    delayed: bool, min_steps: int, max_steps: int, threshold: float,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Exit flags, survivor rows, exit rows and ``{num_survivors, num_exits}`` of one launch."""

    _cuda(signal, hidden, step, depth, reset, cdf, surv, pending)
    n = hidden.numel()
    flags = torch.empty(n, dtype=torch.int8, device=hidden.device)
    surv_rows = torch.empty(n, dtype=torch.int32, device=hidden.device)
    exit_rows = torch.empty(n, dtype=torch.int32, device=hidden.device)
    counts = torch.empty(2, dtype=torch.int32, device=hidden.device)
    _lib.call(
        "cdb_exit_gate_route", _lib.ptr(signal), signal.stride(0) if signal.dim() else 1, _lib.ptr(hidden),
        _lib.ptr(step), _lib.ptr(depth), _lib.ptr(reset), _lib.ptr(cdf), _lib.ptr(surv), _lib.ptr(pending), n, policy,
        int(delayed), min_steps, max_steps, threshold, _lib.ptr(flags), _lib.ptr(surv_rows), _lib.ptr(exit_rows),
        _lib.ptr(counts), _stream(hidden),
    )
    return flags, surv_rows, exit_rows, counts


@exit_gate_route.register_fake
def _(signal, hidden, step, depth, reset, cdf, surv, pending, policy, delayed, min_steps, max_steps, threshold):
    n = hidden.numel()
    i32 = torch.int32
    return hidden.new_empty(n, dtype=torch.int8), hidden.new_empty(n, dtype=i32), hidden.new_empty(n, dtype=i32), \
        hidden.new_empty(2, dtype=i32)
