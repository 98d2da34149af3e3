"""Device executor of the CDB decode step: weights, resident state, stage launches, CUDA graphs.

Resident device state (nothing per-request lives on the host side of a launch):

* the paged KV pool and block table (:class:`~.kv_cache.PagedKVPool`);
* the hidden-state bank ``[bank_slots, H]`` bf16 - each in-flight decode token's state between
  recurrent launches (the reference's bank, ``continuous_depth_batching/model_runner.py:1193-1231``);
* the next-token table ``[resident_slots]`` int32 - the coda/prefill argmax writes each request's
  sampled id there and the next prelude embeds from it, so tokens never visit the host on the
  decode path (the reference's on-device successor gather, ``model_runner.py:395-463``);
* the token log ``[sum(max_new_tokens)]`` int64 - every sampled id, read back once at the end.

A recurrent launch uploads one ``[3, B]`` int32 metadata block (resident slot, position, bank slot
per row) and replays the CUDA graph of its padded bucket (``model_runner.py:896-939``): the
attention work plan, then per shared layer ``RMSNorm -> QKV GEMM -> ragged paged attention (RoPE +
KV append fused) -> O GEMM -> residual+norm -> gate/up GEMM -> SwiGLU -> down GEMM ->
residual+norm``, the last norm scattering into the bank and computing the exit-gate logit.
Every kernel is libcdb_b200's: the projections and the LM head run on its stream-K tcgen05 GEMM
(``cdb_gemm_bf16``, SwiGLU fused into the gate/up projection, greedy argmax fused into the LM
head), which shares one split-partial workspace per replica.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from .kv_cache import LoopedKvLayout, PagedKVPool, kv_slot_for_step
from .ouro import LAYER_NORM_NAMES, OuroShape

SCRATCH_ITEMS = 256


def decode_graph_buckets(max_num_seqs: int) -> list[int]:
    """Padded batch sizes, one CUDA graph each: the list ``continuous_batching/utils.py:65-76`` uses."""

    sizes = [1, 2, 4, 8, 12, *range(16, 257, 8), *range(272, 512, 16), *range(512, max_num_seqs + 1, 32)]
    return sorted({s for s in sizes if s <= max_num_seqs} | {max_num_seqs})


class Uploader:
    """Asynchronous host-to-device copies of small int32 arrays through a ring of pinned buffers.

    A pinned buffer is rewritten only after the event of its previous copy has fired, so the
    host can run many launches ahead of the device without a synchronisation per launch.
    """

    def __init__(self, device: torch.device, slots: int = 64, capacity: int = 1 << 15) -> None:
        self.device = device
        self.slots = slots
        self.host = [torch.empty(capacity, dtype=torch.int32, pin_memory=True) for _ in range(slots)]
        self.dev = [torch.empty(capacity, dtype=torch.int32, device=device) for _ in range(slots)]
        self.events: list[torch.cuda.Event | None] = [None] * slots
        self.i = 0

    def upload(self, values, stream: torch.cuda.Stream, out: torch.Tensor | None = None) -> torch.Tensor:
        arr = np.asarray(values, dtype=np.int32).reshape(-1)
        i = self.i
        self.i = (i + 1) % self.slots
        ev = self.events[i]
        if ev is not None:
            ev.synchronize()
        n = arr.size
        if n > self.host[i].numel():
            self.host[i] = torch.empty(2 * n, dtype=torch.int32, pin_memory=True)
            self.dev[i] = torch.empty(2 * n, dtype=torch.int32, device=self.device)
        self.host[i][:n].numpy()[:] = arr
        dst = self.dev[i][:n] if out is None else out.view(-1)[:n]
        with torch.cuda.stream(stream):
            dst.copy_(self.host[i][:n], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
        self.events[i] = ev
        return dst


@dataclass
class PackedOuroWeights:
    """bf16 device weights with the projections the kernels fuse concatenated.

    ``w_qkv`` is ``[q; k; v]`` stacked; ``w_gu`` holds row pairs ``(gate_j, up_j)`` as
    ``cdb_mlp_gateup_silu_gemm`` reads them.
    """

    embed: torch.Tensor
    w_qkv: list[torch.Tensor]
    w_o: list[torch.Tensor]
    w_gu: list[torch.Tensor]
    w_down: list[torch.Tensor]
    norms: dict[str, list[torch.Tensor]]
    final_norm: torch.Tensor
    gate_w: torch.Tensor
    gate_b: torch.Tensor
    lm_head: torch.Tensor

    @classmethod
    def from_state_dict(cls, shape: OuroShape, sd: dict[str, torch.Tensor], device: torch.device) -> PackedOuroWeights:
        def g(name: str) -> torch.Tensor:
            return sd[name].detach().to(device=device, dtype=torch.bfloat16).contiguous()

        def gate_up(p: str) -> torch.Tensor:
            gate, up = g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")
            return torch.stack([gate, up], dim=1).reshape(2 * gate.shape[0], gate.shape[1]).contiguous()

        L = shape.num_hidden_layers
        pre = [f"model.layers.{i}." for i in range(L)]
        return cls(
            embed=g("model.embed_tokens.weight"),
            w_qkv=[
                torch.cat([g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight"), g(p + "self_attn.v_proj.weight")]).contiguous()
                for p in pre
            ],
            w_o=[g(p + "self_attn.o_proj.weight") for p in pre],
            w_gu=[gate_up(p) for p in pre],
            w_down=[g(p + "mlp.down_proj.weight") for p in pre],
            norms={n: [g(p + n + ".weight") for p in pre] for n in LAYER_NORM_NAMES},
            final_norm=g("model.norm.weight"),
            gate_w=g("model.early_exit_gate.weight").reshape(-1).contiguous(),
            gate_b=g("model.early_exit_gate.bias").reshape(-1).contiguous(),
            lm_head=g("lm_head.weight"),
        )


@dataclass
class _Graph:
    graph: torch.cuda.CUDAGraph
    meta: torch.Tensor  # [3, bucket] int32 static metadata
    launches: int  # libcdb kernels one replay runs


@dataclass
class RunnerStats:
    recurrent_graph_hits: int = 0
    recurrent_graph_captures: int = 0
    captured_calls: int = 0  # library calls recorded into graphs (not executed at capture time)
    replayed_launches: int = 0

    @property
    def kernel_launches(self) -> int:
        """libcdb kernels executed on the device so far (eager calls + kernels inside graph replays)."""

        return _lib.launch_count - self.captured_calls + self.replayed_launches


class OuroRunner:
    """Owns the device side of one engine replica (one GPU)."""

    #: int32 rows of a recurrent launch's metadata block (resident slot, position, bank slot)
    meta_rows = 3

    def __init__(
        self,
        shape: OuroShape,
        state_dict: dict[str, torch.Tensor],
        *,
        device: torch.device,
        kv_policy: str,
        kv_slots_per_layer: int,
        num_blocks: int,
        block_size: int,
        max_model_len: int,
        max_num_seqs: int,
        max_num_batched_tokens: int,
        use_cuda_graph: bool = True,
        fused_lm_head: bool = True,
    ) -> None:
        I = shape.intermediate_size
        self._init_device(
            shape,
            device=device,
            kv_policy=kv_policy,
            kv_slots_per_layer=kv_slots_per_layer,
            layout=LoopedKvLayout(
                num_prelude_layers=0, num_core_layers=shape.num_hidden_layers, num_coda_layers=0,
                total_recurrent_steps=shape.total_ut_steps, policy=kv_policy, requested_slots=kv_slots_per_layer,
            ),
            num_blocks=num_blocks,
            block_size=block_size,
            max_model_len=max_model_len,
            max_num_seqs=max_num_seqs,
            max_num_batched_tokens=max_num_batched_tokens,
            use_cuda_graph=use_cuda_graph,
            fused_lm_head=fused_lm_head,
            max_gemm_n=max(shape.vocab_size, 2 * I, 3 * shape.num_attention_heads * shape.head_dim),
        )
        self.w = PackedOuroWeights.from_state_dict(shape, state_dict, device)
        H, D = shape.hidden_size, shape.head_dim
        Hq = shape.num_attention_heads * D
        Hk = shape.num_key_value_heads * D
        self.qkv_width = Hq + 2 * Hk
        self.k_col, self.v_col = Hq, Hq + Hk
        rows = self.rows
        bf = dict(dtype=torch.bfloat16, device=device)
        self.xw = torch.zeros(rows, H, **bf)
        self.h = torch.zeros(rows, H, **bf)
        self.qkv = torch.zeros(rows, self.qkv_width, **bf)
        self.attn = torch.zeros(rows, Hq, **bf)
        self.o = torch.zeros(rows, H, **bf)
        self.act = torch.zeros(rows, I, **bf)
        self.m = torch.zeros(rows, H, **bf)
        self.gate_out = torch.zeros(max_num_seqs, **bf)
        self.bank_slots = 2 * max_num_seqs + 8
        self.bank = torch.zeros(self.bank_slots, H, **bf)
        self.logits = torch.zeros(max_num_seqs, shape.vocab_size, **bf)
        self.lm_in = torch.zeros(max_num_seqs, shape.hidden_size, **bf)  # gathered LM-head input rows
        # RoPE tables: fp32 inv_freq x position, cos/sin in fp32, cast to bf16 (modeling_ouro.py:560-573)
        max_pos = max_model_len + 1
        inv = 1.0 / (shape.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(torch.float32) / D))
        freqs = torch.arange(max_pos, dtype=torch.float32, device=device)[:, None] * inv.to(device)[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        self.rope_cos = emb.cos().to(torch.bfloat16).contiguous()
        self.rope_sin = emb.sin().to(torch.bfloat16).contiguous()

    def _init_device(
        self,
        shape,
        *,
        device: torch.device,
        kv_policy: str,
        kv_slots_per_layer: int,
        layout: LoopedKvLayout,
        num_blocks: int,
        block_size: int,
        max_model_len: int,
        max_num_seqs: int,
        max_num_batched_tokens: int,
        use_cuda_graph: bool,
        fused_lm_head: bool = True,
        max_gemm_n: int = 65536,
    ) -> None:
        """Model-independent device state: KV pool, stream, uploads, GEMM and attention scratch, graphs."""

        if device.type != "cuda":
            raise RuntimeError("the B200 CDB runner needs a CUDA device; there is no CPU path")
        _lib.load()
        self.shape = shape
        self.device = device
        self.kv_policy = kv_policy
        self.slots = kv_slots_per_layer
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.use_cuda_graph = use_cuda_graph
        self.layout = layout
        self.pool = PagedKVPool(
            num_cache_layers=layout.num_cache_layers,
            num_blocks=num_blocks,
            block_size=block_size,
            num_kv_heads=shape.num_key_value_heads,
            head_dim=shape.head_dim,
            max_model_len=max_model_len,
            resident_slots=max_num_seqs,
            device=device,
        )
        self.stream = torch.cuda.Stream(device=device)
        self.uploader = Uploader(device)
        self.num_sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.attn_ctas = 2 * self.num_sms
        D = shape.head_dim
        self.rows = max(max_num_seqs, max_num_batched_tokens)
        # split partials + tile counters of the stream-K GEMM, shared by every projection (one stream)
        self.gemm = _lib.GemmWorkspace(device, self.rows, max_gemm_n, self.num_sms)
        self.token_table = torch.zeros(max_num_seqs, dtype=torch.int32, device=device)
        self.token_log = torch.zeros(1, dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        # attention plan + split-combine scratch
        nh = shape.num_attention_heads
        hg = 5 if D == 96 else 4
        self.unit_capacity = max(SCRATCH_ITEMS * (nh // hg) * 64, self.rows * (nh // hg)) + _lib.ATTN_PLAN_MAX_CHUNKS
        self.plan_hdr = torch.zeros(_lib.ATTN_PLAN_HEADER_INTS, dtype=torch.int32, device=device)
        self.units = torch.zeros(self.unit_capacity, 4, dtype=torch.int32, device=device)
        self.part_o = torch.zeros(SCRATCH_ITEMS * nh * 64 * D, dtype=torch.float32, device=device)
        self.part_ml = torch.zeros(SCRATCH_ITEMS * nh * 64 * 2, dtype=torch.float32, device=device)
        self.counters = torch.zeros(SCRATCH_ITEMS * nh, dtype=torch.int32, device=device)
        self.scale = float(D) ** -0.5
        # LM head + greedy argmax in one tcgen05 GEMM (no logits in HBM; cdb_lm_head_argmax),
        # unless logits are kept for inspection
        self.fused_lm_head = fused_lm_head
        self.lm_keys = torch.zeros(max_num_seqs, dtype=torch.int64, device=device)
        self.lm_done = torch.zeros(1, dtype=torch.int32, device=device)
        self.buckets = decode_graph_buckets(max_num_seqs)
        self.graphs: dict[tuple[int, int, bool], _Graph] = {}
        self.graph_pool = None
        self.stats = RunnerStats()

    def _lm_head_argmax(self, x: torch.Tensor, n: int, w: torch.Tensor, out_rows, token_rows, keep_logits: bool):
        """Greedy next tokens of rows [0, n) of ``x`` into the token log / table; the logits when kept."""

        s = self.shape
        if self.fused_lm_head and not keep_logits:
            _lib.call(
                "cdb_lm_head_argmax", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), n, s.vocab_size,
                x.shape[1], _lib.ptr(self.token_log), _lib.ptr(out_rows), _lib.ptr(token_rows),
                _lib.ptr(self.token_table), _lib.ptr(self.lm_keys), _lib.ptr(self.lm_done), *self.gemm.args(),
                self.num_sms, _lib.ptr(self.status), self._sp(),
            )
            return None
        self._mm(x[:n], w, self.logits[:n])
        _lib.call(
            "cdb_argmax", _lib.ptr(self.logits), self.logits.stride(0), n, s.vocab_size, _lib.ptr(self.token_log),
            _lib.ptr(out_rows), _lib.ptr(token_rows), _lib.ptr(self.token_table), self._sp(),
        )
        return self.logits[:n].clone() if keep_logits else None

    # ------------------------------------------------------------------ cache-layer layout
    @property
    def num_core_layers(self) -> int:
        """Physical layers one recurrent step runs (the ones whose KV is replicated per slot)."""

        return self.layout.num_core_layers

    def core_cache_layer(self, slot: int, layer: int) -> int:
        """Cache layer of a recurrent layer at a KV slot (``LoopedKvLayout.core_layer_index``,
        ``kv_cache_policy.py:214-227``)."""

        return self.layout.core_slot_layer_index(slot, layer)

    # ------------------------------------------------------------------ small helpers
    def reset(self, log_capacity: int) -> None:
        self.pool.pool.reset()
        self.pool.block_table.fill_(-1)
        if self.token_log.numel() < log_capacity:
            self.token_log = torch.zeros(log_capacity, dtype=torch.int64, device=self.device)
        self.status.zero_()

    def upload(self, values) -> torch.Tensor:
        return self.uploader.upload(values, self.stream)

    def rebind_token(self, req_slot: int, log_row: int) -> None:
        """Set a request's device token (token table row ``req_slot``) to the token at ``log_row``
        of the token log: a request restored from the host pool resumes in a new block-table row,
        and its pending decode token must follow it there."""

        with torch.cuda.stream(self.stream):
            self.token_table[req_slot : req_slot + 1].copy_(self.token_log[log_row : log_row + 1])

    def flush_block_edits(self) -> None:
        self.pool.flush_edits(self.upload, self.stream)

    def check_status(self) -> None:
        st = int(self.status.item())
        if st != 0:
            raise _lib.CDBError(f"device-side error: {_lib.load().cdb_status_string(st).decode()} ({st})")

    def _sp(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _mm(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        """out = a @ w^T on the library's stream-K tcgen05 GEMM."""

        m, k = a.shape
        _lib.call(
            "cdb_gemm_bf16", _lib.ptr(a), a.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(out), out.stride(0),
            m, w.shape[0], k, 0, *self.gemm.args(), self.num_sms, _lib.ptr(self.status), self._sp(),
        )

    def _mm_norm(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, x, w_a, w_next, y, y_rows,
                 gate_w, gate_b, gate_out) -> None:
        """out = a @ w^T, then the residual sandwich norm x += norm(out; w_a), y = norm(x; w_next)
        (cdb_add_rmsnorm). The split-K GEMM reduces its partials itself: leaving them unreduced
        for the norm to sum (cdb_gemm_bf16_partials + cdb_add_rmsnorm_parts) was 2 us faster per
        pair in an isolated graph chain but 1% slower over the bench's decode step."""

        m = a.shape[0]
        H = self.shape.hidden_size
        sp = self._sp()
        self._mm(a, w, out)
        _lib.call(
            "cdb_add_rmsnorm", _lib.ptr(x), x.stride(0), _lib.ptr(out), out.stride(0), _lib.ptr(w_a),
            _lib.ptr(w_next), _lib.ptr(y), y.stride(0), _lib.ptr(y_rows), _lib.ptr(gate_w), _lib.ptr(gate_b),
            _lib.ptr(gate_out), m, H, self.shape.rms_norm_eps, sp,
        )

    def _gate_up(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        """out = silu(a @ Wg^T) * (a @ Wu^T) for interleaved gate/up rows ``w`` (one GEMM)."""

        m, k = a.shape
        _lib.call(
            "cdb_mlp_gateup_silu_gemm", _lib.ptr(a), a.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(out),
            out.stride(0), m, w.shape[0] // 2, k, 0, *self.gemm.args(), self.num_sms, _lib.ptr(self.status),
            self._sp(),
        )

    # ------------------------------------------------------------------ stage bodies
    def _plan(self, item_pos: torch.Tensor, n: int, append: int) -> None:
        s = self.shape
        _lib.call(
            "cdb_attn_plan", _lib.ptr(item_pos), n, append, s.num_attention_heads, s.head_dim, self.block_size,
            self.unit_capacity, SCRATCH_ITEMS, self.num_sms, _lib.ptr(self.plan_hdr), _lib.ptr(self.units), self._sp(),
        )

    def _attention(self, n: int, cache_layer: int, item_slot, item_pos, append: int, rope_mode: int) -> None:
        s = self.shape
        pool = self.pool
        _lib.call(
            "cdb_paged_decode_attn_append",
            _lib.ptr(self.qkv), self.qkv.stride(0), self.k_col, self.v_col,
            _lib.ptr(self.attn), self.attn.stride(0),
            _lib.ptr(pool.kv), pool.num_cache_layers, pool.rows, cache_layer,
            _lib.ptr(pool.block_table), pool.block_table.stride(0), _lib.ptr(item_slot), _lib.ptr(item_pos),
            rope_mode, _lib.ptr(self.rope_cos), _lib.ptr(self.rope_sin), None, append,
            _lib.ptr(self.plan_hdr), _lib.ptr(self.units), _lib.ptr(self.part_o), _lib.ptr(self.part_ml),
            _lib.ptr(self.counters), SCRATCH_ITEMS, n, s.num_attention_heads, s.head_dim, self.block_size,
            self.scale, self.attn_ctas, _lib.ptr(self.status), self._sp(),
        )

    def _prefill_attention(self, cache_layer: int) -> None:
        """Tiled causal attention of the current prefill batch (tiles uploaded by ``prefill``)."""

        s, pool = self.shape, self.pool
        _lib.call(
            "cdb_prefill_attention", _lib.ptr(self.qkv), self.qkv.stride(0), self.k_col, self.v_col,
            _lib.ptr(self.attn), self.attn.stride(0), _lib.ptr(pool.kv), pool.num_cache_layers, pool.rows,
            cache_layer, _lib.ptr(pool.block_table), pool.block_table.stride(0), _lib.ptr(self._tiles),
            self._num_tiles, s.num_attention_heads, s.head_dim, self.block_size, self.scale, _lib.ptr(self.status),
            self._sp(),
        )

    @staticmethod
    def prefill_tiles(item_slot: list[int], item_pos: list[int], tile_rows: int = 64) -> list[tuple[int, int, int, int]]:
        """Split prefill rows into runs of <= 64 consecutive positions of one request, ordered by
        the keys they attend to, most first: the kernel's CTAs start in tile order, so the longest
        tiles start first and the short ones fill the tail."""

        tiles: list[tuple[int, int, int, int]] = []
        start = 0
        n = len(item_slot)
        for i in range(1, n + 1):
            if (
                i == n
                or item_slot[i] != item_slot[start]
                or item_pos[i] != item_pos[i - 1] + 1
                or i - start == tile_rows
            ):
                tiles.append((start, i - start, item_slot[start], item_pos[start]))
                start = i
        tiles.sort(key=lambda t: -(t[3] + t[1]))  # stable: ties keep row order
        return tiles

    def _layer_stack(self, n: int, base_layer: int, item_slot, item_pos, append: int, final_dst, final_rows, gate: bool):
        """All shared layers over rows ``[0, n)`` of the work buffers; residual stream in ``xw``."""

        s, w = self.shape, self.w
        L = s.num_hidden_layers
        sp = self._sp()
        for l in range(L):
            self._mm(self.h[:n], w.w_qkv[l], self.qkv[:n])
            if append:
                self._attention(n, base_layer + l, item_slot, item_pos, 2, 1)  # RoPE + KV append fused
            else:
                _lib.call(
                    "cdb_rope_append_kv", _lib.ptr(self.qkv), self.qkv.stride(0), self.k_col, self.v_col,
                    _lib.ptr(self.pool.kv), self.pool.num_cache_layers, self.pool.rows, base_layer + l,
                    _lib.ptr(self.pool.block_table), self.pool.block_table.stride(0), _lib.ptr(item_slot),
                    _lib.ptr(item_pos), 1, _lib.ptr(self.rope_cos), _lib.ptr(self.rope_sin), None, n,
                    s.num_attention_heads, s.head_dim, self.block_size, sp,
                )
                self._prefill_attention(base_layer + l)
            self._mm_norm(
                self.attn[:n], w.w_o[l], self.o[:n], self.xw, w.norms["input_layernorm_2"][l],
                w.norms["post_attention_layernorm"][l], self.h, None, None, None, None,
            )
            self._gate_up(self.h[:n], w.w_gu[l], self.act[:n])
            # x += norm(m); then the next layer's input norm, or after the last layer the final norm
            # scattered into the bank (and the exit-gate logit)
            last = l == L - 1
            w_next = w.final_norm if last else w.norms["input_layernorm"][l + 1]
            y, y_rows = (final_dst, final_rows) if last else (self.h, None)
            g = last and gate
            self._mm_norm(
                self.act[:n], w.w_down[l], self.m[:n], self.xw, w.norms["post_attention_layernorm_2"][l], w_next,
                y, y_rows, w.gate_w if g else None, w.gate_b if g else None, self.gate_out if g else None,
            )

    def _recurrent_body(self, meta: torch.Tensor, n: int, kv_slot: int, gate: bool) -> None:
        s = self.shape
        item_slot, item_pos, hid = meta[0], meta[1], meta[2]
        self._plan(item_pos, n, 1)
        _lib.call(
            "cdb_rmsnorm", _lib.ptr(self.bank), self.bank.stride(0), _lib.ptr(hid),
            _lib.ptr(self.w.norms["input_layernorm"][0]), _lib.ptr(self.h), self.h.stride(0),
            _lib.ptr(self.xw), self.xw.stride(0), n, s.hidden_size, s.rms_norm_eps, self._sp(),
        )
        self._layer_stack(n, kv_slot * s.num_hidden_layers, item_slot, item_pos, 1, self.bank, hid, gate)

    # ------------------------------------------------------------------ public stages
    def _recurrent_meta(self, item_slot: list[int], item_pos: list[int], hidden: list[int], steps) -> list[list[int]]:
        """The int32 metadata rows of a recurrent launch (``meta_rows`` of them)."""

        return [item_slot, item_pos, hidden]

    def recurrent(
        self,
        item_slot: list[int],
        item_pos: list[int],
        hidden: list[int],
        kv_slot: int,
        gate: bool,
        steps: list[int] | None = None,
    ) -> None:
        """One mixed-depth recurrent launch over ``len(item_slot)`` rows (each at its own step)."""

        n = len(item_slot)
        self.flush_block_edits()
        rows = self._recurrent_meta(item_slot, item_pos, hidden, steps)
        if not self.use_cuda_graph:
            meta = self.upload(rows).view(self.meta_rows, n)
            with torch.cuda.stream(self.stream):
                self._recurrent_body(meta, n, kv_slot, gate)
            return
        bucket = next(b for b in self.buckets if b >= n)
        key = (bucket, kv_slot, gate)
        g = self.graphs.get(key)
        if g is None:
            g = self._capture(bucket, kv_slot, gate)
            self.stats.recurrent_graph_captures += 1
        else:
            self.stats.recurrent_graph_hits += 1
        meta_host = np.full((self.meta_rows, bucket), -1, dtype=np.int32)
        for i, row in enumerate(rows):
            meta_host[i, :n] = row
        meta_host[0, n:] = 0
        self.uploader.upload(meta_host, self.stream, out=g.meta)
        with torch.cuda.stream(self.stream):
            g.graph.replay()
        self.stats.replayed_launches += g.launches

    def _capture(self, bucket: int, kv_slot: int, gate: bool) -> _Graph:
        meta = torch.full((self.meta_rows, bucket), -1, dtype=torch.int32, device=self.device)
        meta[0].zero_()
        # Warm up on a fully padded batch (every kernel skips padding rows), then capture.
        with torch.cuda.stream(self.stream):
            self._recurrent_body(meta, bucket, kv_slot, gate)
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        before = _lib.launch_count
        with torch.cuda.graph(graph, pool=self.graph_pool, stream=self.stream):
            self._recurrent_body(meta, bucket, kv_slot, gate)
        captured = _lib.launch_count - before
        self.stats.captured_calls += captured
        if self.graph_pool is None:
            self.graph_pool = graph.pool()
        g = _Graph(graph=graph, meta=meta, launches=captured)
        self.graphs[(bucket, kv_slot, gate)] = g
        return g

    def prefill(
        self,
        token_ids: list[int],
        item_slot: list[int],
        item_pos: list[int],
        logit_rows: list[int],
        log_rows: list[int],
        req_slots: list[int],
        slot_for_step: list[int],
        keep_logits: bool = False,
    ) -> torch.Tensor | None:
        """Full-depth monolithic prefill over a varlen batch of prompt chunks (no early exit)."""

        s = self.shape
        n = len(token_ids)
        self.flush_block_edits()
        meta = self.upload([token_ids, item_slot, item_pos]).view(3, n)
        k = len(logit_rows)
        sel = self.upload([logit_rows, log_rows, req_slots]).view(3, k) if k else None
        sp = self.stream.cuda_stream
        with torch.cuda.stream(self.stream):
            _lib.call(
                "cdb_embed", _lib.ptr(self.w.embed), s.hidden_size, s.vocab_size, _lib.ptr(meta[0]), None, None,
                _lib.ptr(self.xw), self.xw.stride(0), None, n, 1.0, _lib.ptr(self.status), sp,
            )
            tiles = self.prefill_tiles(item_slot, item_pos)
            self._tiles = self.upload(tiles)
            self._num_tiles = len(tiles)
            for step in range(s.total_ut_steps):
                _lib.call(
                    "cdb_rmsnorm", _lib.ptr(self.xw), self.xw.stride(0), None,
                    _lib.ptr(self.w.norms["input_layernorm"][0]), _lib.ptr(self.h), self.h.stride(0), None, 0, n,
                    s.hidden_size, s.rms_norm_eps, sp,
                )
                base = slot_for_step[step] * s.num_hidden_layers
                self._layer_stack(n, base, meta[1], meta[2], 0, self.xw, None, False)
            if k:
                _lib.call(
                    "cdb_gather_rows", _lib.ptr(self.xw), self.xw.stride(0), _lib.ptr(sel[0]), k, s.hidden_size,
                    _lib.ptr(self.lm_in), self.lm_in.stride(0), sp,
                )
                return self._lm_head_argmax(self.lm_in, k, self.w.lm_head, sel[1], sel[2], keep_logits)
        return None

    def prelude(self, token_ids: list[int], req_slots: list[int], hidden: list[int], positions=None) -> None:
        """Embed each item's token into its bank slot; id -1 takes the request's device token.

        ``positions`` is unused: Ouro's prelude is a lookup with no attention."""

        s = self.shape
        n = len(token_ids)
        if n == 0:
            return
        meta = self.upload([token_ids, req_slots, hidden]).view(3, n)
        with torch.cuda.stream(self.stream):
            _lib.call(
                "cdb_embed", _lib.ptr(self.w.embed), s.hidden_size, s.vocab_size, _lib.ptr(meta[0]),
                _lib.ptr(meta[1]), _lib.ptr(self.token_table), _lib.ptr(self.bank), self.bank.stride(0),
                _lib.ptr(meta[2]), n, 1.0, _lib.ptr(self.status), self.stream.cuda_stream,
            )

    def coda(
        self, hidden: list[int], log_rows: list[int], req_slots: list[int], keep_logits: bool = False, positions=None
    ):
        """LM head + greedy argmax for exited tokens; ids go to the token log and token table.

        ``positions`` is unused: Ouro's coda is the LM head alone."""

        s = self.shape
        n = len(hidden)
        meta = self.upload([hidden, log_rows, req_slots]).view(3, n)
        with torch.cuda.stream(self.stream):
            _lib.call(
                "cdb_gather_rows", _lib.ptr(self.bank), self.bank.stride(0), _lib.ptr(meta[0]), n, s.hidden_size,
                _lib.ptr(self.lm_in), self.lm_in.stride(0), self.stream.cuda_stream,
            )
            return self._lm_head_argmax(self.lm_in, n, self.w.lm_head, meta[1], meta[2], keep_logits)

    def exit_kv_copy(self, rows: list[int], pairs: list[tuple[int, int]]) -> None:
        if not rows or not pairs:
            return
        p = self.pool
        meta = self.upload([rows])
        src = self.upload([a for a, _ in pairs])
        dst = self.upload([b for _, b in pairs])
        with torch.cuda.stream(self.stream):
            _lib.call(
                "cdb_exit_kv_copy", _lib.ptr(p.kv), p.num_cache_layers, p.rows, p.num_kv_heads, p.head_dim,
                _lib.ptr(meta), len(rows), _lib.ptr(src), _lib.ptr(dst), len(pairs), self.stream.cuda_stream,
            )

    def gate_signals(self, n: int) -> torch.Tensor:
        """Host copy of the last recurrent launch's exit-gate logits (synchronises the stream)."""

        with torch.cuda.stream(self.stream):
            out = self.gate_out[:n].float().cpu()
        return out

    def read_tokens(self, count: int) -> list[int]:
        self.stream.synchronize()
        return self.token_log[:count].cpu().tolist()

    def slot_for_step(self, step: int) -> int:
        return kv_slot_for_step(step, policy=self.kv_policy, slots_per_layer=self.slots)
