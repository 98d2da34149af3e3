"""Device executor of the CDB decode step for Huginn (prelude / recurrent core / coda).

Shares the Ouro runner's machinery (paged KV pool and device block table, uploads, the split-KV
attention plan, CUDA graphs per (bucket, KV slot, gate) for the recurrent launch) and differs
in the stages, following ``HuginnCDBAdapter`` (``continuous_depth_batching/adapters/huginn.py``):

* two banks of ``[bank_slots, E]`` bf16 instead of one packed ``[state | injection]`` vector:
  ``inj_bank`` holds the prelude output of every in-flight token, ``state_bank`` its recurrent
  state. A token at step 0 reads a zero state (``state_init="zero"``): its state-source row in
  the launch metadata is -1, which the gather turns into zeros;
* prelude (decode): ``wte(id) * sqrt(E)`` then the prelude blocks, each writing its own cache
  layer at the token's position (``LoopedKvLayout.prelude_layer_index``), into ``inj_bank``;
* recurrent step: ``adapter([state | injection])`` then the core blocks at the launch's KV slot
  (``core_layer_index``), the new state into ``state_bank``; the exit signal is
  ``latent_diff(new, old)`` in bf16 (``exit_gates.py:33-40``);
* coda: ``ln_f`` of the state, the coda blocks (``coda_layer_index``), ``ln_f`` again, the LM
  head tied to ``wte``, greedy argmax into the token log / next-token table;
* prefill: ``HuginnForCausalLM.forward`` at full depth over a varlen batch of prompt chunks
  (prelude, ``total_recurrent_steps`` core steps from a zero state, coda).

Decode prelude and coda launches replay CUDA graphs per padded batch size, as the recurrent
launch does; padding rows carry position -1 (no attention work, no KV append) and bank / output
rows -1 (nothing stored). A prelude padding row embeds token 0 (id 0, slot 0): an id of -1 would
read the request's device token through slot -1.

Every block (``HuginnBlock.forward``, ``modeling_huginn.py:333-336``) is
``QKV GEMM -> q/k bias + interleaved fp32 RoPE + KV append -> paged attention -> proj GEMM ->
x = norm_2(o + x), h = norm_3(x) -> fc GEMM + SwiGLU -> mlp proj GEMM -> x = norm_4(m + x),
h = next norm`` with the two norm pairs in one ``cdb_sandwich_norm`` launch each.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .huginn import BLOCK_NORM_NAMES, STAGES, HuginnShape, huginn_rope_tables
from .kv_cache import LoopedKvLayout
from .runner import SCRATCH_ITEMS, OuroRunner, _Graph


@dataclass
class PackedHuginnWeights:
    """bf16 device weights per stage and block.

    ``fc`` holds row pairs ``(gate_j, up_j)`` (the stored ``[gate; up]`` interleaved) for
    ``cdb_mlp_gateup_silu_gemm``; ``qk_bias`` is ``[2, H, D]``.
    """

    wte: torch.Tensor
    lm_head: torch.Tensor
    blocks: dict[str, list[dict[str, torch.Tensor | None]]]
    adapter: torch.Tensor
    ln_f: torch.Tensor

    @classmethod
    def from_state_dict(cls, shape: HuginnShape, sd: dict[str, torch.Tensor], device: torch.device) -> PackedHuginnWeights:
        def g(name: str) -> torch.Tensor:
            return sd[name].detach().to(device=device, dtype=torch.bfloat16).contiguous()

        blocks: dict[str, list[dict[str, torch.Tensor | None]]] = {}
        i = shape.intermediate_size
        for stage in STAGES:
            blocks[stage] = []
            for layer in range(shape.stage_layers(stage)):
                p = f"transformer.{stage}.{layer}."
                fc = g(p + "mlp.fc.weight")
                fc = torch.stack([fc[:i], fc[i:]], dim=1).reshape(2 * i, fc.shape[1]).contiguous()
                entry: dict[str, torch.Tensor | None] = {
                    "Wqkv": g(p + "attn.Wqkv.weight"),
                    "proj": g(p + "attn.proj.weight"),
                    "fc": fc,
                    "mlp_proj": g(p + "mlp.proj.weight"),
                    "qk_bias": g(p + "attn.qk_bias").reshape(2, shape.n_heads, shape.head_dim).contiguous()
                    if shape.qk_bias
                    else None,
                }
                for norm in BLOCK_NORM_NAMES:
                    entry[norm] = g(p + norm + ".weight")
                blocks[stage].append(entry)
        wte = g("transformer.wte.weight")
        lm = sd.get("lm_head.weight")
        lm_head = wte if lm is None or lm.data_ptr() == sd["transformer.wte.weight"].data_ptr() else g("lm_head.weight")
        return cls(wte, lm_head, blocks, g("transformer.adapter.weight"), g("transformer.ln_f.weight"))


class HuginnRunner(OuroRunner):
    """Owns the device side of one Huginn engine replica (one GPU)."""

    #: resident slot, position, bank slot, state-source bank slot (-1: zero state, step 0)
    meta_rows = 4

    def __init__(
        self,
        shape: HuginnShape,
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
        layout = LoopedKvLayout(
            num_prelude_layers=shape.n_layers_in_prelude, num_core_layers=shape.n_layers_in_recurrent_block,
            num_coda_layers=shape.n_layers_in_coda, total_recurrent_steps=shape.total_recurrent_steps,
            policy=kv_policy, requested_slots=kv_slots_per_layer,
        )
        self._init_device(
            shape,
            device=device,
            kv_policy=kv_policy,
            kv_slots_per_layer=kv_slots_per_layer,
            layout=layout,
            num_blocks=num_blocks,
            block_size=block_size,
            max_model_len=max_model_len,
            max_num_seqs=max_num_seqs,
            max_num_batched_tokens=max_num_batched_tokens,
            use_cuda_graph=use_cuda_graph,
            fused_lm_head=fused_lm_head,
            max_gemm_n=max(shape.vocab_size, 2 * shape.intermediate_size, 3 * shape.n_embd),
        )
        self.w = PackedHuginnWeights.from_state_dict(shape, state_dict, device)
        E, I = shape.n_embd, shape.intermediate_size
        self.qkv_width = 3 * E
        self.k_col, self.v_col = E, 2 * E
        rows = self.rows
        bf = dict(dtype=torch.bfloat16, device=device)
        self.xw = torch.zeros(rows, E, **bf)
        self.h = torch.zeros(rows, E, **bf)
        self.qkv = torch.zeros(rows, 3 * E, **bf)
        self.attn = torch.zeros(rows, E, **bf)
        self.o = torch.zeros(rows, E, **bf)
        self.act = torch.zeros(rows, I, **bf)
        self.m = torch.zeros(rows, E, **bf)
        self.ad_in = torch.zeros(rows, 2 * E, **bf)  # [state | injection] rows of the adapter GEMM
        self.no_rows = torch.full((rows,), -1, dtype=torch.int32, device=device)  # gather -> zeros
        self.gate_out = torch.zeros(max_num_seqs, **bf)  # latent-difference exit signal
        self.bank_slots = 2 * max_num_seqs + 8
        self.state_bank = torch.zeros(self.bank_slots, E, **bf)
        self.inj_bank = torch.zeros(self.bank_slots, E, **bf)
        self.bank = self.state_bank
        self.logits = torch.zeros(max_num_seqs, shape.vocab_size, **bf)
        self.lm_in = torch.zeros(max_num_seqs, E, **bf)
        self.rope_cos, self.rope_sin = huginn_rope_tables(shape, max_model_len + 1, device)
        self.stage_graphs: dict[tuple[str, int], _Graph] = {}

    # ------------------------------------------------------------------ cache-layer layout
    def coda_cache_layer(self, layer: int) -> int:
        """``LoopedKvLayout.coda_layer_index`` (``kv_cache_policy.py:229-233``)."""

        return self.layout.coda_layer_index(layer)

    # ------------------------------------------------------------------ launch helpers
    def _attention_biased(self, n: int, cache_layer: int, item_slot, item_pos, qk_bias) -> None:
        s, pool = self.shape, self.pool
        _lib.call(
            "cdb_paged_decode_attn_append",
            _lib.ptr(self.qkv), self.qkv.stride(0), self.k_col, self.v_col,
            _lib.ptr(self.attn), self.attn.stride(0),
            _lib.ptr(pool.kv), pool.num_cache_layers, pool.rows, cache_layer,
            _lib.ptr(pool.block_table), pool.block_table.stride(0), _lib.ptr(item_slot), _lib.ptr(item_pos),
            2, _lib.ptr(self.rope_cos), _lib.ptr(self.rope_sin), _lib.ptr(qk_bias), 2,  # fused append
            _lib.ptr(self.plan_hdr), _lib.ptr(self.units), _lib.ptr(self.part_o), _lib.ptr(self.part_ml),
            _lib.ptr(self.counters), SCRATCH_ITEMS, n, s.n_heads, s.head_dim, self.block_size,
            self.scale, self.attn_ctas, _lib.ptr(self.status), self._sp(),
        )

    def _sandwich(self, n, xs, x_rows=None, add=None, w1=None, xd=None, xd_rows=None, w2=None, y=None) -> None:
        s = self.shape
        _lib.call(
            "cdb_sandwich_norm", _lib.ptr(xs), xs.stride(0), _lib.ptr(x_rows), _lib.ptr(add),
            0 if add is None else add.stride(0), _lib.ptr(w1), _lib.ptr(xd), 0 if xd is None else xd.stride(0),
            _lib.ptr(xd_rows), _lib.ptr(w2), _lib.ptr(y), 0 if y is None else y.stride(0), n, s.n_embd, s.norm_eps,
            self._sp(),
        )

    def _gather(self, src, rows, n, dst) -> None:
        _lib.call(
            "cdb_gather_rows", _lib.ptr(src), src.stride(0), _lib.ptr(rows), n, self.shape.n_embd, _lib.ptr(dst),
            dst.stride(0), self._sp(),
        )

    def _mlp(self, n: int, bw) -> None:
        self._gate_up(self.h[:n], bw["fc"], self.act[:n])

    def _blocks(self, stage, n, cache_layer_of, item_slot, item_pos, append, last_xd, last_rows, last_w2) -> None:
        """The blocks of one stage over rows [0, n): x in ``xw``, norm_1(x) in ``h`` on entry.

        The last block writes norm_4's output to ``last_xd`` (rows ``last_rows``) and, when
        ``last_w2`` is given, ``rmsnorm(x; last_w2)`` into ``h``.
        """

        blocks = self.w.blocks[stage]
        for layer, bw in enumerate(blocks):
            cl = cache_layer_of(layer)
            self._mm(self.h[:n], bw["Wqkv"], self.qkv[:n])
            if append:
                self._attention_biased(n, cl, item_slot, item_pos, bw["qk_bias"])
            else:
                s, pool = self.shape, self.pool
                _lib.call(
                    "cdb_rope_append_kv", _lib.ptr(self.qkv), self.qkv.stride(0), self.k_col, self.v_col,
                    _lib.ptr(pool.kv), pool.num_cache_layers, pool.rows, cl, _lib.ptr(pool.block_table),
                    pool.block_table.stride(0), _lib.ptr(item_slot), _lib.ptr(item_pos), 2, _lib.ptr(self.rope_cos),
                    _lib.ptr(self.rope_sin), _lib.ptr(bw["qk_bias"]), n, s.n_heads, s.head_dim, self.block_size,
                    self._sp(),
                )
                self._prefill_attention(cl)
            self._mm(self.attn[:n], bw["proj"], self.o[:n])
            self._sandwich(n, self.xw, add=self.o, w1=bw["norm_2"], xd=self.xw, w2=bw["norm_3"], y=self.h)
            self._mlp(n, bw)
            self._mm(self.act[:n], bw["mlp_proj"], self.m[:n])
            if layer + 1 < len(blocks):
                self._sandwich(
                    n, self.xw, add=self.m, w1=bw["norm_4"], xd=self.xw, w2=blocks[layer + 1]["norm_1"], y=self.h
                )
            else:
                self._sandwich(
                    n, self.xw, add=self.m, w1=bw["norm_4"], xd=last_xd, xd_rows=last_rows, w2=last_w2,
                    y=self.h if last_w2 is not None else None,
                )

    def _first_norm(self, n: int, stage: str) -> None:
        self._sandwich(n, self.xw, w2=self.w.blocks[stage][0]["norm_1"], y=self.h)

    # ------------------------------------------------------------------ recurrent step
    def _recurrent_meta(self, item_slot, item_pos, hidden, steps) -> list[list[int]]:
        if steps is None:
            raise ValueError("the Huginn recurrent launch needs each item's recurrent step")
        return [item_slot, item_pos, hidden, [-1 if st == 0 else h for h, st in zip(hidden, steps, strict=True)]]

    def _recurrent_body(self, meta: torch.Tensor, n: int, kv_slot: int, gate: bool) -> None:
        s = self.shape
        E = s.n_embd
        item_slot, item_pos, hid, ssrc = meta[0], meta[1], meta[2], meta[3]
        self._plan(item_pos, n, 1)
        self._gather(self.state_bank, ssrc, n, self.ad_in[:, :E])
        self._gather(self.inj_bank, hid, n, self.ad_in[:, E:])
        self._mm(self.ad_in[:n], self.w.adapter, self.xw[:n])
        self._first_norm(n, "core_block")
        self._blocks(
            "core_block", n, lambda l: self.core_cache_layer(kv_slot, l), item_slot, item_pos, True,
            self.state_bank, hid, None,
        )
        if gate:
            # new state: state_bank[hid[r]]; old state: row r of ad_in's state half
            _lib.call(
                "cdb_latent_diff", _lib.ptr(self.state_bank), self.state_bank.stride(0), _lib.ptr(self.ad_in),
                self.ad_in.stride(0), _lib.ptr(hid), n, E, _lib.ptr(self.gate_out), self._sp(),
            )

    # ------------------------------------------------------------------ stages
    def _prelude_body(self, meta: torch.Tensor, n: int) -> None:
        """meta rows: token id (-1: the request's device token), request slot, bank slot, position."""

        s = self.shape
        _lib.call(
            "cdb_embed", _lib.ptr(self.w.wte), s.n_embd, s.vocab_size, _lib.ptr(meta[0]), _lib.ptr(meta[1]),
            _lib.ptr(self.token_table), _lib.ptr(self.xw), self.xw.stride(0), None, n, s.embed_scale,
            _lib.ptr(self.status), self._sp(),
        )
        self._plan(meta[3], n, 1)
        self._first_norm(n, "prelude")
        self._blocks("prelude", n, lambda l: l, meta[1], meta[3], True, self.inj_bank, meta[2], None)

    def _coda_body(self, meta: torch.Tensor, n: int, keep_logits: bool = False):
        """meta rows: bank slot, token-log row, request slot, position."""

        self._plan(meta[3], n, 1)
        first = self.w.blocks["coda"][0]["norm_1"]
        self._sandwich(n, self.state_bank, x_rows=meta[0], w1=self.w.ln_f, xd=self.xw, w2=first, y=self.h)
        self._blocks("coda", n, self.coda_cache_layer, meta[2], meta[3], True, self.xw, None, self.w.ln_f)
        return self._lm_head_argmax(self.h, n, self.w.lm_head, meta[1], meta[2], keep_logits)

    #: metadata of a padding row per stage (token id, slot, bank, position / bank, log, slot, position)
    _STAGE_PAD = {"prelude": (0, 0, -1, -1), "coda": (-1, -1, -1, -1)}

    def _stage_meta_host(self, kind: str, bucket: int) -> np.ndarray:
        pad = np.asarray(self._STAGE_PAD[kind], dtype=np.int32)[:, None]
        return np.repeat(pad, bucket, axis=1)

    def _stage_graph(self, kind: str, bucket: int) -> _Graph:
        """The prelude or coda launch at ``bucket`` rows, captured once (padding rows: position -1,
        bank and output rows -1)."""

        key = (kind, bucket)
        g = self.stage_graphs.get(key)
        if g is not None:
            return g
        body = self._prelude_body if kind == "prelude" else self._coda_body
        meta = torch.from_numpy(self._stage_meta_host(kind, bucket)).to(self.device)
        with torch.cuda.stream(self.stream):  # warm up on an all-padding batch
            body(meta, bucket)
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        before = _lib.launch_count
        with torch.cuda.graph(graph, pool=self.graph_pool, stream=self.stream):
            body(meta, bucket)
        captured = _lib.launch_count - before
        self.stats.captured_calls += captured
        if self.graph_pool is None:
            self.graph_pool = graph.pool()
        g = _Graph(graph=graph, meta=meta, launches=captured)
        self.stage_graphs[key] = g
        return g

    def _replay_stage(self, kind: str, rows: list[list[int]]) -> None:
        n = len(rows[0])
        bucket = next(b for b in self.buckets if b >= n)
        g = self._stage_graph(kind, bucket)
        meta_host = self._stage_meta_host(kind, bucket)
        for i, row in enumerate(rows):
            meta_host[i, :n] = row
        self.uploader.upload(meta_host, self.stream, out=g.meta)
        with torch.cuda.stream(self.stream):
            g.graph.replay()
        self.stats.replayed_launches += g.launches

    def _graphable(self, n: int) -> bool:
        return self.use_cuda_graph and n <= self.buckets[-1]

    def prelude(self, token_ids: list[int], req_slots: list[int], hidden: list[int], positions=None) -> None:
        """``run_prelude`` for each item's token at its position; the output goes to ``inj_bank``."""

        if positions is None:
            raise ValueError("the Huginn prelude attends: positions are required")
        n = len(token_ids)
        if n == 0:
            return
        self.flush_block_edits()
        rows = [list(token_ids), list(req_slots), list(hidden), list(positions)]
        if self._graphable(n):
            self._replay_stage("prelude", rows)
            return
        meta = self.upload(rows).view(4, n)
        with torch.cuda.stream(self.stream):
            self._prelude_body(meta, n)

    def coda(
        self, hidden: list[int], log_rows: list[int], req_slots: list[int], keep_logits: bool = False, positions=None
    ):
        """``run_coda`` + LM head + greedy argmax for exited tokens."""

        if positions is None:
            raise ValueError("the Huginn coda attends: positions are required")
        n = len(hidden)
        self.flush_block_edits()
        rows = [list(hidden), list(log_rows), list(req_slots), list(positions)]
        if self._graphable(n) and not (keep_logits or not self.fused_lm_head):
            self._replay_stage("coda", rows)
            return None
        meta = self.upload(rows).view(4, n)
        with torch.cuda.stream(self.stream):
            return self._coda_body(meta, n, keep_logits)

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
        """``HuginnForCausalLM.forward`` at full depth over a varlen batch of prompt chunks."""

        s = self.shape
        E = s.n_embd
        n = len(token_ids)
        self.flush_block_edits()
        meta = self.upload([token_ids, item_slot, item_pos]).view(3, n)
        k = len(logit_rows)
        sel = self.upload([logit_rows, log_rows, req_slots]).view(3, k) if k else None
        with torch.cuda.stream(self.stream):
            _lib.call(
                "cdb_embed", _lib.ptr(self.w.wte), E, s.vocab_size, _lib.ptr(meta[0]), None, None, _lib.ptr(self.xw),
                self.xw.stride(0), None, n, s.embed_scale, _lib.ptr(self.status), self._sp(),
            )
            tiles = self.prefill_tiles(item_slot, item_pos)
            self._tiles = self.upload(tiles)
            self._num_tiles = len(tiles)
            self._first_norm(n, "prelude")
            self._blocks("prelude", n, lambda l: l, meta[1], meta[2], False, self.ad_in[:, E:], None, None)
            self._gather(self.xw, self.no_rows, n, self.ad_in[:, :E])  # state_init="zero"
            for step in range(s.total_recurrent_steps):
                self._mm(self.ad_in[:n], self.w.adapter, self.xw[:n])
                self._first_norm(n, "core_block")
                slot = slot_for_step[step]
                self._blocks(
                    "core_block", n, lambda l, slot=slot: self.core_cache_layer(slot, l), meta[1], meta[2], False,
                    self.ad_in[:, :E], None, None,
                )
            first = self.w.blocks["coda"][0]["norm_1"]
            self._sandwich(n, self.ad_in[:, :E], w1=self.w.ln_f, xd=self.xw, w2=first, y=self.h)
            self._blocks("coda", n, self.coda_cache_layer, meta[1], meta[2], False, self.xw, None, self.w.ln_f)
            if k:
                self._gather(self.h, sel[0], k, self.lm_in)
                return self._lm_head_argmax(self.lm_in, k, self.w.lm_head, sel[1], sel[2], keep_logits)
        return None
