"""CPU restatement of the Huginn stage math on the CDB decode and prefill paths.

TEST INFRASTRUCTURE ONLY: this is the checker the CUDA path is compared against. Only
``tests/``, ``__graft_entry__.smoke()``, the golden generator and ``bench.py``'s CPU
baseline use it.

Each op follows ``models/huginn/modeling_huginn.py`` in order and dtype, so run in bf16 it
rounds where the reference's bf16 PyTorch path rounds:

* ``HuginnRMSNorm.forward`` ``:132-146``: fp32 ``x * rsqrt(mean(x^2) + eps)``, cast back, times
  the weight in the model dtype (the same rounding as Ouro's norm).
* ``freqs_cis_for_positions`` ``:143-172``: ``pos.float() * inv_freq`` -> fp32 cos/sin.
* ``HuginnAttention.forward`` ``:240-287``: ``Wqkv`` split into q|k|v, ``q + q_bias`` and
  ``k + k_bias`` in the model dtype, interleaved-pair rotation in fp32
  (``apply_rotary_emb_complex_like`` ``:175-197``) cast back, paged attention, ``proj``.
* ``HuginnMLP.forward`` ``:298-301``: ``proj(silu(gate) * up)``, ``[gate | up] = fc(x)``.
* ``HuginnBlock.forward`` ``:333-336``: ``x = norm_2(attn(norm_1 x) + x)``,
  ``x = norm_4(mlp(norm_3 x) + x)``.
* ``run_prelude`` ``:424-435`` (``wte(ids) * sqrt(n_embd)`` then the prelude blocks),
  ``run_core_step`` ``:437-452`` (``adapter(cat([state, injection]))`` then the core blocks),
  ``run_coda`` ``:454-460`` (``ln_f``, coda blocks, ``ln_f``), LM head tied to ``wte``.
* ``HuginnCDBAdapter`` ``continuous_depth_batching/adapters/huginn.py:105-189``: the engine's
  hidden vector is ``[state | injection]``; the prelude returns ``[zeros | injection]``
  (``state_init="zero"``); a recurrent step rewrites the state half; the exit signal is
  ``latent_diff(next, prev)`` (``models/huginn/exit_gates.py:33-40``) in the model dtype.
* Cache layers follow ``LoopedKvLayout`` (``kv_cache_policy.py:132-233``): prelude layers
  first, then core layers slot-major, then coda layers.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from continuous_depth_batching_b200.huginn import BLOCK_NORM_NAMES, STAGES, HuginnShape

from .ouro_math import OracleKVCache, _softmax_attend, rms_norm


def huginn_cos_sin(shape: HuginnShape, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin ``[T, D/2]`` for integer positions (``freqs_cis_for_positions``)."""

    d = shape.head_dim
    inv = 1.0 / (shape.rope_base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    freqs = positions.float().unsqueeze(-1) * inv
    return freqs.cos(), freqs.sin()


def rotate_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x ``[T, H, D]`` rotated on (even, odd) pairs in fp32, cast back to x's dtype."""

    x2 = x.unflatten(-1, (-1, 2)).float()
    c = cos[:, None, :]
    s = sin[:, None, :]
    out = torch.stack([x2[..., 0] * c - x2[..., 1] * s, x2[..., 1] * c + x2[..., 0] * s], dim=-1).flatten(2)
    return out.type_as(x)


def latent_diff(state: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    """``||s - s_prev|| / max(||s||, 1e-9)`` per row, in the state dtype."""

    return ((state - prev).norm(dim=-1) / state.norm(dim=-1).clamp_min(1e-9)).to(state.dtype)


@dataclass
class HuginnWeights:
    """The reference state dict regrouped per stage and block, in the compute dtype."""

    shape: HuginnShape
    dtype: torch.dtype
    wte: torch.Tensor
    blocks: dict[str, list[dict[str, torch.Tensor]]]
    adapter: torch.Tensor
    ln_f: torch.Tensor
    lm_head: torch.Tensor

    @classmethod
    def from_state_dict(cls, shape: HuginnShape, sd: dict[str, torch.Tensor], dtype: torch.dtype) -> HuginnWeights:
        g = {k: v.detach().to("cpu", dtype) for k, v in sd.items()}
        blocks: dict[str, list[dict[str, torch.Tensor]]] = {}
        for stage in STAGES:
            blocks[stage] = []
            for layer in range(shape.stage_layers(stage)):
                p = f"transformer.{stage}.{layer}."
                entry = {
                    "Wqkv": g[p + "attn.Wqkv.weight"],
                    "proj": g[p + "attn.proj.weight"],
                    "fc": g[p + "mlp.fc.weight"],
                    "mlp_proj": g[p + "mlp.proj.weight"],
                }
                if shape.qk_bias:
                    entry["qk_bias"] = g[p + "attn.qk_bias"]
                for norm in BLOCK_NORM_NAMES:
                    entry[norm] = g[p + norm + ".weight"]
                blocks[stage].append(entry)
        lm = g.get("lm_head.weight", g["transformer.wte.weight"])
        return cls(shape, dtype, g["transformer.wte.weight"], blocks, g["transformer.adapter.weight"], g["transformer.ln_f.weight"], lm)


class HuginnOracle:
    """Staged Huginn math over an :class:`OracleKVCache` with the ``LoopedKvLayout`` layer order."""

    def __init__(self, weights: HuginnWeights, cache: OracleKVCache, core_slots: int) -> None:
        self.w = weights
        self.shape = weights.shape
        self.cache = cache
        self.core_slots = core_slots
        self.scale = self.shape.head_dim**-0.5

    # -- layout (LoopedKvLayout.prelude/core/coda_layer_index) -------------------------
    def cache_layer(self, stage: str, layer: int, slot: int = 0) -> int:
        s = self.shape
        if stage == "prelude":
            return layer
        if stage == "core_block":
            return s.n_layers_in_prelude + slot * s.n_layers_in_recurrent_block + layer
        return s.n_layers_in_prelude + self.core_slots * s.n_layers_in_recurrent_block + layer

    # -- attention contracts --------------------------------------------------------------
    def _decode_attend(self, layer: int, positions: list[int], block_rows: list[list[int]]):
        kc, vc = self.cache.k[layer], self.cache.v[layer]

        def attend(q, k, v):
            out = torch.zeros(q.shape, dtype=torch.float32)
            for b, p in enumerate(positions):
                row = self.cache.rows_for(block_rows[b], p, p + 1)
                kc[row] = k[b : b + 1]
                vc[row] = v[b : b + 1]
                rows = self.cache.rows_for(block_rows[b], 0, p + 1)
                out[b : b + 1] = _softmax_attend(q[b : b + 1], kc[rows], vc[rows], self.scale, p)
            return out

        return attend

    def _prefill_attend(self, layer: int, spans, chunks):
        kc, vc = self.cache.k[layer], self.cache.v[layer]

        def attend(q, k, v):
            out = torch.zeros(q.shape, dtype=torch.float32)
            for (a, b, past), (_t, _p, blocks) in zip(spans, chunks, strict=True):
                wrows = self.cache.rows_for(blocks, past, past + (b - a))
                kc[wrows] = k[a:b]
                vc[wrows] = v[a:b]
                rrows = self.cache.rows_for(blocks, 0, past + (b - a))
                out[a:b] = _softmax_attend(q[a:b], kc[rrows], vc[rrows], self.scale, past)
            return out

        return attend

    # -- one sandwich block over T rows ------------------------------------------------------
    def _block(self, x: torch.Tensor, bw: dict[str, torch.Tensor], cos, sin, attend) -> torch.Tensor:
        s = self.shape
        eps = s.norm_eps
        t = x.shape[0]
        e, h, d = s.n_embd, s.n_heads, s.head_dim
        qkv = F.linear(rms_norm(x, bw["norm_1"], eps), bw["Wqkv"])
        q, k, v = qkv.split([e, e, e], dim=-1)
        q = q.view(t, h, d)
        k = k.view(t, h, d)
        v = v.view(t, h, d)
        if s.qk_bias:
            q_bias, k_bias = bw["qk_bias"].split(1, dim=0)
            q = (q + q_bias[0]).to(q.dtype)
            k = (k + k_bias[0]).to(q.dtype)
        q = rotate_interleaved(q, cos, sin)
        k = rotate_interleaved(k, cos, sin)
        attn = attend(q, k, v).to(x.dtype).reshape(t, -1)
        x = rms_norm(F.linear(attn, bw["proj"]) + x, bw["norm_2"], eps)
        gate, up = F.linear(rms_norm(x, bw["norm_3"], eps), bw["fc"]).chunk(2, dim=-1)
        m = F.linear(F.silu(gate) * up, bw["mlp_proj"])
        return rms_norm(m + x, bw["norm_4"], eps)

    def _stage(self, stage: str, x, cos, sin, attend_for_layer) -> torch.Tensor:
        for layer, bw in enumerate(self.w.blocks[stage]):
            x = self._block(x, bw, cos, sin, attend_for_layer(layer))
        return x

    # -- stages on the decode path (one token per row, mixed positions) --------------------
    def embed(self, token_ids: list[int]) -> torch.Tensor:
        return self.w.wte[torch.tensor(token_ids, dtype=torch.long)] * self.shape.embed_scale

    def prelude(self, token_ids: list[int], positions: list[int], block_rows: list[list[int]]) -> torch.Tensor:
        """Packed ``[zeros | injection]`` rows; writes the prelude cache layers at each position."""

        cos, sin = huginn_cos_sin(self.shape, torch.tensor(positions, dtype=torch.long))
        x = self.embed(token_ids)
        inj = self._stage(
            "prelude", x, cos, sin, lambda l: self._decode_attend(self.cache_layer("prelude", l), positions, block_rows)
        )
        return torch.cat([torch.zeros_like(inj), inj], dim=-1)

    def recurrent_step(
        self, packed: torch.Tensor, positions: list[int], block_rows: list[list[int]], kv_slot: int
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """One core step on packed rows; returns the new packed rows and the latent-diff signal."""

        e = self.shape.n_embd
        state, inj = packed[:, :e], packed[:, e:]
        cos, sin = huginn_cos_sin(self.shape, torch.tensor(positions, dtype=torch.long))
        x = F.linear(torch.cat([state, inj], dim=-1), self.w.adapter)
        nxt = self._stage(
            "core_block",
            x,
            cos,
            sin,
            lambda l: self._decode_attend(self.cache_layer("core_block", l, kv_slot), positions, block_rows),
        )
        return torch.cat([nxt, inj], dim=-1), latent_diff(nxt, state)

    def coda(self, packed: torch.Tensor, positions: list[int], block_rows: list[list[int]]) -> torch.Tensor:
        """Final hidden rows (``ln_f``, coda blocks, ``ln_f``) of the state half."""

        s = self.shape
        cos, sin = huginn_cos_sin(s, torch.tensor(positions, dtype=torch.long))
        x = rms_norm(packed[:, : s.n_embd], self.w.ln_f, s.norm_eps)
        x = self._stage("coda", x, cos, sin, lambda l: self._decode_attend(self.cache_layer("coda", l), positions, block_rows))
        return rms_norm(x, self.w.ln_f, s.norm_eps)

    def lm_head(self, hidden: torch.Tensor) -> torch.Tensor:
        return F.linear(hidden, self.w.lm_head)

    # -- monolithic full-depth prefill over prompt chunks (HuginnForCausalLM.forward) ----------
    def prefill(self, chunks: list[tuple[list[int], int, list[int]]], slot_for_step: list[int]) -> torch.Tensor:
        """``forward`` at full depth over a varlen batch; final hidden rows ``[T, E]``."""

        s = self.shape
        ids: list[int] = []
        pos: list[int] = []
        spans = []
        for tokens, past, _blocks in chunks:
            spans.append((len(ids), len(ids) + len(tokens), past))
            ids.extend(tokens)
            pos.extend(range(past, past + len(tokens)))
        cos, sin = huginn_cos_sin(s, torch.tensor(pos, dtype=torch.long))
        inj = self._stage(
            "prelude", self.embed(ids), cos, sin, lambda l: self._prefill_attend(self.cache_layer("prelude", l), spans, chunks)
        )
        state = torch.zeros_like(inj)
        for step in range(s.total_recurrent_steps):
            x = F.linear(torch.cat([state, inj], dim=-1), self.w.adapter)
            slot = slot_for_step[step]
            state = self._stage(
                "core_block",
                x,
                cos,
                sin,
                lambda l, slot=slot: self._prefill_attend(self.cache_layer("core_block", l, slot), spans, chunks),
            )
        x = rms_norm(state, self.w.ln_f, s.norm_eps)
        x = self._stage("coda", x, cos, sin, lambda l: self._prefill_attend(self.cache_layer("coda", l), spans, chunks))
        return rms_norm(x, self.w.ln_f, s.norm_eps)

    def copy_rows(self, src_layer: int, dst_layers: list[int], rows: torch.Tensor) -> None:
        ks, vs = self.cache.k[src_layer][rows], self.cache.v[src_layer][rows]
        for dst in dst_layers:
            self.cache.k[dst][rows] = ks
            self.cache.v[dst][rows] = vs
