"""CPU restatement of the Ouro layer math on the CDB decode and prefill paths.

TEST INFRASTRUCTURE ONLY: this is the checker the CUDA path is compared against. Only
``tests/``, ``__graft_entry__.smoke()``, the golden generator and ``bench.py``'s CPU
baseline use it.

Every op follows the reference's order and rounding points so that, run in bf16, it rounds
where the reference's bf16 PyTorch path rounds:

* ``OuroRMSNorm.forward`` ``models/ouro/modeling_ouro.py:445-450``: upcast to fp32,
  ``x * rsqrt(mean(x^2) + eps)``, cast back, then ``weight * x`` in the model dtype.
* rotary ``:172-204`` and ``OuroRotaryEmbedding.forward`` ``:560-573``: cos/sin computed in
  fp32 from ``inv_freq x position`` and cast to the model dtype, ``q*cos + rotate_half(q)*sin``.
* ``OuroDecoderLayer.forward`` ``:470-503`` (sandwich norms):
  ``x += in_norm2(o_proj(attn(rope(qkv(in_norm(x))))))``;
  ``x += post_norm2(down(silu(gate(h)) * up(h)))`` with ``h = post_norm(x)``.
* ``OuroModel._run_recurrent_step`` ``:670-690`` / ``OuroCDBAdapter.recurrent_step``
  ``adapters/ouro.py:214-264``: all shared layers then the final ``norm``; the exit gate
  ``Linear(H,1)`` reads the normed state.
* ``OuroModel.forward`` ``:698-712``: prefill runs every recurrent step over the prompt chunk,
  each step writing its KV slot (``kv_cache_policy.kv_layer_index``).
* LM head ``adapters/ouro.py:321-329`` + greedy ``argmax`` (first index on ties).

The paged KV cache is one ``[(num_blocks+2)*block_size, Hkv, D]`` K and V tensor per cache
layer (``continuous_batching/cache.py:131-145``); a token row is ``block*bs + offset``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from continuous_depth_batching_b200.ouro import LAYER_NORM_NAMES, OuroShape


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dtype = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return weight * (xf * torch.rsqrt(var + eps)).to(dtype)


def rotary_cos_sin(shape: OuroShape, positions: torch.Tensor, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin ``[T, D]`` for integer positions, fp32 math then cast (``modeling_ouro.py:560-573``)."""

    d = shape.head_dim
    inv = 1.0 / (shape.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64).to(torch.float32) / d))
    freqs = positions.to(torch.float32)[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x ``[T, heads, D]``; cos/sin ``[T, D]``."""

    return x * cos[:, None, :] + rotate_half(x) * sin[:, None, :]


@dataclass
class OuroWeights:
    """The reference state dict regrouped per layer, in the compute dtype."""

    shape: OuroShape
    dtype: torch.dtype
    embed: torch.Tensor
    layers: list[dict[str, torch.Tensor]]
    norm: torch.Tensor
    gate_w: torch.Tensor
    gate_b: torch.Tensor
    lm_head: torch.Tensor

    @classmethod
    def from_state_dict(cls, shape: OuroShape, sd: dict[str, torch.Tensor], dtype: torch.dtype) -> OuroWeights:
        g = {k: v.detach().to("cpu", dtype) for k, v in sd.items()}
        layers = []
        for layer in range(shape.num_hidden_layers):
            p = f"model.layers.{layer}."
            entry = {
                "q": g[p + "self_attn.q_proj.weight"],
                "k": g[p + "self_attn.k_proj.weight"],
                "v": g[p + "self_attn.v_proj.weight"],
                "o": g[p + "self_attn.o_proj.weight"],
                "gate": g[p + "mlp.gate_proj.weight"],
                "up": g[p + "mlp.up_proj.weight"],
                "down": g[p + "mlp.down_proj.weight"],
            }
            for norm in LAYER_NORM_NAMES:
                entry[norm] = g[p + norm + ".weight"]
            layers.append(entry)
        return cls(
            shape=shape,
            dtype=dtype,
            embed=g["model.embed_tokens.weight"],
            layers=layers,
            norm=g["model.norm.weight"],
            gate_w=g["model.early_exit_gate.weight"],
            gate_b=g["model.early_exit_gate.bias"],
            lm_head=g["lm_head.weight"],
        )


class OracleKVCache:
    """Per-cache-layer K/V rows ``[(num_blocks+2)*bs, Hkv, D]`` (two spare blocks, as the reference)."""

    def __init__(self, shape: OuroShape, num_cache_layers: int, num_blocks: int, block_size: int, dtype: torch.dtype):
        rows = (num_blocks + 2) * block_size
        self.block_size = block_size
        self.k = [torch.zeros(rows, shape.num_key_value_heads, shape.head_dim, dtype=dtype) for _ in range(num_cache_layers)]
        self.v = [torch.zeros(rows, shape.num_key_value_heads, shape.head_dim, dtype=dtype) for _ in range(num_cache_layers)]

    def rows_for(self, blocks: list[int], start: int, stop: int) -> torch.Tensor:
        bs = self.block_size
        return torch.tensor([blocks[p // bs] * bs + p % bs for p in range(start, stop)], dtype=torch.long)


def _softmax_attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, offset: int) -> torch.Tensor:
    """q [Lq,H,D], k/v [Lk,Hkv,D], query i sees keys <= i+offset. fp32 out [Lq,H,D]."""

    h, hkv = q.shape[1], k.shape[1]
    if hkv != h:
        k = k.repeat_interleave(h // hkv, dim=1)
        v = v.repeat_interleave(h // hkv, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * scale
    lq, lk = q.shape[0], k.shape[0]
    mask = torch.arange(lk)[None, :] > (torch.arange(lq)[:, None] + offset)
    s = s.masked_fill(mask[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v.float())


class OuroOracle:
    """Staged Ouro math (prefill, recurrent step, LM head) over an :class:`OracleKVCache`."""

    def __init__(self, weights: OuroWeights, cache: OracleKVCache) -> None:
        self.w = weights
        self.shape = weights.shape
        self.cache = cache
        self.scale = self.shape.head_dim**-0.5

    # -- one shared decoder layer over T rows -------------------------------------------
    def _layer(self, x: torch.Tensor, lw: dict[str, torch.Tensor], cos, sin, attend) -> torch.Tensor:
        s = self.shape
        eps = s.rms_norm_eps
        t = x.shape[0]
        residual = x
        h = rms_norm(x, lw["input_layernorm"], eps)
        q = F.linear(h, lw["q"]).view(t, s.num_attention_heads, s.head_dim)
        k = F.linear(h, lw["k"]).view(t, s.num_key_value_heads, s.head_dim)
        v = F.linear(h, lw["v"]).view(t, s.num_key_value_heads, s.head_dim)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        attn = attend(q, k, v).to(x.dtype).reshape(t, -1)
        h = rms_norm(F.linear(attn, lw["o"]), lw["input_layernorm_2"], eps)
        x = residual + h
        residual = x
        h = rms_norm(x, lw["post_attention_layernorm"], eps)
        m = F.linear(F.silu(F.linear(h, lw["gate"])) * F.linear(h, lw["up"]), lw["down"])
        return residual + rms_norm(m, lw["post_attention_layernorm_2"], eps)

    # -- prelude --------------------------------------------------------------------------
    def embed(self, token_ids: list[int]) -> torch.Tensor:
        return self.w.embed[torch.tensor(token_ids, dtype=torch.long)]

    # -- recurrent step (decode): one token per row, mixed positions ---------------------
    def recurrent_step(
        self,
        hidden: torch.Tensor,
        positions: list[int],
        block_rows: list[list[int]],
        cache_layer_base: int,
        with_gate: bool = True,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        """``hidden [B, H]``; each row writes KV at its position then attends over ``0..pos``.

        ``cache_layer_base`` is ``kv_slot * num_hidden_layers`` (``kv_cache_policy.py:106-128``).
        Returns the final-normed state and the exit-gate logits ``[B]``.
        """

        s = self.shape
        pos_t = torch.tensor(positions, dtype=torch.long)
        cos, sin = rotary_cos_sin(s, pos_t, self.w.dtype)
        x = hidden
        for layer, lw in enumerate(self.w.layers):
            kc = self.cache.k[cache_layer_base + layer]
            vc = self.cache.v[cache_layer_base + layer]

            def attend(q, k, v, kc=kc, vc=vc):
                out = torch.zeros(q.shape, dtype=torch.float32)
                for b, p in enumerate(positions):
                    row = self.cache.rows_for(block_rows[b], p, p + 1)
                    kc[row] = k[b : b + 1]
                    vc[row] = v[b : b + 1]
                    rows = self.cache.rows_for(block_rows[b], 0, p + 1)
                    out[b : b + 1] = _softmax_attend(q[b : b + 1], kc[rows], vc[rows], self.scale, p)
                return out

            x = self._layer(x, lw, cos, sin, attend)
        x = rms_norm(x, self.w.norm, s.rms_norm_eps)
        gate = (F.linear(x, self.w.gate_w, self.w.gate_b)[:, 0]) if with_gate else None
        return x, gate

    # -- monolithic full-depth prefill over prompt chunks --------------------------------
    def prefill(
        self,
        chunks: list[tuple[list[int], int, list[int]]],
        slot_for_step: list[int],
    ) -> torch.Tensor:
        """Run every recurrent step over a varlen batch of prompt chunks.

        ``chunks``: ``(token_ids, past_length, block_ids)`` per request. Returns the final
        hidden state of every query row ``[T, H]`` (rows in chunk order).
        """

        s = self.shape
        ids: list[int] = []
        pos: list[int] = []
        spans = []
        for tokens, past, _blocks in chunks:
            spans.append((len(ids), len(ids) + len(tokens), past))
            ids.extend(tokens)
            pos.extend(range(past, past + len(tokens)))
        cos, sin = rotary_cos_sin(s, torch.tensor(pos, dtype=torch.long), self.w.dtype)
        x = self.embed(ids)
        for step in range(s.total_ut_steps):
            base = slot_for_step[step] * s.num_hidden_layers
            for layer, lw in enumerate(self.w.layers):
                kc = self.cache.k[base + layer]
                vc = self.cache.v[base + layer]

                def attend(q, k, v, kc=kc, vc=vc):
                    out = torch.zeros(q.shape, dtype=torch.float32)
                    for (a, b, past), (_t, _p, blocks) in zip(spans, chunks, strict=True):
                        wrows = self.cache.rows_for(blocks, past, past + (b - a))
                        kc[wrows] = k[a:b]
                        vc[wrows] = v[a:b]
                        rrows = self.cache.rows_for(blocks, 0, past + (b - a))
                        out[a:b] = _softmax_attend(q[a:b], kc[rrows], vc[rrows], self.scale, past)
                    return out

                x = self._layer(x, lw, cos, sin, attend)
            x = rms_norm(x, self.w.norm, s.rms_norm_eps)
        return x

    # -- coda -------------------------------------------------------------------------------
    def lm_head(self, hidden: torch.Tensor) -> torch.Tensor:
        return F.linear(hidden, self.w.lm_head)

    def copy_rows(self, src_layer: int, dst_layers: list[int], rows: torch.Tensor) -> None:
        """``PagedAttentionCache.copy_kv_rows`` (``continuous_depth_batching/cache.py:105-113``)."""

        ks, vs = self.cache.k[src_layer][rows], self.cache.v[src_layer][rows]
        for dst in dst_layers:
            self.cache.k[dst][rows] = ks
            self.cache.v[dst][rows] = vs
