"""Huginn model shape, parameter naming and a weight container for the CDB engine.

Huginn (``models/huginn/modeling_huginn.py``) is a looped decoder with a non-recurrent
prelude, a recurrent core applied ``total_recurrent_steps`` times and a non-recurrent coda,
all built from the same sandwich-normed block (``HuginnBlock`` ``:312-338``):

    x = norm_2(attn(norm_1(x)) + x);  x = norm_4(mlp(norm_3(x)) + x)

The attention (``HuginnAttention`` ``:216-287``) projects q|k|v with one ``Wqkv``, adds a
learned per-head ``qk_bias`` to q and k, rotates interleaved pairs in fp32
(``apply_rotary_emb_complex_like`` ``:175-197``) and projects back with ``proj``; the MLP
(``HuginnMLP`` ``:290-301``) is ``proj(silu(gate) * up)`` with ``[gate | up] = fc(x)``. A core
step is ``adapter([state | injection])`` followed by the core blocks (``run_core_step``
``:442-455``); the prelude embeds ``wte(ids) * sqrt(n_embd)`` and runs the prelude blocks; the
coda is ``ln_f``, the coda blocks, ``ln_f`` again, then the LM head tied to ``wte``.

The engine reads a Huginn model through these parameter names only (the reference's own
``HuginnForCausalLM`` works unchanged). :class:`HuginnForCausalLM` here is a parameter container
with that layout for machines without the reference package.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace
from typing import Any

import torch
from torch import nn

BLOCK_NORM_NAMES = ("norm_1", "norm_2", "norm_3", "norm_4")
STAGES = ("prelude", "core_block", "coda")


@dataclass(frozen=True)
class HuginnShape:
    """The architecture numbers the kernels are specialised on (``HuginnConfig`` fields)."""

    vocab_size: int = 65536
    n_embd: int = 5280
    n_heads: int = 55
    intermediate_size: int = 17920
    n_layers_in_prelude: int = 2
    n_layers_in_recurrent_block: int = 4
    n_layers_in_coda: int = 2
    total_recurrent_steps: int = 32
    rope_base: float = 50000.0
    norm_eps: float = 1e-6
    qk_bias: bool = True
    max_position_embeddings: int = 4096

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_heads

    @property
    def hidden_size(self) -> int:
        return self.n_embd

    @property
    def num_attention_heads(self) -> int:
        return self.n_heads

    @property
    def num_key_value_heads(self) -> int:
        return self.n_heads

    @property
    def embed_scale(self) -> float:
        """``HuginnConfig.embed_scale`` (``configuration_huginn.py``): ``sqrt(n_embd)``."""

        return math.sqrt(self.n_embd)

    def stage_layers(self, stage: str) -> int:
        return {
            "prelude": self.n_layers_in_prelude,
            "core_block": self.n_layers_in_recurrent_block,
            "coda": self.n_layers_in_coda,
        }[stage]

    @classmethod
    def from_config(cls, config: Any) -> HuginnShape:
        """Read an HF ``HuginnConfig`` (or any object with the same attribute names)."""

        return cls(
            vocab_size=int(getattr(config, "padded_vocab_size", None) or config.vocab_size),
            n_embd=int(config.n_embd),
            n_heads=int(config.n_heads),
            intermediate_size=int(config.intermediate_size),
            n_layers_in_prelude=int(config.n_layers_in_prelude),
            n_layers_in_recurrent_block=int(config.n_layers_in_recurrent_block),
            n_layers_in_coda=int(config.n_layers_in_coda),
            total_recurrent_steps=int(config.total_recurrent_steps),
            rope_base=float(config.rope_base),
            norm_eps=float(config.norm_eps),
            qk_bias=bool(config.qk_bias),
            max_position_embeddings=int(getattr(config, "block_size", 4096)),
        )

    def to_config(self) -> SimpleNamespace:
        """A config object carrying the HF attribute names (``model_type='huginn'``)."""

        return SimpleNamespace(
            model_type="huginn",
            vocab_size=self.vocab_size,
            padded_vocab_size=self.vocab_size,
            n_embd=self.n_embd,
            n_heads=self.n_heads,
            intermediate_size=self.intermediate_size,
            n_layers_in_prelude=self.n_layers_in_prelude,
            n_layers_in_recurrent_block=self.n_layers_in_recurrent_block,
            n_layers_in_coda=self.n_layers_in_coda,
            total_recurrent_steps=self.total_recurrent_steps,
            mean_recurrence=self.total_recurrent_steps,
            rope_base=self.rope_base,
            norm_eps=self.norm_eps,
            qk_bias=self.qk_bias,
            bias=False,
            state_init="zero",
            block_size=self.max_position_embeddings,
            head_dim=self.head_dim,
            num_attention_heads=self.n_heads,
            num_key_value_heads=self.n_heads,
            hidden_size=self.n_embd,
            _attn_implementation="paged|flash_attention_3",
        )

    def param_count_core_step(self) -> int:
        """Dense parameters one recurrent step multiplies (adapter + core blocks)."""

        e, i = self.n_embd, self.intermediate_size
        block = 3 * e * e + e * e + 2 * i * e + i * e
        return 2 * e * e + self.n_layers_in_recurrent_block * block


def huginn_parameter_shapes(shape: HuginnShape) -> dict[str, tuple[int, ...]]:
    """Every parameter the CDB path reads, by reference state-dict name."""

    e, i, v = shape.n_embd, shape.intermediate_size, shape.vocab_size
    h, d = shape.n_heads, shape.head_dim
    out: dict[str, tuple[int, ...]] = {"transformer.wte.weight": (v, e)}
    for stage in STAGES:
        for layer in range(shape.stage_layers(stage)):
            p = f"transformer.{stage}.{layer}."
            out[p + "attn.Wqkv.weight"] = (3 * e, e)
            if shape.qk_bias:
                out[p + "attn.qk_bias"] = (2, 1, h, d)
            out[p + "attn.proj.weight"] = (e, e)
            out[p + "mlp.fc.weight"] = (2 * i, e)
            out[p + "mlp.proj.weight"] = (e, i)
            for norm in BLOCK_NORM_NAMES:
                out[p + norm + ".weight"] = (e,)
    out["transformer.adapter.weight"] = (e, 2 * e)
    out["transformer.ln_f.weight"] = (e,)
    out["lm_head.weight"] = (v, e)
    return out


def random_huginn_state_dict(
    shape: HuginnShape,
    *,
    seed: int = 0,
    dtype: torch.dtype = torch.float32,
    device: str | torch.device = "cpu",
    std: float = 0.02,
    norm_jitter: float = 0.05,
    qk_bias_std: float = 0.02,
    embed_std: float | None = None,
) -> dict[str, torch.Tensor]:
    """Seeded random-init weights with the reference's parameter names.

    Matrices are ``N(0, std)``, norm gains ``1 + N(0, norm_jitter)``, ``qk_bias``
    ``N(0, qk_bias_std)``. The LM head is tied to the embedding (``tie_embeddings=True``), so
    ``lm_head.weight`` is the same values as ``transformer.wte.weight`` (``embed_std`` widens
    both: a peaked output distribution). Drawn in sorted-name order from one generator.
    """

    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    shapes = huginn_parameter_shapes(shape)
    out: dict[str, torch.Tensor] = {}
    for name in sorted(shapes):
        if name == "lm_head.weight":
            continue
        dims = shapes[name]
        if ".norm_" in name or name == "transformer.ln_f.weight":
            t = 1.0 + norm_jitter * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        elif name.endswith("qk_bias"):
            t = qk_bias_std * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        elif name == "transformer.wte.weight" and embed_std is not None:
            t = embed_std * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        else:
            t = std * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        out[name] = t.to(dtype)
    out["lm_head.weight"] = out["transformer.wte.weight"].clone()
    return out


class _Param(nn.Module):
    def __init__(self, dims: tuple[int, ...]) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(dims), requires_grad=False)


class HuginnForCausalLM(nn.Module):
    """Parameter container with the reference ``HuginnForCausalLM`` state-dict layout."""

    def __init__(self, shape: HuginnShape) -> None:
        super().__init__()
        self.shape = shape
        self.config = shape.to_config()
        shapes = huginn_parameter_shapes(shape)
        tr = nn.Module()
        tr.wte = _Param(shapes["transformer.wte.weight"])
        for stage in STAGES:
            blocks = nn.ModuleList()
            for layer in range(shape.stage_layers(stage)):
                p = f"transformer.{stage}.{layer}."
                block = nn.Module()
                attn = nn.Module()
                attn.Wqkv = _Param(shapes[p + "attn.Wqkv.weight"])
                attn.proj = _Param(shapes[p + "attn.proj.weight"])
                if shape.qk_bias:
                    attn.qk_bias = nn.Parameter(torch.empty(shapes[p + "attn.qk_bias"]), requires_grad=False)
                mlp = nn.Module()
                mlp.fc = _Param(shapes[p + "mlp.fc.weight"])
                mlp.proj = _Param(shapes[p + "mlp.proj.weight"])
                block.attn = attn
                block.mlp = mlp
                for norm in BLOCK_NORM_NAMES:
                    setattr(block, norm, _Param(shapes[p + norm + ".weight"]))
                blocks.append(block)
            setattr(tr, stage, blocks)
        tr.adapter = _Param(shapes["transformer.adapter.weight"])
        tr.ln_f = _Param(shapes["transformer.ln_f.weight"])
        self.transformer = tr
        self.lm_head = _Param(shapes["lm_head.weight"])

    @classmethod
    def random_init(
        cls,
        shape: HuginnShape,
        *,
        seed: int = 0,
        dtype: torch.dtype = torch.bfloat16,
        device: str | torch.device = "cpu",
        **kwargs: Any,
    ) -> HuginnForCausalLM:
        model = cls(shape)
        sd = random_huginn_state_dict(shape, seed=seed, dtype=dtype, device=device, **kwargs)
        model.to(device=device, dtype=dtype)
        model.load_state_dict(sd, strict=True)
        return model


def huginn_rope_tables(shape: HuginnShape, max_positions: int, device: torch.device | str = "cpu"):
    """fp32 cos/sin ``[max_positions, head_dim/2]`` of ``freqs_cis_for_positions``
    (``modeling_huginn.py:143-172``): ``pos.float() * inv_freq`` then cos and sin in fp32."""

    d = shape.head_dim
    inv = 1.0 / (shape.rope_base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    inv = inv.to(device)
    freqs = torch.arange(max_positions, device=device).float().unsqueeze(-1) * inv
    return freqs.cos().contiguous(), freqs.sin().contiguous()
