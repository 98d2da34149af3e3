"""Ouro model shape, parameter naming and a weight container for the CDB engine.

The engine consumes an Ouro causal LM through its parameters only, keyed by the names the
reference's HF module uses (``models/ouro/modeling_ouro.py``: ``OuroForCausalLM`` ``:764-775``,
``OuroModel`` ``:634-652``, ``OuroDecoderLayer`` ``:456-468``, ``OuroAttention`` ``:359-375``,
``OuroMLP`` ``:156-164``). So the reference's own ``OuroForCausalLM`` (or any module with that
state-dict layout) can be handed to :meth:`ContinuousDepthBatchingEngine.from_model` unchanged.

:class:`OuroForCausalLM` here is a parameter container with that layout for machines where the
reference package is not installed (the GPU box); it has no forward of its own, because every
stage of the CDB decode step runs through the CUDA library.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace
from typing import Any

import torch
from torch import nn

LAYER_NORM_NAMES = ("input_layernorm", "input_layernorm_2", "post_attention_layernorm", "post_attention_layernorm_2")
ATTN_PROJ_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj")
MLP_PROJ_NAMES = ("gate_proj", "up_proj", "down_proj")


@dataclass(frozen=True)
class OuroShape:
    """The architecture numbers the kernels are specialised on."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-6
    max_position_embeddings: int = 32768
    total_ut_steps: int = 4

    @classmethod
    def from_config(cls, config: Any) -> OuroShape:
        """Read an HF ``OuroConfig`` (or any object with the same attribute names)."""

        heads = int(config.num_attention_heads)
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // heads
        rope = getattr(config, "rope_parameters", None)
        theta = None
        if isinstance(rope, dict):
            theta = rope.get("rope_theta")
        if theta is None:
            theta = getattr(config, "rope_theta", 10000.0)
        kv_heads = getattr(config, "num_key_value_heads", None) or heads
        return cls(
            vocab_size=int(config.vocab_size),
            hidden_size=int(config.hidden_size),
            intermediate_size=int(config.intermediate_size),
            num_hidden_layers=int(config.num_hidden_layers),
            num_attention_heads=heads,
            num_key_value_heads=int(kv_heads),
            head_dim=int(head_dim),
            rope_theta=float(theta),
            rms_norm_eps=float(getattr(config, "rms_norm_eps", 1e-6)),
            max_position_embeddings=int(getattr(config, "max_position_embeddings", 32768)),
            total_ut_steps=int(getattr(config, "total_ut_steps", 4) or 4),
        )

    def to_config(self) -> SimpleNamespace:
        """A config object carrying the HF attribute names (``model_type='ouro'``)."""

        return SimpleNamespace(
            model_type="ouro",
            vocab_size=self.vocab_size,
            hidden_size=self.hidden_size,
            intermediate_size=self.intermediate_size,
            num_hidden_layers=self.num_hidden_layers,
            num_attention_heads=self.num_attention_heads,
            num_key_value_heads=self.num_key_value_heads,
            head_dim=self.head_dim,
            rope_theta=self.rope_theta,
            rope_parameters={"rope_type": "default", "rope_theta": self.rope_theta},
            rms_norm_eps=self.rms_norm_eps,
            max_position_embeddings=self.max_position_embeddings,
            total_ut_steps=self.total_ut_steps,
            hidden_act="silu",
            _attn_implementation="paged|flash_attention_3",
        )

    def param_count_recurrent(self) -> int:
        """Dense parameters one recurrent step multiplies (all shared layers + exit gate)."""

        h, i = self.hidden_size, self.intermediate_size
        qkv = h * (self.num_attention_heads + 2 * self.num_key_value_heads) * self.head_dim
        o = self.num_attention_heads * self.head_dim * h
        return self.num_hidden_layers * (qkv + o + 3 * h * i) + h


def ouro_parameter_shapes(shape: OuroShape) -> dict[str, tuple[int, ...]]:
    """Every parameter the CDB decode path reads, by reference state-dict name."""

    h, i, v = shape.hidden_size, shape.intermediate_size, shape.vocab_size
    qd = shape.num_attention_heads * shape.head_dim
    kd = shape.num_key_value_heads * shape.head_dim
    out: dict[str, tuple[int, ...]] = {"model.embed_tokens.weight": (v, h)}
    for layer in range(shape.num_hidden_layers):
        p = f"model.layers.{layer}."
        out[p + "self_attn.q_proj.weight"] = (qd, h)
        out[p + "self_attn.k_proj.weight"] = (kd, h)
        out[p + "self_attn.v_proj.weight"] = (kd, h)
        out[p + "self_attn.o_proj.weight"] = (h, qd)
        out[p + "mlp.gate_proj.weight"] = (i, h)
        out[p + "mlp.up_proj.weight"] = (i, h)
        out[p + "mlp.down_proj.weight"] = (h, i)
        for norm in LAYER_NORM_NAMES:
            out[p + norm + ".weight"] = (h,)
    out["model.norm.weight"] = (h,)
    out["model.early_exit_gate.weight"] = (1, h)
    out["model.early_exit_gate.bias"] = (1,)
    out["lm_head.weight"] = (v, h)
    return out


def random_ouro_state_dict(
    shape: OuroShape,
    *,
    seed: int = 0,
    dtype: torch.dtype = torch.float32,
    device: str | torch.device = "cpu",
    std: float = 0.02,
    norm_jitter: float = 0.05,
    gate_std: float | None = None,
    lm_head_std: float | None = None,
) -> dict[str, torch.Tensor]:
    """Seeded random-init weights with the reference's parameter names.

    Matrices are ``N(0, std)`` (the HF ``initializer_range`` default); RMSNorm gains are
    ``1 + N(0, norm_jitter)`` so the gain multiply is exercised; the exit-gate bias is zero.
    ``lm_head_std`` widens the LM head alone (a peaked output distribution, as a trained model
    has, so greedy tokens are not decided by margins below bf16 resolution).
    Tensors are drawn in sorted-name order from one generator on ``device`` so the same seed
    gives the same weights on every machine with the same torch build and device type.
    """

    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    gate_std = std if gate_std is None else gate_std
    for name in sorted(ouro_parameter_shapes(shape)):
        dims = ouro_parameter_shapes(shape)[name]
        if name.endswith("layernorm.weight") or name.endswith("layernorm_2.weight") or name == "model.norm.weight":
            t = 1.0 + norm_jitter * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        elif name == "model.early_exit_gate.bias":
            t = torch.zeros(dims, device=device, dtype=torch.float32)
        elif name == "model.early_exit_gate.weight":
            t = gate_std * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        elif name == "lm_head.weight" and lm_head_std is not None:
            t = lm_head_std * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        else:
            t = std * torch.randn(dims, generator=gen, device=device, dtype=torch.float32)
        out[name] = t.to(dtype)
    return out


class _Param(nn.Module):
    def __init__(self, dims: tuple[int, ...], bias: tuple[int, ...] | None = None) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(dims), requires_grad=False)
        if bias is not None:
            self.bias = nn.Parameter(torch.empty(bias), requires_grad=False)


class OuroForCausalLM(nn.Module):
    """Parameter container with the reference ``OuroForCausalLM`` state-dict layout.

    ``config`` carries the HF attribute names the engine reads. Build one with
    :meth:`random_init` for synthetic benchmarking, or ``load_state_dict`` real weights.
    """

    def __init__(self, shape: OuroShape) -> None:
        super().__init__()
        self.shape = shape
        self.config = shape.to_config()
        shapes = ouro_parameter_shapes(shape)
        model = nn.Module()
        model.embed_tokens = _Param(shapes["model.embed_tokens.weight"])
        layers = nn.ModuleList()
        for layer in range(shape.num_hidden_layers):
            p = f"model.layers.{layer}."
            block = nn.Module()
            attn = nn.Module()
            for proj in ATTN_PROJ_NAMES:
                setattr(attn, proj, _Param(shapes[p + f"self_attn.{proj}.weight"]))
            mlp = nn.Module()
            for proj in MLP_PROJ_NAMES:
                setattr(mlp, proj, _Param(shapes[p + f"mlp.{proj}.weight"]))
            block.self_attn = attn
            block.mlp = mlp
            for norm in LAYER_NORM_NAMES:
                setattr(block, norm, _Param(shapes[p + norm + ".weight"]))
            layers.append(block)
        model.layers = layers
        model.norm = _Param(shapes["model.norm.weight"])
        model.early_exit_gate = _Param((1, shape.hidden_size), (1,))
        self.model = model
        self.lm_head = _Param(shapes["lm_head.weight"])

    @classmethod
    def random_init(
        cls,
        shape: OuroShape,
        *,
        seed: int = 0,
        dtype: torch.dtype = torch.bfloat16,
        device: str | torch.device = "cpu",
        **kwargs: Any,
    ) -> OuroForCausalLM:
        model = cls(shape)
        sd = random_ouro_state_dict(shape, seed=seed, dtype=dtype, device=device, **kwargs)
        model.to(device=device, dtype=dtype)
        model.load_state_dict(sd, strict=True)
        return model

    def get_decoder(self) -> nn.Module:
        return self.model


def rope_inv_freq(shape: OuroShape) -> torch.Tensor:
    """``1 / theta^(2j/D)`` in fp32, as ``OuroRotaryEmbedding.compute_default_rope_parameters``
    (``modeling_ouro.py:528-549``) builds it."""

    d = shape.head_dim
    exps = torch.arange(0, d, 2, dtype=torch.int64).to(dtype=torch.float32) / d
    return 1.0 / (shape.rope_theta**exps)


def flops_per_recurrent_token(shape: OuroShape) -> float:
    """Dense GEMM FLOPs one token-step of the recurrent stage costs (2 per weight)."""

    return 2.0 * shape.param_count_recurrent()

