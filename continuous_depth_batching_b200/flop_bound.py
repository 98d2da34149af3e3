"""Per-token FLOP weights of a looped model and the speed-up bound they put on early exit.

Restates the reference's ``looped_cdb/benchmarks/flop_bound.py:39-112``. A token decoded at
recurrent depth ``d`` costs ``F0 + d * Fr``: ``Fr`` is one application of the recurrent core, paid
once per step, and ``F0`` is what every token pays whatever its depth (prelude, coda, final norm
and output head). Against full depth ``r``, a schedule with mean exit depth ``d_bar`` can at best run

    (F0 + r * Fr) / (F0 + d_bar * Fr)

times faster (the paper's eq. (1)). Each stage's cost is dominated by matmuls that touch every
weight once per token, so both terms are counted in parameters, and only their ratio matters. The
token embedding is a lookup and costs nothing. A weight tied between the embedding and the output
head is counted for the head.

The split is read off the model's parameter names, which are the reference's, so the same
function serves the reference's own modules and this package's
(:class:`~continuous_depth_batching_b200.ouro.OuroForCausalLM`,
:class:`~continuous_depth_batching_b200.huginn.HuginnForCausalLM`). It works on models built on
the ``meta`` device, so a full-size model needs no memory.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any

from torch import nn

__all__ = ["StageFlops", "stage_flops", "stage_flops_from_json"]


@dataclass(frozen=True)
class StageFlops:
    """Depth-independent (``f0``) and per-recurrent-step (``fr``) weights, in parameters."""

    f0: int
    fr: int

    def __post_init__(self) -> None:
        if self.fr <= 0:
            raise ValueError(f"fr must be positive, got {self.fr}")
        if self.f0 < 0:
            raise ValueError(f"f0 must be non-negative, got {self.f0}")

    @property
    def f0_over_fr(self) -> float:
        """The depth-independent cost in units of one recurrent step."""

        return self.f0 / self.fr

    def ideal_speedup(self, *, max_depth: int, mean_depth: float) -> float:
        """The FLOP bound on the speed-up of a schedule whose tokens exit at ``mean_depth`` on
        average, against every token at ``max_depth``."""

        if mean_depth <= 0:
            raise ValueError(f"mean_depth must be positive, got {mean_depth}")
        if max_depth <= 0:
            raise ValueError(f"max_depth must be positive, got {max_depth}")
        return (self.f0 + max_depth * self.fr) / (self.f0 + mean_depth * self.fr)

    def to_json_dict(self) -> dict[str, int]:
        return {"f0_params": self.f0, "fr_params": self.fr}


def stage_flops_from_json(payload: dict[str, Any]) -> StageFlops:
    """The weights a run recorded with :meth:`StageFlops.to_json_dict`."""

    return StageFlops(f0=int(payload["f0_params"]), fr=int(payload["fr_params"]))


def _sizes(model: nn.Module) -> dict[str, int]:
    # named_parameters lists a tied tensor once; the module-level walk sees it under every module
    # that applies it, which is how the bound counts it
    sizes: dict[str, int] = {}
    for mod_name, module in model.named_modules():
        for p_name, p in module.named_parameters(recurse=False):
            sizes[f"{mod_name}.{p_name}" if mod_name else p_name] = p.numel()
    return sizes


def stage_flops(model: nn.Module) -> StageFlops:
    """The ``f0`` / ``fr`` split of an Ouro or Huginn model.

    * Huginn: the core is the input-injection adapter plus the recurrent block (the adapter runs
      at the top of every step); the depth-independent stages are the prelude, the coda, the final
      norm and the output head.
    * Ouro: the core is the shared layer stack; the depth-independent weights are the final norm
      and the output head (the exit gate is neither).

    Raises ``TypeError`` for any other structure rather than guessing a split."""

    sizes = _sizes(model)
    names = list(sizes)

    def total(pattern: str) -> int:
        rx = re.compile(pattern)
        return sum(sizes[n] for n in names if rx.match(n))

    if any(n.startswith("transformer.core_block.") for n in names):
        core = total(r"transformer\.(adapter|core_block)\.")
        boundary = total(r"transformer\.(prelude|coda|ln_f)\.") + total(r"lm_head\.")
        return StageFlops(f0=boundary, fr=core)
    config = getattr(model, "config", None)
    if getattr(config, "model_type", None) == "ouro" and any(n.startswith("model.layers.") for n in names):
        layers = int(config.num_hidden_layers)
        core = sum(
            sizes[n] for n in names if (m := re.match(r"model\.layers\.(\d+)\.", n)) and int(m.group(1)) < layers
        )
        boundary = total(r"model\.norm\.") + total(r"lm_head\.")
        return StageFlops(f0=boundary, fr=core)
    raise TypeError(f"cannot derive the prelude-core-coda FLOP weights of {type(model).__name__}")
