"""``ContinuousDepthBatchingConfig``: the reference's config surface, validated the same way.

Field names, defaults and validation messages follow
``looped_cdb/continuous_depth_batching/config.py:52-246`` so existing call sites construct it
unchanged. Fields that only tune the reference's PyTorch/FlashAttention runtime
(``use_cuda_graph_prefill``, ``mem_fraction_static``) are accepted; ``use_async_batching`` and
``delay_gate_consumption`` select the same decision timing as the reference (the B200 engine's
host runs ahead of the device in every mode, so they change *when* a decision is applied, exactly
as in the reference, never how work is overlapped).
"""

from __future__ import annotations

import math
from copy import deepcopy
from dataclasses import dataclass

from .kv_cache import KV_CACHE_POLICIES, copies_exit_kv, resolve_kv_slots_per_layer

DEFAULT_MAX_NUM_SEQS = 256
KV_PRESSURE_MODES = ("none", "reserve", "recompute", "offload")


@dataclass
class ContinuousDepthBatchingConfig:
    """Configuration for continuous depth batching (mirror of the reference dataclass)."""

    block_size: int = 16
    num_blocks: int | None = None
    mem_fraction_static: float | None = None
    max_num_batched_tokens: int = 8192
    safety_margin: float = 0.2
    replay_eos_finishes: bool = False
    max_model_len: int = 16384
    use_async_batching: bool = True
    use_cuda_graph: bool = True
    use_cuda_graph_prefill: bool = True
    max_recurrent_steps: int | None = None
    exit_threshold: float | None = None
    synthetic_exit_replay: bool = False
    min_recurrent_steps: int = 1
    delay_gate_consumption: bool = True
    min_coda_batch_size: int = 1
    max_num_seqs: int = DEFAULT_MAX_NUM_SEQS
    min_free_slots: int | None = None
    refill: bool = True
    kv_policy: str = "single"
    kv_slots_per_layer: int | None = None
    kv_pressure_mode: str = "recompute"
    cpu_offload_space: float | None = None

    def decode_block_table_width(self) -> int:
        return -(-self.max_model_len // self.block_size)

    def get_resolved(self) -> ContinuousDepthBatchingConfig:
        """Deep-copied, validated, resolved config (``config.py:124-134``: validate, derive the
        KV slot count, validate the resolved values)."""

        cfg = deepcopy(self)
        cfg.validate()
        assert cfg.max_recurrent_steps is not None
        cfg.kv_slots_per_layer = resolve_kv_slots_per_layer(
            cfg.kv_policy, total_recurrent_steps=cfg.max_recurrent_steps, requested_slots=cfg.kv_slots_per_layer
        )
        cfg.validate_resolved()
        return cfg

    def validate(self) -> None:
        """The reference's checks in its order (``config.py:136-210``) and one of this library's:
        the paged-attention kernels are built for 16-token blocks."""

        if self.block_size <= 0:
            raise ValueError(f"block_size must be positive, but got {self.block_size}")
        if self.block_size != 16:
            raise NotImplementedError("the B200 paged-attention kernels are built for block_size=16")
        if self.num_blocks is not None and self.num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, but got {self.num_blocks}")
        m = self.mem_fraction_static
        if m is not None and (not math.isfinite(m) or not 0 < m < 1):
            raise ValueError(f"mem_fraction_static must be finite and in (0, 1), but got {m}")
        if self.num_blocks is not None and self.mem_fraction_static is not None:
            raise ValueError("Set either num_blocks or mem_fraction_static, not both")
        if self.max_num_batched_tokens <= 0:
            raise ValueError(f"max_num_batched_tokens must be positive, but got {self.max_num_batched_tokens}")
        if self.max_model_len <= 0:
            raise ValueError(f"max_model_len must be positive, but got {self.max_model_len}")
        if self.max_recurrent_steps is None:
            raise ValueError("max_recurrent_steps must be explicitly set for CDB")
        if self.max_recurrent_steps <= 1:
            raise ValueError(f"max_recurrent_steps must be greater than 1, but got {self.max_recurrent_steps}")
        if self.max_num_seqs <= 0:
            raise ValueError(f"max_num_seqs must be positive, but got {self.max_num_seqs}")
        if self.min_free_slots is not None and self.min_free_slots <= 0:
            raise ValueError(f"min_free_slots must be positive, but got {self.min_free_slots}")
        if self.min_coda_batch_size <= 0:
            raise ValueError(f"min_coda_batch_size must be positive, but got {self.min_coda_batch_size}")
        if self.min_coda_batch_size > self.max_num_seqs:
            raise ValueError(
                f"min_coda_batch_size must not exceed max_num_seqs, but got "
                f"{self.min_coda_batch_size} > {self.max_num_seqs}"
            )
        if self.replay_eos_finishes and not self.use_async_batching:
            raise ValueError("replay_eos_finishes requires use_async_batching")
        if not (0 <= self.safety_margin < 1):
            raise ValueError(f"safety_margin must be in [0, 1), but got {self.safety_margin}")
        if self.kv_policy not in KV_CACHE_POLICIES:
            raise ValueError(f"Unsupported kv_policy={self.kv_policy!r}; expected one of {KV_CACHE_POLICIES}")
        if copies_exit_kv(self.kv_policy) and self.kv_pressure_mode == "recompute":
            raise ValueError(
                "kv_policy='last_exited' cannot run with kv_pressure_mode='recompute': recompute-preemption "
                "re-prefills the whole sequence at full depth, replacing previously exited tokens' "
                "exit-step KV with full-depth KV. Use 'reserve', 'offload', or 'none', which preserve KV."
            )
        if self.min_recurrent_steps <= 0:
            raise ValueError(f"min_recurrent_steps must be positive, but got {self.min_recurrent_steps}")
        # validate_kv_pressure_config (utils.py:35-54)
        if self.kv_pressure_mode not in KV_PRESSURE_MODES:
            raise ValueError(f"kv_pressure_mode must be one of {KV_PRESSURE_MODES}, but got {self.kv_pressure_mode!r}")
        if self.cpu_offload_space is not None and self.cpu_offload_space < 0:
            raise ValueError(f"cpu_offload_space must be non-negative when set, but got {self.cpu_offload_space}")
        if self.kv_pressure_mode == "offload":
            if not self.cpu_offload_space:
                raise ValueError(
                    "kv_pressure_mode='offload' requires cpu_offload_space > 0 (the pinned CPU pool size)"
                )
        elif self.cpu_offload_space:
            raise ValueError(
                "cpu_offload_space is only used by kv_pressure_mode='offload', but "
                f"kv_pressure_mode={self.kv_pressure_mode!r} was set with cpu_offload_space={self.cpu_offload_space}"
            )
        if self.exit_threshold is not None and self.synthetic_exit_replay:
            raise ValueError("Only one CDB exit policy can be active")

    def validate_resolved(self) -> None:
        assert self.max_recurrent_steps is not None and self.kv_slots_per_layer is not None
        if self.min_recurrent_steps > self.max_recurrent_steps:
            raise ValueError(
                f"min_recurrent_steps={self.min_recurrent_steps} exceeds max_recurrent_steps={self.max_recurrent_steps}"
            )
        if (
            not copies_exit_kv(self.kv_policy)
            and self.exit_threshold is not None
            and self.min_recurrent_steps < self.kv_slots_per_layer
        ):
            raise ValueError(
                "kv_slots_per_layer must be <= min_recurrent_steps for gated early exit, "
                f"got kv_slots_per_layer={self.kv_slots_per_layer}, min_recurrent_steps={self.min_recurrent_steps}"
            )


def validate_exit_threshold(threshold: float | None, rule: str) -> None:
    """``ExitPolicy.__post_init__`` (``exit_policy.py:62-73``): the threshold is read on the
    adapter's signal scale, a probability for Ouro's cumulative hazard (``rule="hazard"``), a
    nonnegative score for Huginn's latent-difference direct threshold (``rule="direct"``)."""

    if threshold is None:
        return
    if not math.isfinite(threshold):
        raise ValueError("exit_threshold must be finite")
    if rule == "direct":
        if threshold < 0:
            raise ValueError("exit_threshold must be nonnegative for direct-threshold policies")
    elif not 0 < threshold <= 1:
        raise ValueError("exit_threshold must be in (0, 1] for probability policies")
