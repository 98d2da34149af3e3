"""The reference's plugin seam (``CDBModelAdapter``, ``continuous_depth_batching/model_adapter.py:14-122``)
as this engine resolves it.

The reference engine drives a model through an adapter's staged methods (``prelude``,
``recurrent_step``, ``lm_head``) and asks it for its exit-policy spec and KV layout. This engine
runs those stages itself, on device-resident state and CUDA graphs of the library's kernels, for
the two model families the reference ships adapters for. ``resolve_cdb_model_adapter`` therefore
accepts:

* no adapter: the family is inferred from the model, as the reference infers it
  (``OuroCDBAdapter.supports`` / ``HuginnCDBAdapter.supports``);
* the reference's own ``OuroCDBAdapter`` / ``HuginnCDBAdapter`` (or subclasses) wrapping the model
  - their family is taken from the adapter;
* this module's :class:`OuroB200Adapter` / :class:`HuginnB200Adapter`.

Anything else is a custom adapter whose stages are arbitrary Python; it cannot run inside this
engine's device-resident launches, so it is rejected with ``TypeError`` (the reference's own
error type for an unusable adapter, ``model_adapter.py:108-110``). Such a model can still use this
library's attention through the reference engine: ``hf_attention.register()`` installs the paged
decode/prefill kernels under the reference's attention key.
"""

from __future__ import annotations

from dataclasses import dataclass

from .kv_cache import LoopedKvLayout

#: exit rules as the reference names them (``exit_policy.py``: ExitDecisionRule)
CUMULATIVE_HAZARD = "cumulative_hazard"
DIRECT_THRESHOLD = "direct_threshold"


@dataclass(frozen=True)
class ExitPolicySpec:
    """What a recurrent step's exit signal means (``exit_policy.py:ExitPolicySpec``): the rule and
    the step whose hidden state it scores (``same_step``)."""

    rule: str
    decision_horizon: str = "same_step"


class B200ModelAdapter:
    """A model family this engine runs natively, with the reference adapter's queries."""

    family = ""
    stages_use_attention = False

    def __init__(self, model) -> None:
        self.model = model
        self.max_recurrent_steps: int | None = None
        self.exit_signal = True
        self.kv_policy: str | None = None
        self.kv_slots_per_layer: int | None = None

    @classmethod
    def supports(cls, model) -> bool:
        return getattr(getattr(model, "config", None), "model_type", None) == cls.family

    def configure_recurrent_steps(self, max_recurrent_steps: int) -> None:
        self.max_recurrent_steps = int(max_recurrent_steps)

    def configure_exit_signal(self, enabled: bool) -> None:
        self.exit_signal = bool(enabled)

    def configure_kv_policy(self, policy: str, slots_per_layer: int | None = None) -> None:
        self.kv_policy = policy
        self.kv_slots_per_layer = slots_per_layer

    def exit_policy_spec(self) -> ExitPolicySpec:
        raise NotImplementedError

    def decides_exit_before_loop(self) -> bool:
        return False

    def preloop_exit_pdf(self, hidden_states):
        del hidden_states
        return None

    def kv_cache_layout(self) -> LoopedKvLayout:
        raise NotImplementedError


class OuroB200Adapter(B200ModelAdapter):
    """Ouro: a shared-block loop; prelude = embedding lookup, coda = final norm + LM head, exit
    signal = the trained gate's hazard logit (``adapters/ouro.py:116-329``)."""

    family = "ouro"
    stages_use_attention = False

    def exit_policy_spec(self) -> ExitPolicySpec:
        return ExitPolicySpec(CUMULATIVE_HAZARD)

    def kv_cache_layout(self) -> LoopedKvLayout:
        cfg = self.model.config
        steps = self.max_recurrent_steps or int(cfg.total_ut_steps)
        return LoopedKvLayout(
            num_prelude_layers=0, num_core_layers=int(cfg.num_hidden_layers), num_coda_layers=0,
            total_recurrent_steps=steps, policy=self.kv_policy or "single", requested_slots=self.kv_slots_per_layer,
        )


class HuginnB200Adapter(B200ModelAdapter):
    """Huginn: prelude / recurrent core / coda transformer blocks with their own KV; exit signal =
    the relative latent difference, exiting below the threshold (``adapters/huginn.py:41-189``)."""

    family = "huginn"
    stages_use_attention = True

    def exit_policy_spec(self) -> ExitPolicySpec:
        return ExitPolicySpec(DIRECT_THRESHOLD)

    def kv_cache_layout(self) -> LoopedKvLayout:
        cfg = self.model.config
        steps = self.max_recurrent_steps or int(cfg.mean_recurrence)
        return LoopedKvLayout(
            num_prelude_layers=int(cfg.n_layers_in_prelude), num_core_layers=int(cfg.n_layers_in_recurrent_block),
            num_coda_layers=int(cfg.n_layers_in_coda), total_recurrent_steps=steps, policy=self.kv_policy or "single",
            requested_slots=self.kv_slots_per_layer,
        )


_REFERENCE_ADAPTERS = {"OuroCDBAdapter": OuroB200Adapter, "HuginnCDBAdapter": HuginnB200Adapter}


def resolve_cdb_model_adapter(model, adapter=None) -> B200ModelAdapter:
    """The engine's adapter for ``model`` (``resolve_cdb_model_adapter``, ``model_adapter.py:105-122``)."""

    if adapter is None:
        for cls in (OuroB200Adapter, HuginnB200Adapter):
            if cls.supports(model):
                return cls(model)
        raise TypeError(
            f"Continuous depth batching requires an explicit model adapter or a supported looped model; got {type(model)!r}"
        )
    if isinstance(adapter, B200ModelAdapter):
        return adapter
    for klass in type(adapter).__mro__:
        ours = _REFERENCE_ADAPTERS.get(klass.__name__)
        if ours is not None:
            wrapped = getattr(adapter, "model", model)
            if wrapped is not model:
                raise TypeError("model_adapter wraps a different model than the one passed to from_model")
            return ours(model)
    raise TypeError(
        f"the B200 engine runs the Ouro and Huginn stages natively on device-resident state; a custom adapter "
        f"({type(adapter).__name__}) with Python stages cannot run inside its launches. Use the reference engine with "
        f"continuous_depth_batching_b200.hf_attention.register() to run such a model's attention on these kernels."
    )
