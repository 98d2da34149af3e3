"""The plugin seam on the CPU: ``resolve_cdb_model_adapter`` infers the family as the reference
does, accepts the reference's own Ouro/Huginn adapters and this package's, and rejects a custom
adapter with ``TypeError`` (never a bare ``NotImplementedError``)."""

from __future__ import annotations

import pytest

from continuous_depth_batching_b200 import HuginnForCausalLM, OuroForCausalLM, OuroShape
from continuous_depth_batching_b200.huginn import HuginnShape
from continuous_depth_batching_b200.model_adapter import (
    CUMULATIVE_HAZARD,
    DIRECT_THRESHOLD,
    HuginnB200Adapter,
    OuroB200Adapter,
    resolve_cdb_model_adapter,
)

OURO = OuroShape(vocab_size=64, hidden_size=32, intermediate_size=48, num_hidden_layers=3, num_attention_heads=2,
                 num_key_value_heads=2, head_dim=16, total_ut_steps=4, max_position_embeddings=128)


def _huginn():
    return HuginnForCausalLM(HuginnShape(vocab_size=64, n_embd=40, n_heads=2, intermediate_size=48,
                                         n_layers_in_prelude=1, n_layers_in_recurrent_block=2, n_layers_in_coda=1,
                                         total_recurrent_steps=6))


def test_inferred_families_and_specs():
    ouro = resolve_cdb_model_adapter(OuroForCausalLM(OURO))
    assert isinstance(ouro, OuroB200Adapter) and not ouro.stages_use_attention
    assert ouro.exit_policy_spec().rule == CUMULATIVE_HAZARD
    ouro.configure_kv_policy("last_exited")
    layout = ouro.kv_cache_layout()
    assert (layout.num_core_layers, layout.slots_per_layer, layout.num_cache_layers) == (3, 4, 12)
    hug = resolve_cdb_model_adapter(_huginn())
    assert isinstance(hug, HuginnB200Adapter) and hug.stages_use_attention
    assert hug.exit_policy_spec().rule == DIRECT_THRESHOLD
    assert hug.kv_cache_layout().num_cache_layers == 1 + 2 + 1


def test_reference_adapters_are_accepted_by_class():
    model = OuroForCausalLM(OURO)

    class CDBModelAdapter:  # stand-ins with the reference's class names
        pass

    class OuroCDBAdapter(CDBModelAdapter):
        def __init__(self, m):
            self.model = m

    class Tuned(OuroCDBAdapter):
        pass

    assert isinstance(resolve_cdb_model_adapter(model, OuroCDBAdapter(model)), OuroB200Adapter)
    assert isinstance(resolve_cdb_model_adapter(model, Tuned(model)), OuroB200Adapter)
    with pytest.raises(TypeError, match="different model"):
        resolve_cdb_model_adapter(model, OuroCDBAdapter(OuroForCausalLM(OURO)))
    ours = OuroB200Adapter(model)
    assert resolve_cdb_model_adapter(model, ours) is ours


def test_custom_adapter_and_unknown_model_rejected():
    class MyAdapter:
        def recurrent_step(self, *a, **k):
            raise AssertionError

    with pytest.raises(TypeError, match="custom adapter"):
        resolve_cdb_model_adapter(OuroForCausalLM(OURO), MyAdapter())
    with pytest.raises(TypeError, match="supported looped model"):
        resolve_cdb_model_adapter(object())
