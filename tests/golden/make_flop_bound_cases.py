"""Record the reference's per-stage FLOP weights (``benchmarks/flop_bound.py``) for four models.

Run with ``CDB_REFERENCE_SRC`` pointing at the reference checkout's ``src`` directory::

    CDB_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_flop_bound_cases.py

It builds the reference's own ``OuroForCausalLM`` and ``HuginnForCausalLM`` on the ``meta``
device (no weights are allocated) at BASELINE config 0's shape, the Ouro-1.4B shape, the small
Huginn test shape and the Huginn-0125 shape, and records ``stage_flops(model)`` of each, with the
shape, into ``tests/golden/flop_bound_cases.json``; ``tests/test_flop_bound.py`` checks this
package's restatement on its own models of the same shapes against it.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
if not os.environ.get("CDB_REFERENCE_SRC"):
    raise SystemExit("set CDB_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, os.environ["CDB_REFERENCE_SRC"])

from continuous_depth_batching_b200.huginn import HuginnShape  # noqa: E402
from continuous_depth_batching_b200.ouro import OuroShape  # noqa: E402

OURO = {
    "ouro_cfg0": OuroShape(vocab_size=1024, hidden_size=256, intermediate_size=704, num_hidden_layers=4,
                           num_attention_heads=4, num_key_value_heads=4, head_dim=64, rope_theta=10000.0,
                           rms_norm_eps=1e-6, max_position_embeddings=2048, total_ut_steps=4),
    "ouro_1p4b": OuroShape(vocab_size=49152, hidden_size=2048, intermediate_size=5632, num_hidden_layers=24,
                           num_attention_heads=16, num_key_value_heads=16, head_dim=128, rope_theta=10000.0,
                           rms_norm_eps=1e-6, max_position_embeddings=4096, total_ut_steps=4),
}
HUGINN = {
    "huginn_small": HuginnShape(vocab_size=1024, n_embd=480, n_heads=5, intermediate_size=1280, n_layers_in_prelude=1,
                                n_layers_in_recurrent_block=2, n_layers_in_coda=1, total_recurrent_steps=6,
                                rope_base=50000.0, norm_eps=1e-6, qk_bias=True, max_position_embeddings=2048),
    "huginn_0125": HuginnShape(vocab_size=65536, n_embd=5280, n_heads=55, intermediate_size=17920,
                               n_layers_in_prelude=2, n_layers_in_recurrent_block=4, n_layers_in_coda=2,
                               total_recurrent_steps=32, rope_base=50000.0, norm_eps=1e-6, qk_bias=True,
                               max_position_embeddings=4096),
}


def main() -> None:
    from looped_cdb.benchmarks.flop_bound import stage_flops
    from looped_cdb.models.huginn.configuration_huginn import HuginnConfig
    from looped_cdb.models.huginn.modeling_huginn import HuginnForCausalLM
    from looped_cdb.models.ouro.configuration_ouro import OuroConfig
    from looped_cdb.models.ouro.modeling_ouro import OuroForCausalLM

    cases = []
    for name, s in OURO.items():
        cfg = OuroConfig(
            vocab_size=s.vocab_size, hidden_size=s.hidden_size, intermediate_size=s.intermediate_size,
            num_hidden_layers=s.num_hidden_layers, num_attention_heads=s.num_attention_heads,
            num_key_value_heads=s.num_key_value_heads, max_position_embeddings=s.max_position_embeddings,
            rope_theta=s.rope_theta, rms_norm_eps=s.rms_norm_eps, total_ut_steps=s.total_ut_steps,
            layer_types=["full_attention"] * s.num_hidden_layers, pad_token_id=None,
        )
        with torch.device("meta"):
            model = OuroForCausalLM(cfg)
        f = stage_flops(model)
        cases.append({"name": name, "family": "ouro", "shape": s.__dict__, "f0": f.f0, "fr": f.fr})
    for name, s in HUGINN.items():
        cfg = HuginnConfig(
            n_embd=s.n_embd, n_heads=s.n_heads,
            n_layers=s.n_layers_in_prelude + s.n_layers_in_recurrent_block + s.n_layers_in_coda,
            n_layers_in_prelude=s.n_layers_in_prelude, n_layers_in_recurrent_block=s.n_layers_in_recurrent_block,
            n_layers_in_coda=s.n_layers_in_coda, mean_recurrence=s.total_recurrent_steps,
            block_size=s.max_position_embeddings, vocab_size=s.vocab_size, intermediate_size=s.intermediate_size,
            norm_eps=s.norm_eps, rope_base=s.rope_base, qk_bias=s.qk_bias, bos_token_id=None, eos_token_id=None,
            pad_token_id=None,
        )
        with torch.device("meta"):
            model = HuginnForCausalLM(cfg)
        f = stage_flops(model)
        cases.append({"name": name, "family": "huginn", "shape": s.__dict__, "f0": f.f0, "fr": f.fr})
    for c in cases:
        print(c["name"], c["f0"], c["fr"])
    (HERE / "flop_bound_cases.json").write_text(
        json.dumps({"generator": "tests/golden/make_flop_bound_cases.py", "cases": cases}, indent=1)
    )


if __name__ == "__main__":
    main()
