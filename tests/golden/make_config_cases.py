"""Record how the reference's ContinuousDepthBatchingConfig validates a set of settings.

Run in a container that has the reference checkout (read-only), with ``CDB_REFERENCE_SRC``
pointing at its ``src`` directory::

    CDB_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_config_cases.py

For each case (keyword arguments on top of ``max_recurrent_steps=4``) it calls the reference's
``get_resolved`` against an Ouro model config (paged FlashAttention-3, full attention) and records
either the resolved ``kv_slots_per_layer`` or the exception type and message. Then it builds the
reference's ``ExitPolicy`` for the Ouro (cumulative hazard) and Huginn (direct threshold) exit
specs with the case's threshold, and records whether that accepts it. Output:
``tests/golden/config_cases.json``; ``tests/test_config.py`` checks this package against it.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
if not os.environ.get("CDB_REFERENCE_SRC"):
    raise SystemExit("set CDB_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, os.environ["CDB_REFERENCE_SRC"])

CASES: list[dict] = [
    {},
    {"block_size": 0},
    {"num_blocks": 0},
    {"num_blocks": 64, "mem_fraction_static": 0.5},
    {"mem_fraction_static": 1.5},
    {"mem_fraction_static": 0.0},
    {"mem_fraction_static": 0.7},
    {"max_num_batched_tokens": 0},
    {"max_model_len": 0},
    {"max_recurrent_steps": None},
    {"max_recurrent_steps": 1},
    {"max_num_seqs": 0},
    {"min_free_slots": 0},
    {"min_coda_batch_size": 0},
    {"min_coda_batch_size": 300},
    {"min_coda_batch_size": 256},
    {"replay_eos_finishes": True, "use_async_batching": False},
    {"replay_eos_finishes": True},
    {"safety_margin": 1.0},
    {"safety_margin": -0.1},
    {"kv_policy": "per_step"},
    {"kv_policy": "last_exited"},
    {"kv_policy": "last_exited", "kv_pressure_mode": "reserve"},
    {"kv_policy": "depth_indexed"},
    {"kv_policy": "first_then_shared"},
    {"kv_policy": "first_then_shared", "kv_slots_per_layer": 3},
    {"kv_policy": "first_then_shared", "kv_slots_per_layer": 5},
    {"kv_policy": "first_then_shared", "kv_slots_per_layer": 0},
    {"kv_policy": "single", "kv_slots_per_layer": 2},
    {"min_recurrent_steps": 0},
    {"min_recurrent_steps": 5},
    {"kv_pressure_mode": "bogus"},
    {"kv_pressure_mode": "offload"},
    {"kv_pressure_mode": "offload", "cpu_offload_space": 4.0},
    {"cpu_offload_space": 4.0},
    {"cpu_offload_space": -1.0},
    {"exit_threshold": 0.5, "synthetic_exit_replay": True},
    {"exit_threshold": 0.5},
    {"exit_threshold": 1.5},
    {"exit_threshold": 0.0},
    {"exit_threshold": -0.5},
    {"exit_threshold": float("inf")},
    {"exit_threshold": 0.5, "kv_policy": "depth_indexed"},
    {"exit_threshold": 0.5, "kv_policy": "first_then_shared", "min_recurrent_steps": 2},
    {"exit_threshold": 0.5, "kv_policy": "last_exited", "kv_pressure_mode": "reserve"},
    {"synthetic_exit_replay": True, "refill": False},
]


def _model_config():
    from looped_cdb.models.ouro.configuration_ouro import OuroConfig

    cfg = OuroConfig(
        vocab_size=1024, hidden_size=256, intermediate_size=704, num_hidden_layers=4, num_attention_heads=4,
        num_key_value_heads=4, max_position_embeddings=2048, total_ut_steps=4,
        layer_types=["full_attention"] * 4, pad_token_id=None,
    )
    cfg._attn_implementation = "paged|flash_attention_3"
    return cfg


def _exit_policy(spec_name: str, cfg) -> str:
    """'ok' or 'ExceptionType: message' for building the reference ExitPolicy of an exit spec."""

    from looped_cdb.continuous_depth_batching import exit_policy as ep

    spec = ep.ExitPolicySpec(getattr(ep.ExitDecisionRule, spec_name))
    try:
        ep.ExitPolicy(
            spec=spec, threshold=cfg.exit_threshold, min_recurrent_steps=cfg.min_recurrent_steps,
            max_recurrent_steps=cfg.max_recurrent_steps, delay_gate_consumption=cfg.delay_gate_consumption,
            use_async_batching=cfg.use_async_batching, synthetic_exit_replay=cfg.synthetic_exit_replay,
        )
    except Exception as e:  # noqa: BLE001 - the outcome is what is recorded
        return f"{type(e).__name__}: {e}"
    return "ok"


def main() -> None:
    from looped_cdb.continuous_depth_batching import ContinuousDepthBatchingConfig

    model_cfg = _model_config()
    out = []
    for case in CASES:
        kw = {"max_recurrent_steps": 4, **case}
        rec: dict = {"kwargs": kw}
        try:
            resolved = ContinuousDepthBatchingConfig(**kw).get_resolved(model_cfg)
        except Exception as e:  # noqa: BLE001
            rec["error"] = {"type": type(e).__name__, "message": str(e)}
        else:
            rec["kv_slots_per_layer"] = resolved.kv_slots_per_layer
            rec["exit_policy"] = {
                "ouro": _exit_policy("CUMULATIVE_HAZARD", resolved),
                "huginn": _exit_policy("DIRECT_THRESHOLD", resolved),
            }
        out.append(rec)
    (HERE / "config_cases.json").write_text(json.dumps({"generator": "tests/golden/make_config_cases.py",
                                                        "cases": out}, indent=1))
    print("wrote", len(out), "cases")


if __name__ == "__main__":
    main()
