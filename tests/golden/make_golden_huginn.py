"""Generate the Huginn golden fixtures by running the reference engine itself on CPU.

Run in a container that has the reference checkout (read-only), with ``CDB_REFERENCE_SRC``
pointing at its ``src`` directory::

    CDB_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden_huginn.py [--async]

It builds the reference's own ``HuginnForCausalLM`` at a small shape with Huginn's structure
(prelude / recurrent core / coda, 96-wide heads, ``qk_bias``, interleaved RoPE, tied LM head),
loads seeded weights from :func:`continuous_depth_batching_b200.huginn.random_huginn_state_dict`,
registers the CPU restatement of the paged FlashAttention contract and drives the reference
``ContinuousDepthBatchingEngine.generate_batch`` (``HuginnCDBAdapter``, synchronous mode).
Runs: the live latent-difference exit gate (direct threshold) with refill, then its recorded
exit depths replayed with refill, without refill, and under ``last_exited``.

Outputs ``tests/golden/huginn_small.json`` (tokens, stats, launch traces with block-table rows)
and ``tests/golden/huginn_small_logits.npz`` (the first LM-head calls of the live run).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))
if not os.environ.get("CDB_REFERENCE_SRC"):
    raise SystemExit("set CDB_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, os.environ["CDB_REFERENCE_SRC"])

from make_golden import Recorder, replay_depths  # noqa: E402

from continuous_depth_batching_b200.huginn import HuginnShape, random_huginn_state_dict  # noqa: E402
from oracle.paged_attention import cpu_paged_attention_forward  # noqa: E402
from oracle.workloads import config0_workload  # noqa: E402

SMALL = HuginnShape(
    vocab_size=1024,
    n_embd=480,
    n_heads=5,
    intermediate_size=1280,
    n_layers_in_prelude=1,
    n_layers_in_recurrent_block=2,
    n_layers_in_coda=1,
    total_recurrent_steps=6,
    rope_base=50000.0,
    norm_eps=1e-6,
    qk_bias=True,
    max_position_embeddings=2048,
)
# Relative latent-difference threshold of the live run: a level the random-init states cross
# after a few steps, so the run mixes exit depths.
EXIT_THRESHOLD = 0.4
EMBED_STD = 0.5


def build_reference_model(shape: HuginnShape):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from looped_cdb.models.huginn.configuration_huginn import HuginnConfig
    from looped_cdb.models.huginn.modeling_huginn import HuginnForCausalLM

    ALL_ATTENTION_FUNCTIONS["paged|flash_attention_3"] = cpu_paged_attention_forward
    config = HuginnConfig(
        n_embd=shape.n_embd,
        n_heads=shape.n_heads,
        n_layers=shape.n_layers_in_prelude + shape.n_layers_in_recurrent_block + shape.n_layers_in_coda,
        n_layers_in_prelude=shape.n_layers_in_prelude,
        n_layers_in_recurrent_block=shape.n_layers_in_recurrent_block,
        n_layers_in_coda=shape.n_layers_in_coda,
        mean_recurrence=shape.total_recurrent_steps,
        block_size=shape.max_position_embeddings,
        vocab_size=shape.vocab_size,
        intermediate_size=shape.intermediate_size,
        norm_eps=shape.norm_eps,
        rope_base=shape.rope_base,
        qk_bias=shape.qk_bias,
        bos_token_id=None,
        eos_token_id=None,
        pad_token_id=None,
    )
    torch.manual_seed(0)
    model = HuginnForCausalLM(config)
    model.config._attn_implementation = "paged|flash_attention_3"
    state = random_huginn_state_dict(shape, seed=0, embed_std=EMBED_STD)
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected, unexpected
    assert not missing, missing
    assert torch.equal(model.lm_head.weight, model.transformer["wte"].weight)
    model.eval()
    return model


def run_case(
    name: str, *, kv_policy: str, refill: bool, live_gate: bool, exit_depths=None, num_blocks=4096, async_mode=False
):
    from looped_cdb.continuous_depth_batching import ContinuousDepthBatchingConfig, ContinuousDepthBatchingEngine

    model = build_reference_model(SMALL)
    prompts, max_new = config0_workload()
    cfg = ContinuousDepthBatchingConfig(
        block_size=16,
        num_blocks=num_blocks,
        max_recurrent_steps=SMALL.total_recurrent_steps,
        exit_threshold=EXIT_THRESHOLD if live_gate else None,
        synthetic_exit_replay=not live_gate,
        use_async_batching=async_mode,
        use_cuda_graph=False,
        use_cuda_graph_prefill=False,
        refill=refill,
        kv_policy=kv_policy,
        kv_pressure_mode="reserve" if kv_policy == "last_exited" else "recompute",
        max_model_len=2048,
    )
    engine = ContinuousDepthBatchingEngine.from_model(model, cfg)
    rec = Recorder(engine)
    with torch.no_grad():
        outs = engine.generate_batch(
            prompts, max_new_tokens=max_new, eos_token_id=None, warmup=False, exit_depths=exit_depths
        )
    stats = engine.last_stats
    result = {
        "name": name,
        "kv_policy": kv_policy,
        "refill": refill,
        "live_gate": live_gate,
        "async": async_mode,
        "tokens": [o.generated_tokens for o in outs],
        "exit_depths": exit_depths,
        "stats": {
            "prefill_batches": stats.prefill_batches,
            "recurrent_batches": stats.recurrent_batches,
            "coda_batches": stats.coda_batches,
            "recurrent_steps": stats.recurrent_steps,
            "coda_tokens": stats.coda_tokens,
            "generated_tokens": stats.generated_tokens,
            "scheduler_refills": stats.scheduler_refills,
            "exit_depth_histogram": {str(k): v for k, v in sorted(stats.exit_depth_histogram.items())},
            "recompute_preemptions": getattr(engine.offloading_manager, "num_recompute_preemptions", 0),
        },
        "launches": rec.launches,
    }
    return result, rec.logits


def main() -> None:
    """``python tests/golden/make_golden_huginn.py [--async]`` (``--async``: the reference's default
    delayed-gate timing, plus a live-gate no-refill run, into ``huginn_small_async.*``)."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    async_mode = "--async" in sys.argv[1:]
    sfx = "_async" if async_mode else ""
    runs = []
    logits_out: dict[str, np.ndarray] = {}
    live, live_logits = run_case(
        "live_gate_refill" + sfx, kv_policy="single", refill=True, live_gate=True, async_mode=async_mode
    )
    runs.append(live)
    depths = replay_depths(live, async_mode)
    for name, policy, refill in (
        ("replay_refill", "single", True),
        ("replay_norefill", "single", False),
        ("replay_last_exited", "last_exited", True),
    ):
        res, _ = run_case(
            name + sfx, kv_policy=policy, refill=refill, live_gate=False, exit_depths=depths, async_mode=async_mode
        )
        runs.append(res)
    if async_mode:
        live_nr, _ = run_case("live_gate_norefill" + sfx, kv_policy="single", refill=False, live_gate=True,
                              async_mode=True)
        runs.append(live_nr)
    for i, arr in enumerate(live_logits[:6]):
        logits_out[f"live_gate_refill{sfx}_{i}"] = arr.astype(np.float32)
    prompts, max_new = config0_workload()
    shape = dict(SMALL.__dict__)
    payload = {
        "generator": "tests/golden/make_golden_huginn.py",
        "shape": shape,
        "embed_std": EMBED_STD,
        "exit_threshold": EXIT_THRESHOLD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "num_blocks": 4096,
        "runs": runs,
    }
    (HERE / f"huginn_small{sfx}.json").write_text(json.dumps(payload, separators=(",", ":")))
    np.savez_compressed(HERE / f"huginn_small{sfx}_logits.npz", **logits_out)
    print("wrote", HERE / f"huginn_small{sfx}.json", "runs:", [r["name"] for r in runs])
    for r in runs:
        print(r["name"], r["stats"])


def pressure_main() -> None:
    """``--pressure``: the synchronous replay (refill on) in a 40-block pool, where stalled decoders
    are soft-reset and re-prefilled through the prelude, core and coda cache layers, into
    ``huginn_small_pressure.json``."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gold = json.loads((HERE / "huginn_small.json").read_text())
    depths = next(r for r in gold["runs"] if r["name"] == "replay_refill")["exit_depths"]
    res, _ = run_case("replay_refill_blocks40", kv_policy="single", refill=True, live_gate=False,
                      exit_depths=depths, num_blocks=40)
    res["num_blocks"] = 40
    prompts, max_new = config0_workload()
    payload = {"generator": "tests/golden/make_golden_huginn.py --pressure", "shape": SMALL.__dict__,
               "embed_std": EMBED_STD, "weights_seed": 0, "prompts": prompts, "max_new_tokens": max_new,
               "block_size": 16, "runs": [res]}
    (HERE / "huginn_small_pressure.json").write_text(json.dumps(payload, separators=(",", ":")))
    print(res["name"], res["stats"])


if __name__ == "__main__":
    if "--pressure" in sys.argv[1:]:
        pressure_main()
        raise SystemExit(0)
    main()
