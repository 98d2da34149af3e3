"""Pin the CPU oracle against fixtures recorded from the reference engine itself.

``tests/golden/make_golden.py`` ran the reference ``ContinuousDepthBatchingEngine`` (BASELINE
config 0 shape, seeded weights) and recorded every launch, in the synchronous mode
(``ouro_cfg0.json``) and in the reference's default delayed-gate mode (``use_async_batching`` +
``delay_gate_consumption``, ``ouro_cfg0_async.json``). The oracle must
reproduce each run exactly: generated tokens, the ordered launch trace with every item's
(request, position, recurrent step) and block-table row, refill counts, exit histograms, and
(fp32) the LM-head logits.
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from continuous_depth_batching_b200.huginn import HuginnShape, random_huginn_state_dict
from continuous_depth_batching_b200.ouro import OuroShape, random_ouro_state_dict
from oracle.engine import OracleConfig, OracleEngine, exit_depth_histogram

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load_ouro(name: str):
    data = json.loads((GOLDEN / name).read_text())
    shape = OuroShape(**data["shape"])
    sd = random_ouro_state_dict(shape, seed=data["weights_seed"], gate_std=data["gate_std"])
    return data, shape, sd


@pytest.fixture(scope="module")
def golden():
    return _load_ouro("ouro_cfg0.json")


@pytest.fixture(scope="module")
def golden_async():
    return _load_ouro("ouro_cfg0_async.json")


@pytest.fixture(scope="module")
def golden_policies():
    return _load_ouro("ouro_cfg0_policies.json")


def _config(run: dict, data: dict) -> OracleConfig:
    return OracleConfig(
        block_size=data["block_size"],
        num_blocks=data["num_blocks"],
        max_recurrent_steps=4,
        max_model_len=2048,
        exit_threshold=0.5 if run["live_gate"] else None,
        synthetic_exit_replay=not run["live_gate"],
        refill=run["refill"],
        kv_policy=run["kv_policy"],
        kv_pressure_mode="reserve" if run["kv_policy"] == "last_exited" else "recompute",
        delayed=run.get("async", False),
    )


ASYNC_RUNS = [
    "live_gate_refill_async",
    "replay_refill_async",
    "replay_norefill_async",
    "replay_last_exited_async",
    "live_gate_norefill_async",
]


@pytest.mark.parametrize("name", ASYNC_RUNS)
def test_oracle_reproduces_reference_async_run(golden_async, name):
    """Delayed gate consumption: every decision applied one launch late; no-refill waves lead
    with the previous wave's exiters in exit order."""

    data, shape, sd = golden_async
    run = next(r for r in data["runs"] if r["name"] == name)
    engine = OracleEngine(shape, sd, _config(run, data), torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    assert exit_depth_histogram(engine) == run["stats"]["exit_depth_histogram"]
    assert engine.refills == run["stats"]["scheduler_refills"]
    assert engine.stats["recurrent_batches"] == run["stats"]["recurrent_batches"]
    assert engine.stats["coda_batches"] == run["stats"]["coda_batches"]
    if name == "live_gate_refill_async":
        logits = np.load(GOLDEN / "ouro_cfg0_async_logits.npz")
        for i in range(6):
            np.testing.assert_allclose(engine.logits[i][1].numpy(), logits[f"{name}_{i}"], rtol=0, atol=1e-5)


@pytest.mark.parametrize(
    "name", ["replay_first_then_shared", "replay_first_then_shared_async", "replay_depth_indexed_full"]
)
def test_oracle_reproduces_reference_kv_policy_run(golden_policies, name):
    """The other KV layouts: first_then_shared (2 slots, step s -> slot min(s, 1); slot-homogeneous
    recurrent batches) in both timings, and depth_indexed at full depth (4 slots)."""

    data, shape, sd = golden_policies
    run = next(r for r in data["runs"] if r["name"] == name)
    engine = OracleEngine(shape, sd, _config(run, data), torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    assert exit_depth_histogram(engine) == run["stats"]["exit_depth_histogram"]
    assert engine.refills == run["stats"]["scheduler_refills"]


@pytest.mark.parametrize("name", ["replay_refill_eos_stop_async", "replay_norefill_eos_stop_async"])
def test_oracle_early_finish_tokens_in_delayed_timing(name):
    """Early finishes in the delayed timing: the reference stages a successor before it knows the
    token and cancels it once an EOS or stop sequence is consumed; this restatement reads the token
    first and stages none. The generated tokens (the finishing ones included) are the reference's;
    the launches differ from the first such finish on, by the cancelled item or its KV block."""

    data, shape, sd = _load_ouro("ouro_cfg0_finish.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    engine = OracleEngine(shape, sd, _config(run, data), torch.float32)
    tokens = engine.generate(
        data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"], eos_token_ids=run["eos_token_id"],
        stop_sequences=run["stop_sequences"],
    )
    assert tokens == run["tokens"]


@pytest.mark.parametrize("name", ["replay_refill_eos_stop", "replay_norefill_eos_stop"])
def test_oracle_reproduces_reference_early_finish_run(name):
    """Requests finishing on EOS ids (kept in the output) or on stop sequences, refill on and off."""

    data, shape, sd = _load_ouro("ouro_cfg0_finish.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    engine = OracleEngine(shape, sd, _config(run, data), torch.float32)
    tokens = engine.generate(
        data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"], eos_token_ids=run["eos_token_id"],
        stop_sequences=run["stop_sequences"],
    )
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    assert exit_depth_histogram(engine) == run["stats"]["exit_depth_histogram"]


@pytest.mark.parametrize(
    "name,preemptions",
    [
        ("replay_refill_blocks56", 0),
        ("replay_refill_blocks48", 3),
        ("replay_refill_blocks40", 2),
        ("replay_norefill_blocks48", 2),
        ("replay_norefill_blocks40", 1),
        ("replay_refill_reserve_blocks40", 0),
        ("replay_norefill_reserve_blocks40", 0),
        ("replay_refill_blocks48_async", 4),
        ("replay_refill_blocks40_async", 3),
        ("replay_norefill_blocks48_async", 2),
        ("replay_norefill_blocks40_async", 1),
        ("replay_first_then_shared_blocks40", 3),
    ],
)
def test_oracle_reproduces_reference_pressure_run(name, preemptions):
    """KV pressure under recompute: a decoder whose next block cannot be had stalls, is restaged
    at the head of the next tick, and when nothing can run the stalled request with the shortest
    context is reset to prompt + generated text and re-queued, blocking new admissions until a
    request retires. Under reserve admission the same pool admits a prompt only while every
    admitted request's worst-case blocks fit, and nothing is preempted. In the delayed timing a
    wave's boundary coda is consumed during the next wave, so its finished requests hold their
    blocks until then and a successor that found no block sits that wave out."""

    data, shape, sd = _load_ouro("ouro_cfg0_pressure.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    cfg = dataclasses.replace(
        _config(run, {**data, "num_blocks": run["num_blocks"]}),
        kv_pressure_mode=run.get("kv_pressure_mode", "recompute"), max_model_len=run.get("max_model_len", 2048),
    )
    engine = OracleEngine(shape, sd, cfg, torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    assert engine.stats["recompute_preemptions"] == run["stats"]["recompute_preemptions"] == preemptions
    assert exit_depth_histogram(engine) == run["stats"]["exit_depth_histogram"]


OFFLOAD_RUNS = [
    # name, (recompute, offload, restores)
    ("replay_refill_blocks48_host64", (0, 3, 3)),
    ("replay_refill_blocks40_host2", (0, 2, 2)),
    ("replay_refill_blocks48_host1", (2, 1, 1)),
    ("replay_norefill_blocks40_host64", (0, 1, 1)),
    ("replay_norefill_blocks48_host2", (1, 1, 1)),
    ("replay_refill_blocks40_host64_last_exited", (0, 0, 0)),
    ("replay_norefill_blocks40_host64_last_exited", (0, 1, 1)),
    ("replay_refill_blocks40_host2_async", (1, 2, 2)),
    ("replay_norefill_blocks40_host64_async", (0, 1, 1)),
]


@pytest.mark.parametrize("name,counts", OFFLOAD_RUNS)
def test_oracle_reproduces_reference_offload_run(name, counts):
    """KV pressure under offload: a stalled victim's blocks go to a host pool of ``num_cpu_blocks``
    blocks (recompute when they do not fit) and come back, ahead of fresh prompts, into newly
    allocated blocks. Tokens equal the reference's, so the restored KV is the victim's own."""

    data, shape, sd = _load_ouro("ouro_cfg0_offload.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    cfg = _config(run, {**data, "num_blocks": run["num_blocks"]})
    cfg.kv_pressure_mode = "offload"
    cfg.num_cpu_blocks = run["num_cpu_blocks"]
    engine = OracleEngine(shape, sd, cfg, torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    st = run["stats"]
    assert (st["recompute_preemptions"], st["offload_preemptions"], st["restores"]) == counts
    assert (
        engine.stats["recompute_preemptions"], engine.stats["offload_preemptions"], engine.stats["restores"]
    ) == counts


@pytest.mark.parametrize(
    "name,preemptions",
    [
        ("cb_async", 0),
        ("cb_sync", 0),
        ("cb_async_blocks40", 1),
        ("cb_sync_blocks48", 2),
        ("cb_async_eos_stop", 0),
        ("cb_sync_eos_stop", 0),
        ("cb_async_blocks40_host64", 0),
        ("cb_sync_blocks48_host2", 1),
        ("cb_async_blocks36_host3", 0),
        ("cb_async_reserve_blocks40", 0),
        ("cb_sync_reserve_blocks40", 0),
        ("cb_async_chunked48", 0),
        ("cb_sync_chunked48", 0),
    ],
)
def test_cb_oracle_reproduces_reference_run(name, preemptions):
    """The full-depth continuous-batching baseline (pipelined and serialized, ample and short KV
    pools, early finishes on EOS ids and stop sequences): tokens, the ordered prefill/decode
    batches with their block-table rows, and (pipelined, ample cache) every LM-head launch's
    logits equal the reference engine's."""

    from oracle.cb_engine import OracleCBEngine

    data, shape, sd = _load_ouro("ouro_cfg0_cb.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    host = run.get("num_cpu_blocks") or 0
    cfg = OracleConfig(
        block_size=16, num_blocks=run["num_blocks"], max_recurrent_steps=4, max_model_len=run["max_model_len"],
        kv_pressure_mode=run["kv_pressure_mode"], num_cpu_blocks=host,
        max_num_batched_tokens=run["max_num_batched_tokens"],
    )
    engine = OracleCBEngine(shape, sd, cfg, torch.float32, async_mode=run["async"])
    tokens = engine.generate(
        data["prompts"], data["max_new_tokens"], eos_token_ids=run["eos_token_id"],
        stop_sequences=run["stop_sequences"],
    )
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    st = run["stats"]
    assert engine.stats["recompute_preemptions"] == st["recompute_preemptions"] == preemptions
    assert engine.stats["decode_batches"] == st["decode_batches"]
    assert engine.stats["prefill_batches"] == st["prefill_batches"]
    assert sum(len(it["items"]) for it in engine.launches if it["kind"] == "decode") == st["decode_tokens"]
    if host:
        assert (engine.stats["offload_preemptions"], engine.stats["restores"]) == (
            st["offload_preemptions"], st["restores"]
        )
    if name == "cb_async":
        logits = np.load(GOLDEN / "ouro_cfg0_cb_logits.npz")
        assert len(engine.logits) == len(logits.files)
        for i, (_kind, lg) in enumerate(engine.logits):
            np.testing.assert_allclose(lg.numpy(), logits[f"{name}_{i}"], rtol=0, atol=1e-5)


def test_oracle_reproduces_reference_huginn_pressure_run():
    """Huginn in a 40-block pool under recompute: stalled decoders are soft-reset and re-prefilled
    through the prelude, core and coda cache layers; tokens and launches equal the reference's."""

    data, shape, sd = _load_huginn("huginn_small_pressure.json")
    run = data["runs"][0]
    cfg = OracleConfig(
        block_size=16, num_blocks=run["num_blocks"], max_recurrent_steps=shape.total_recurrent_steps,
        max_model_len=2048, synthetic_exit_replay=True, refill=True, kv_policy="single",
    )
    engine = OracleEngine(shape, sd, cfg, torch.float32)
    assert engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"]) == run["tokens"]
    assert engine.launches == run["launches"]
    assert engine.stats["recompute_preemptions"] == run["stats"]["recompute_preemptions"] > 0


@pytest.mark.parametrize("name", ["cb_async", "cb_sync"])
def test_cb_oracle_reproduces_reference_huginn_run(name):
    """The CB baseline on the small Huginn shape (every recurrent step on its own KV slot, as the
    reference cache lays out a model that names no layout): tokens and batches equal the
    reference's."""

    from oracle.cb_engine import OracleCBEngine

    data = json.loads((GOLDEN / "huginn_small_cb.json").read_text())
    shape = HuginnShape(**data["shape"])
    sd = random_huginn_state_dict(shape, seed=data["weights_seed"], embed_std=data["embed_std"])
    run = next(r for r in data["runs"] if r["name"] == name)
    cfg = OracleConfig(
        block_size=16, num_blocks=run["num_blocks"], max_recurrent_steps=shape.total_recurrent_steps,
        max_model_len=2048, kv_policy=run["kv_policy"],
    )
    engine = OracleCBEngine(shape, sd, cfg, torch.float32, async_mode=run["async"])
    assert engine.generate(data["prompts"], data["max_new_tokens"]) == run["tokens"]
    assert engine.launches == run["launches"]


@pytest.mark.parametrize(
    "name",
    [
        "replay_refill_chunked48",
        "replay_refill_chunked48_async",
        "replay_norefill_chunked48",
        "replay_refill_seqs6",
        "replay_refill_coda4",
    ],
)
def test_oracle_reproduces_reference_knobs_run(name):
    """Chunked prompts (48-token prefill budget) in both timings and without refill, a cap of 6
    resident requests, and a coda minimum of 4: tokens and launches equal the reference's."""

    data, shape, sd = _load_ouro("ouro_cfg0_knobs.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    cfg = dataclasses.replace(_config(run, data), **run["config"])
    engine = OracleEngine(shape, sd, cfg, torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]


@pytest.mark.parametrize("name", ["live_gate_refill", "replay_refill", "replay_norefill", "replay_last_exited"])
def test_oracle_reproduces_reference_run(golden, name):
    data, shape, sd = golden
    run = next(r for r in data["runs"] if r["name"] == name)
    engine = OracleEngine(shape, sd, _config(run, data), torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert len(engine.launches) == len(run["launches"])
    for mine, ref in zip(engine.launches, run["launches"], strict=True):
        assert mine == ref
    assert exit_depth_histogram(engine) == run["stats"]["exit_depth_histogram"]
    assert engine.refills == run["stats"]["scheduler_refills"]
    assert engine.stats["recurrent_batches"] == run["stats"]["recurrent_batches"]
    assert engine.stats["coda_batches"] == run["stats"]["coda_batches"]
    if name == "live_gate_refill":
        logits = np.load(GOLDEN / "ouro_cfg0_logits.npz")
        for i in range(6):
            ref = logits[f"live_gate_refill_{i}"]
            mine = engine.logits[i][1].numpy()
            np.testing.assert_allclose(mine, ref, rtol=0, atol=1e-5)


# ----------------------------------------------------------------------------- Huginn
# tests/golden/make_golden_huginn.py ran the reference HuginnForCausalLM + HuginnCDBAdapter at a
# small shape with Huginn's structure (prelude/core/coda, 96-wide heads, qk_bias, interleaved
# RoPE, tied LM head) under the live latent-difference gate and three replays.


def _load_huginn(name: str):
    from continuous_depth_batching_b200.huginn import HuginnShape, random_huginn_state_dict

    data = json.loads((GOLDEN / name).read_text())
    shape = HuginnShape(**data["shape"])
    sd = random_huginn_state_dict(shape, seed=data["weights_seed"], embed_std=data["embed_std"])
    return data, shape, sd


@pytest.fixture(scope="module")
def golden_huginn():
    return _load_huginn("huginn_small.json")


@pytest.fixture(scope="module")
def golden_huginn_async():
    return _load_huginn("huginn_small_async.json")


@pytest.mark.parametrize("name", ["live_gate_refill", "replay_refill", "replay_norefill", "replay_last_exited"])
def test_oracle_reproduces_reference_huginn_run(golden_huginn, name):
    _check_huginn(golden_huginn, name, "huginn_small_logits.npz")


@pytest.mark.parametrize("name", ASYNC_RUNS)
def test_oracle_reproduces_reference_huginn_async_run(golden_huginn_async, name):
    _check_huginn(golden_huginn_async, name, "huginn_small_async_logits.npz")


def _check_huginn(golden, name, logits_file):
    data, shape, sd = golden
    run = next(r for r in data["runs"] if r["name"] == name)
    cfg = OracleConfig(
        block_size=data["block_size"],
        num_blocks=data["num_blocks"],
        max_recurrent_steps=shape.total_recurrent_steps,
        max_model_len=2048,
        exit_threshold=data["exit_threshold"] if run["live_gate"] else None,
        synthetic_exit_replay=not run["live_gate"],
        refill=run["refill"],
        kv_policy=run["kv_policy"],
        kv_pressure_mode="reserve" if run["kv_policy"] == "last_exited" else "recompute",
        delayed=run.get("async", False),
    )
    engine = OracleEngine(shape, sd, cfg, torch.float32)
    tokens = engine.generate(data["prompts"], data["max_new_tokens"], exit_depths=run["exit_depths"])
    assert tokens == run["tokens"]
    assert engine.launches == run["launches"]
    assert exit_depth_histogram(engine) == run["stats"]["exit_depth_histogram"]
    assert engine.refills == run["stats"]["scheduler_refills"]
    assert engine.stats["recurrent_batches"] == run["stats"]["recurrent_batches"]
    assert engine.stats["coda_batches"] == run["stats"]["coda_batches"]
    if name.startswith("live_gate_refill"):
        logits = np.load(GOLDEN / logits_file)
        for i in range(len(logits.files)):
            np.testing.assert_allclose(engine.logits[i][1].numpy(), logits[f"{name}_{i}"], rtol=0, atol=1e-5)
