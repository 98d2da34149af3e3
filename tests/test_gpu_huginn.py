"""Huginn on the B200 engine: schedule parity with the reference trace and numerics vs the oracle.

* Schedule parity (bit-exact): with the replayed exit schedule of the reference run, the
  engine's ordered launch trace (prefill / recurrent / coda launches, each item's request,
  position, recurrent step and block-table row) equals the trace recorded from the reference
  engine with ``HuginnCDBAdapter`` (``tests/golden/huginn_small.json``), for refill, no-refill
  and ``last_exited``, with and without CUDA graphs.
* Numerics (``tests/numerics.py`` criteria): teacher-forced on the fp32 oracle's tokens, the
  logits of every LM-head launch are as accurate against fp32 as the reference-style bf16
  oracle's, at the small golden shape and at Huginn-0125's layer widths (5280 wide, 55 heads of
  96, 17920 intermediate, 65536 vocabulary) with one block per stage.
* Live latent-difference gate: teacher-forced on the reference's tokens, the exit step the GPU
  picks for each token equals the reference's at >= 95% of tokens (decisions within bf16 noise
  of the threshold may flip).
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from continuous_depth_batching_b200 import ContinuousDepthBatchingConfig, ContinuousDepthBatchingEngine
from continuous_depth_batching_b200.huginn import HuginnForCausalLM, HuginnShape, random_huginn_state_dict
from oracle.engine import OracleConfig, OracleEngine
from oracle.workloads import ouro_lognormal_workload
from tests.numerics import assert_report, compare_lm_launches

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _golden():
    data = json.loads((GOLDEN / "huginn_small.json").read_text())
    return data, HuginnShape(**data["shape"])


def _engine(shape, sd, *, kv_policy="single", refill=True, threshold=None, num_blocks=4096, max_model_len=2048,
            graphs=True, async_mode=False):
    model = HuginnForCausalLM(shape)
    model.load_state_dict({k: v.to(torch.float32) for k, v in sd.items()})
    cfg = ContinuousDepthBatchingConfig(
        block_size=16,
        num_blocks=num_blocks,
        max_recurrent_steps=shape.total_recurrent_steps,
        exit_threshold=threshold,
        synthetic_exit_replay=threshold is None,
        use_async_batching=async_mode,
        use_cuda_graph=graphs,
        refill=refill,
        kv_policy=kv_policy,
        kv_pressure_mode="reserve" if kv_policy == "last_exited" else "recompute",
        max_model_len=max_model_len,
    )
    return ContinuousDepthBatchingEngine.from_model(model, cfg, device="cuda")


@pytest.mark.parametrize("name", ["replay_refill", "replay_norefill", "replay_last_exited"])
@pytest.mark.parametrize("graphs", [True, False])
def test_huginn_schedule_matches_reference(name, graphs):
    data, shape = _golden()
    run = next(r for r in data["runs"] if r["name"] == name)
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    eng = _engine(shape, sd, kv_policy=run["kv_policy"], refill=run["refill"], graphs=graphs)
    eng.record_trace = True
    outs = eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, exit_depths=run["exit_depths"]
    )
    assert eng.launch_trace == run["launches"]
    assert [len(o.generated_tokens) for o in outs] == data["max_new_tokens"]
    hist = {str(k): v for k, v in sorted(eng.last_stats.exit_depth_histogram.items())}
    assert hist == run["stats"]["exit_depth_histogram"]
    assert eng.last_stats.scheduler_refills == run["stats"]["scheduler_refills"]


def _oracle(shape, sd, prompts, max_new, depths, dtype, forced=None, kv_policy="single"):
    cfg = OracleConfig(
        block_size=16, num_blocks=4096, max_recurrent_steps=shape.total_recurrent_steps, max_model_len=4096,
        synthetic_exit_replay=True, kv_policy=kv_policy,
        kv_pressure_mode="reserve" if kv_policy == "last_exited" else "recompute",
    )
    eng = OracleEngine(shape, sd, cfg, dtype)
    toks = eng.generate(prompts, max_new, exit_depths=depths, forced_tokens=forced)
    return eng, toks


def _compare_teacher_forced(shape, sd, prompts, max_new, depths, kv_policy="single"):
    o32, toks = _oracle(shape, sd, prompts, max_new, depths, torch.float32, kv_policy=kv_policy)
    o16, _ = _oracle(shape, sd, prompts, max_new, depths, torch.bfloat16, forced=toks, kv_policy=kv_policy)
    eng = _engine(shape, sd, kv_policy=kv_policy, max_model_len=4096)
    eng.record_trace = True
    eng.keep_logits = True
    eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths, forced_tokens=toks)
    assert eng.launch_trace == o32.launches == o16.launches
    kinds = [k for k, _ in eng.lm_logits]
    assert kinds == [k for k, _ in o16.logits] == [k for k, _ in o32.logits]
    rep = compare_lm_launches([lg for _, lg in eng.lm_logits], [lg for _, lg in o16.logits], [lg for _, lg in o32.logits])
    print(rep)
    return rep


@pytest.mark.parametrize("kv_policy", ["single", "last_exited"])
def test_huginn_teacher_forced_logits_small(kv_policy):
    data, shape = _golden()
    name = "replay_last_exited" if kv_policy == "last_exited" else "replay_refill"
    run = next(r for r in data["runs"] if r["name"] == name)
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    n = 8
    assert_report(
        _compare_teacher_forced(
            shape, sd, data["prompts"][:n], data["max_new_tokens"][:n], run["exit_depths"][:n], kv_policy=kv_policy
        )
    )


def test_huginn_teacher_forced_0125_widths():
    """Huginn-0125 layer widths (E 5280, 55 x 96 heads, I 17920, V 65536), one block per stage."""

    shape = HuginnShape(
        vocab_size=65536, n_embd=5280, n_heads=55, intermediate_size=17920, n_layers_in_prelude=1,
        n_layers_in_recurrent_block=1, n_layers_in_coda=1, total_recurrent_steps=4, max_position_embeddings=4096,
    )
    sd = random_huginn_state_dict(shape, seed=2, embed_std=0.05)
    prompts, max_new, depths = ouro_lognormal_workload(
        3, vocab_size=shape.vocab_size, seed=5, prompt_median=24, prompt_cap=40, out_median=5, out_cap=6,
        depth_probs=(0.3, 0.3, 0.2, 0.2),
    )
    assert_report(_compare_teacher_forced(shape, sd, prompts, max_new, depths))


def test_huginn_live_latent_gate_matches_reference_decisions():
    data, shape = _golden()
    run = next(r for r in data["runs"] if r["name"] == "live_gate_refill")
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    eng = _engine(shape, sd, threshold=data["exit_threshold"])
    outs = eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, forced_tokens=run["tokens"]
    )
    ref_depths = [[] for _ in run["tokens"]]
    for launch in run["launches"]:
        if launch["kind"] == "coda":
            for req, _pos, step in launch["items"]:
                ref_depths[req].append(step)
    mine = [o.exit_depths for o in outs]
    pairs = [(a, b) for x, y in zip(mine, ref_depths, strict=True) for a, b in zip(x, y, strict=True)]
    assert len(pairs) == sum(len(x) for x in ref_depths)
    agree = sum(int(a == b) for a, b in pairs) / len(pairs)
    print({"exit_agreement": agree, "tokens": len(pairs)})
    assert agree >= 0.95


def _golden_async():
    data = json.loads((GOLDEN / "huginn_small_async.json").read_text())
    return data, HuginnShape(**data["shape"])


@pytest.mark.parametrize("name", ["replay_refill_async", "replay_norefill_async", "replay_last_exited_async"])
def test_huginn_async_schedule_matches_reference(name):
    """The reference's default delayed-gate timing, bit-exact against huginn_small_async.json."""

    data, shape = _golden_async()
    run = next(r for r in data["runs"] if r["name"] == name)
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    eng = _engine(shape, sd, kv_policy=run["kv_policy"], refill=run["refill"], async_mode=True)
    eng.record_trace = True
    eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, exit_depths=run["exit_depths"]
    )
    assert eng.launch_trace == run["launches"]
    hist = {str(k): v for k, v in sorted(eng.last_stats.exit_depth_histogram.items())}
    assert hist == run["stats"]["exit_depth_histogram"]
    assert eng.last_stats.scheduler_refills == run["stats"]["scheduler_refills"]


@pytest.mark.parametrize("name,refill", [("live_gate_refill_async", True), ("live_gate_norefill_async", False)])
def test_huginn_async_live_gate_matches_reference_decisions(name, refill):
    from tests.test_gpu_engine import exit_agreement

    data, shape = _golden_async()
    run = next(r for r in data["runs"] if r["name"] == name)
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    eng = _engine(shape, sd, refill=refill, threshold=data["exit_threshold"], async_mode=True)
    outs = eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, forced_tokens=run["tokens"]
    )
    agree = exit_agreement(outs, run)
    print({"run": name, "exit_agreement": agree})
    assert agree >= 0.95


@pytest.mark.parametrize("async_mode", [True, False])
def test_huginn_cb_baseline_matches_reference_and_oracle(async_mode):
    """The full-depth CB baseline on a Huginn model (prelude, 6 core steps and coda per decode
    batch, every step on its own KV slot as the reference cache lays a Huginn model out): batches
    and block tables equal the reference CB engine's (``tests/golden/huginn_small_cb.json``), and
    teacher-forced on the fp32 CB oracle's tokens every LM-head launch meets the numerics criteria."""

    from continuous_depth_batching_b200 import ContinuousBatchingConfig, ContinuousBatchingEngine
    from oracle.cb_engine import OracleCBEngine

    data = json.loads((GOLDEN / "huginn_small_cb.json").read_text())
    shape = HuginnShape(**data["shape"])
    run = next(r for r in data["runs"] if r["async"] == async_mode)
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    ocfg = OracleConfig(
        block_size=16, num_blocks=4096, max_recurrent_steps=shape.total_recurrent_steps, max_model_len=2048,
        kv_policy=run["kv_policy"],
    )
    o32 = OracleCBEngine(shape, sd, ocfg, torch.float32, async_mode=async_mode)
    toks = o32.generate(data["prompts"], data["max_new_tokens"])
    assert toks == run["tokens"]
    o16 = OracleCBEngine(shape, sd, ocfg, torch.bfloat16, async_mode=async_mode)
    o16.generate(data["prompts"], data["max_new_tokens"], forced_tokens=toks)
    model = HuginnForCausalLM(shape)
    model.load_state_dict({k: v.to(torch.float32) for k, v in sd.items()})
    cfg = ContinuousBatchingConfig(block_size=16, num_blocks=4096, use_async_batching=async_mode, max_model_len=2048)
    eng = ContinuousBatchingEngine.from_model(model, cfg, device="cuda")
    assert eng.cdb_config.kv_policy == run["kv_policy"]
    eng.record_trace = True
    eng.keep_logits = True
    eng.generate_batch(data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, forced_tokens=toks)
    assert eng.launch_trace == run["launches"] == o32.launches == o16.launches
    rep = compare_lm_launches([lg for _, lg in eng.lm_logits], [lg for _, lg in o16.logits], [lg for _, lg in o32.logits])
    print(rep)
    assert_report(rep)


def test_huginn_graphed_fused_coda_matches_stored_logits():
    """The decode prelude and coda replay CUDA graphs (padded to the bucket size, padding rows at
    position -1); the coda's fused LM head + argmax there must pick the argmax of the logits the
    eager coda stores for the same teacher-forced inputs at >= 99% of positions (the two launches
    run the GEMMs at different padded widths, so near-ties may flip)."""

    data, shape = _golden()
    run = next(r for r in data["runs"] if r["name"] == "replay_refill")
    sd = random_huginn_state_dict(shape, seed=0, embed_std=data["embed_std"])
    prompts, max_new, depths = data["prompts"], data["max_new_tokens"], run["exit_depths"]
    _o32, toks = _oracle(shape, sd, prompts, max_new, depths, torch.float32)
    preds = []
    for keep in (False, True):
        eng = _engine(shape, sd)
        eng.record_trace = True
        eng.keep_logits = keep
        outs = eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths,
                                  forced_tokens=toks)
        eng.runner.check_status()
        assert eng.launch_trace == run["launches"]
        kinds = {kind for kind, _bucket in eng.runner.stage_graphs}
        assert kinds == ({"prelude"} if keep else {"prelude", "coda"}), kinds
        preds.append([t for o in outs for t in o.generated_tokens])
    n = len(preds[0])
    assert n == len(preds[1]) == sum(max_new)
    agree = sum(int(a == b) for a, b in zip(preds[0], preds[1], strict=True)) / n
    print({"graphed_fused_vs_eager_stored": agree, "tokens": n})
    assert agree >= 0.99
