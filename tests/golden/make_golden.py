"""Generate the golden fixtures by running the reference engine itself on CPU.

Run in a container that has the reference checkout (read-only), with ``CDB_REFERENCE_SRC``
pointing at its ``src`` directory::

    CDB_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden.py [--async]

It builds the reference's own ``OuroForCausalLM`` at BASELINE config 0's shape, loads the
seeded weights from :func:`continuous_depth_batching_b200.ouro.random_ouro_state_dict`,
registers the CPU restatement of the paged FlashAttention contract
(:mod:`oracle.paged_attention`; FlashAttention-3 is a binary the image does not have) and
drives the reference ``ContinuousDepthBatchingEngine.generate_batch`` in its synchronous mode
(``use_async_batching=False``) or, with ``--async``, its default delayed-gate mode. Each run records the generated tokens, per-token exit depths,
engine stats, the launch trace (every prefill, recurrent and coda launch with its items,
positions, recurrent steps and block-table rows) and the logits of every LM-head call.

Outputs: ``tests/golden/ouro_cfg0.json`` (traces) and ``tests/golden/ouro_cfg0_logits.npz``;
with ``--async`` the reference's default timing (``use_async_batching=True``,
``delay_gate_consumption=True``) into ``ouro_cfg0_async.json`` / ``ouro_cfg0_async_logits.npz``.
The GPU box has no reference checkout; the tests only read these files.
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
if not os.environ.get("CDB_REFERENCE_SRC"):
    raise SystemExit("set CDB_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, os.environ["CDB_REFERENCE_SRC"])

from continuous_depth_batching_b200.ouro import OuroShape, random_ouro_state_dict  # noqa: E402
from oracle.paged_attention import cpu_paged_attention_forward  # noqa: E402
from oracle.workloads import config0_workload  # noqa: E402

CFG0 = OuroShape(
    vocab_size=1024,
    hidden_size=256,
    intermediate_size=704,
    num_hidden_layers=4,
    num_attention_heads=4,
    num_key_value_heads=4,
    head_dim=64,
    rope_theta=10000.0,
    rms_norm_eps=1e-6,
    max_position_embeddings=2048,
    total_ut_steps=4,
)
# A gate wide enough that the live hazard policy is not decided by the sign of a logit
# that sits within rounding of zero.
GATE_STD = 0.12


def build_reference_model(shape: OuroShape, kv_policy: str):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from looped_cdb.models.ouro.configuration_ouro import OuroConfig
    from looped_cdb.models.ouro.kv_cache_policy import configure_kv_cache_policy
    from looped_cdb.models.ouro.modeling_ouro import OuroForCausalLM

    ALL_ATTENTION_FUNCTIONS["paged|flash_attention_3"] = cpu_paged_attention_forward
    config = OuroConfig(
        vocab_size=shape.vocab_size,
        hidden_size=shape.hidden_size,
        intermediate_size=shape.intermediate_size,
        num_hidden_layers=shape.num_hidden_layers,
        num_attention_heads=shape.num_attention_heads,
        num_key_value_heads=shape.num_key_value_heads,
        max_position_embeddings=shape.max_position_embeddings,
        rope_theta=shape.rope_theta,
        rms_norm_eps=shape.rms_norm_eps,
        total_ut_steps=shape.total_ut_steps,
        layer_types=["full_attention"] * shape.num_hidden_layers,
        pad_token_id=None,
    )
    torch.manual_seed(0)
    model = OuroForCausalLM(config)
    model.config._attn_implementation = "paged|flash_attention_3"
    state = random_ouro_state_dict(shape, seed=0, gate_std=GATE_STD)
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected, unexpected
    assert all("lookahead" in m or "preloop" in m for m in missing), missing
    model.eval()
    configure_kv_cache_policy(model, kv_policy=kv_policy)
    return model


class Recorder:
    """Wraps the reference runner to log every launch, in order."""

    def __init__(self, engine) -> None:
        self.engine = engine
        self.launches: list[dict] = []
        self.logits: list[np.ndarray] = []
        runner = engine.runner
        cache = engine.cache
        bs = cache.block_size
        rid_index = lambda rid: int(rid.split("-")[1])  # noqa: E731

        def blocks_of(rid: str, length: int) -> list[int]:
            blocks = cache.cache_allocator.block_table[rid]
            return [int(b) for b in blocks[: -(-length // bs)]]

        orig_rec = runner.compute_recurrent_batch

        def compute_recurrent_batch(items, recurrent_kwargs=None):
            self.launches.append(
                {
                    "kind": "recurrent",
                    "items": [
                        [rid_index(it.state.request_id), it.token_position, it.recurrent_step] for it in items
                    ],
                    "blocks": [blocks_of(it.state.request_id, it.token_position + 1) for it in items],
                }
            )
            return orig_rec(items, recurrent_kwargs=recurrent_kwargs)

        orig_pre = runner.stage_prefill_batch

        def stage_prefill_batch(model, requests, **kw):
            entries = []
            for fut in requests:
                st = fut.state
                entries.append([rid_index(st.request_id), st.position_offset, fut.query_length, int(fut.has_new_token)])
            launch = {"kind": "prefill", "items": entries}
            self.launches.append(launch)
            out = orig_pre(model, requests, **kw)
            launch["blocks"] = [blocks_of(fut.state.request_id, fut.state.position_offset) for fut in requests]
            return out

        orig_coda = runner.stage_coda_batch

        def stage_coda_batch(items, allow_async=True):
            self.launches.append(
                {
                    "kind": "coda",
                    "items": [[rid_index(it.state.request_id), it.token_position, it.recurrent_step] for it in items],
                }
            )
            return orig_coda(items, allow_async=allow_async)

        runner.compute_recurrent_batch = compute_recurrent_batch
        runner.stage_prefill_batch = stage_prefill_batch
        runner.stage_coda_batch = stage_coda_batch

        lm_head = engine.model.lm_head
        orig_fwd = lm_head.forward

        def lm_forward(x):
            y = orig_fwd(x)
            self.logits.append(y.detach().reshape(-1, y.shape[-1]).float().numpy().copy())
            return y

        lm_head.forward = lm_forward


def run_case(
    name: str, *, kv_policy: str, refill: bool, live_gate: bool, exit_depths=None, num_blocks=4096, async_mode=False,
    eos_token_id=None, stop_sequences=None, pressure_mode=None, cpu_offload_space=None, max_model_len=2048,
    extra_cfg: dict | None = None,
):
    from looped_cdb.continuous_depth_batching import ContinuousDepthBatchingConfig, ContinuousDepthBatchingEngine

    model = build_reference_model(CFG0, kv_policy)
    prompts, max_new = config0_workload()
    cfg = ContinuousDepthBatchingConfig(
        block_size=16,
        num_blocks=num_blocks,
        max_recurrent_steps=CFG0.total_ut_steps,
        exit_threshold=0.5 if live_gate else None,
        synthetic_exit_replay=not live_gate,
        use_async_batching=async_mode,
        use_cuda_graph=False,
        use_cuda_graph_prefill=False,
        refill=refill,
        kv_policy=kv_policy,
        kv_pressure_mode=pressure_mode or ("reserve" if kv_policy == "last_exited" else "recompute"),
        cpu_offload_space=cpu_offload_space,
        max_model_len=max_model_len,
        **(extra_cfg or {}),
    )
    engine = ContinuousDepthBatchingEngine.from_model(model, cfg)
    rec = Recorder(engine)
    with torch.no_grad():
        outs = engine.generate_batch(
            prompts, max_new_tokens=max_new, eos_token_id=eos_token_id, stop_sequences=stop_sequences, warmup=False,
            exit_depths=exit_depths,
        )
    states_exit = {}
    for st in list(engine.scheduler.active_requests.values()):
        states_exit[st.request_id] = st.exit_depths
    stats = engine.last_stats
    result = {
        "name": name,
        "kv_policy": kv_policy,
        "refill": refill,
        "live_gate": live_gate,
        "async": async_mode,
        "eos_token_id": eos_token_id,
        "stop_sequences": stop_sequences,
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
            "offload_preemptions": getattr(engine.offloading_manager, "num_offload_preemptions", 0),
            "restores": getattr(engine.offloading_manager, "num_restores", 0),
            "num_cpu_blocks": getattr(engine.offloading_manager, "_num_cpu_blocks", 0),
        },
        "launches": rec.launches,
    }
    return result, rec.logits


def recorded_exit_depths(result: dict) -> list[list[int]]:
    """Per-request exit steps of a live-gate run, read back from its recurrent trace."""

    n = len(result["tokens"])
    last_step: dict[tuple[int, int], int] = {}
    for launch in result["launches"]:
        if launch["kind"] == "coda":
            for rid, pos, step in launch["items"]:
                last_step[(rid, pos)] = step
    depths = [[] for _ in range(n)]
    for (rid, pos), step in sorted(last_step.items()):
        depths[rid].append(step)
    return depths


def replay_depths(result: dict, async_mode: bool) -> list[list[int]]:
    """Replay depths that reproduce a live run. With delayed gate consumption (async mode) a
    replayed depth d exits at step d + 1, so the depths are the recorded exit steps minus one."""

    depths = recorded_exit_depths(result)
    return [[s - 1 for s in ds] for ds in depths] if async_mode else depths


def finish_main() -> None:
    """``--finish``: the replayed schedule with requests finishing early on EOS ids [363, 924] or
    the stop sequences [[314, 314], [585, 585]] (ids the seeded model emits), refill on and off,
    into ``ouro_cfg0_finish.json``."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gold = json.loads((HERE / "ouro_cfg0.json").read_text())
    depths = next(r for r in gold["runs"] if r["name"] == "replay_refill")["exit_depths"]
    runs = []
    for name, refill in (("replay_refill_eos_stop", True), ("replay_norefill_eos_stop", False)):
        res, _ = run_case(
            name, kv_policy="single", refill=refill, live_gate=False, exit_depths=depths,
            eos_token_id=[363, 924], stop_sequences=[[314, 314], [585, 585]],
        )
        runs.append(res)
    # the same in the delayed (default) timing, with the async replay depths
    agold = json.loads((HERE / "ouro_cfg0_async.json").read_text())
    for name, refill in (("replay_refill_eos_stop_async", True), ("replay_norefill_eos_stop_async", False)):
        tag = "refill" if refill else "norefill"
        adepths = next(r for r in agold["runs"] if r["name"] == f"replay_{tag}_async")["exit_depths"]
        res, _ = run_case(
            name, kv_policy="single", refill=refill, live_gate=False, exit_depths=adepths, async_mode=True,
            eos_token_id=[363, 924], stop_sequences=[[314, 314], [585, 585]],
        )
        runs.append(res)
    prompts, max_new = config0_workload()
    payload = {
        "generator": "tests/golden/make_golden.py --finish",
        "shape": CFG0.__dict__,
        "gate_std": GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "num_blocks": 4096,
        "runs": runs,
    }
    (HERE / "ouro_cfg0_finish.json").write_text(json.dumps(payload, separators=(",", ":")))
    for r in runs:
        print(r["name"], r["stats"], [len(t) for t in r["tokens"]])


def pressure_main() -> None:
    """``--pressure``: the replayed schedules (synchronous) in KV pools too small for the workload,
    under the default ``kv_pressure_mode="recompute"``: refill at 56 blocks (decoders stall and are
    restaged), 48 and 40 blocks (stalled decoders are preempted by soft reset and re-prefilled), and
    no-refill at 48 and 40 blocks; then both loops at 40 blocks under ``"reserve"`` admission
    (``max_model_len`` 512); then both loops at 48 and 40 blocks in the reference's default timing
    (delayed gate consumption), into ``ouro_cfg0_pressure.json``."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gold = json.loads((HERE / "ouro_cfg0.json").read_text())
    runs = []
    for refill, nbs in ((True, (56, 48, 40)), (False, (48, 40))):
        tag = "refill" if refill else "norefill"
        depths = next(r for r in gold["runs"] if r["name"] == f"replay_{tag}")["exit_depths"]
        for nb in nbs:
            res, _ = run_case(
                f"replay_{tag}_blocks{nb}", kv_policy="single", refill=refill, live_gate=False, exit_depths=depths,
                num_blocks=nb,
            )
            res["num_blocks"] = nb
            runs.append(res)
        # reserve admission: each admitted request commits its worst-case blocks up front, so
        # nothing is ever preempted (max_model_len 512 keeps a max-length request within 40 blocks)
        res, _ = run_case(
            f"replay_{tag}_reserve_blocks40", kv_policy="single", refill=refill, live_gate=False, exit_depths=depths,
            num_blocks=40, pressure_mode="reserve", max_model_len=512,
        )
        res["num_blocks"] = 40
        res["kv_pressure_mode"] = "reserve"
        res["max_model_len"] = 512
        runs.append(res)
    # first_then_shared (step 0 in slot 0, later steps share slot 1) under recompute pressure
    pgold = json.loads((HERE / "ouro_cfg0_policies.json").read_text())
    pdepths = next(r for r in pgold["runs"] if r["name"] == "replay_first_then_shared")["exit_depths"]
    res, _ = run_case(
        "replay_first_then_shared_blocks40", kv_policy="first_then_shared", refill=True, live_gate=False,
        exit_depths=pdepths, num_blocks=40,
    )
    res["num_blocks"] = 40
    runs.append(res)
    # the reference's default timing (delayed gate consumption) under recompute pressure
    agold = json.loads((HERE / "ouro_cfg0_async.json").read_text())
    for refill, nb in ((True, 48), (True, 40), (False, 48), (False, 40)):
        tag = "refill" if refill else "norefill"
        depths = next(r for r in agold["runs"] if r["name"] == f"replay_{tag}_async")["exit_depths"]
        res, _ = run_case(
            f"replay_{tag}_blocks{nb}_async", kv_policy="single", refill=refill, live_gate=False, exit_depths=depths,
            num_blocks=nb, async_mode=True,
        )
        res["num_blocks"] = nb
        runs.append(res)
    prompts, max_new = config0_workload()
    payload = {
        "generator": "tests/golden/make_golden.py --pressure",
        "shape": CFG0.__dict__,
        "gate_std": GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "runs": runs,
    }
    (HERE / "ouro_cfg0_pressure.json").write_text(json.dumps(payload, separators=(",", ":")))
    for r in runs:
        print(r["name"], r["stats"])


def policies_main() -> None:
    """``--policies``: the replayed schedule under the other KV layouts, into
    ``ouro_cfg0_policies.json``: ``first_then_shared`` (2 slots, step s -> slot min(s, 1)) in both
    timings, and ``depth_indexed`` at full depth (it only admits exits that wrote every slot)."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gold = json.loads((HERE / "ouro_cfg0.json").read_text())
    depths = next(r for r in gold["runs"] if r["name"] == "replay_refill")["exit_depths"]
    at_least_1 = [[max(d, 1) for d in ds] for ds in depths]
    full = [[CFG0.total_ut_steps - 1 for _ in ds] for ds in depths]
    runs = []
    for name, policy, dep, async_mode in (
        ("replay_first_then_shared", "first_then_shared", at_least_1, False),
        ("replay_first_then_shared_async", "first_then_shared", depths, True),
        ("replay_depth_indexed_full", "depth_indexed", full, False),
    ):
        res, _ = run_case(name, kv_policy=policy, refill=True, live_gate=False, exit_depths=dep, async_mode=async_mode)
        runs.append(res)
    prompts, max_new = config0_workload()
    payload = {
        "generator": "tests/golden/make_golden.py --policies",
        "shape": CFG0.__dict__,
        "gate_std": GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "num_blocks": 4096,
        "runs": runs,
    }
    (HERE / "ouro_cfg0_policies.json").write_text(json.dumps(payload, separators=(",", ":")))
    for r in runs:
        print(r["name"], r["stats"])


def main() -> None:
    """``python tests/golden/make_golden.py [--async]``: the synchronous runs, or with ``--async``
    the same runs under the reference's default timing (use_async_batching=True,
    delay_gate_consumption=True) plus a live-gate no-refill run, into ``ouro_cfg0_async.*``."""

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

    replay, replay_logits = run_case(
        "replay_refill" + sfx, kv_policy="single", refill=True, live_gate=False, exit_depths=depths,
        async_mode=async_mode,
    )
    runs.append(replay)
    norefill, _ = run_case(
        "replay_norefill" + sfx, kv_policy="single", refill=False, live_gate=False, exit_depths=depths,
        async_mode=async_mode,
    )
    runs.append(norefill)
    lastx, _ = run_case(
        "replay_last_exited" + sfx, kv_policy="last_exited", refill=True, live_gate=False, exit_depths=depths,
        async_mode=async_mode,
    )
    runs.append(lastx)
    if async_mode:
        live_nr, _ = run_case("live_gate_norefill" + sfx, kv_policy="single", refill=False, live_gate=True,
                              async_mode=True)
        runs.append(live_nr)

    for i, arr in enumerate(live_logits[:6]):
        logits_out[f"live_gate_refill{sfx}_{i}"] = arr.astype(np.float32)
    prompts, max_new = config0_workload()
    payload = {
        "generator": "tests/golden/make_golden.py",
        "shape": CFG0.__dict__,
        "gate_std": GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "num_blocks": 4096,
        "runs": runs,
    }
    (HERE / f"ouro_cfg0{sfx}.json").write_text(json.dumps(payload, separators=(",", ":")))
    np.savez_compressed(HERE / f"ouro_cfg0{sfx}_logits.npz", **logits_out)
    print("wrote", HERE / f"ouro_cfg0{sfx}.json", "runs:", [r["name"] for r in runs])
    for r in runs:
        print(r["name"], r["stats"])


def offload_main() -> None:
    """``--offload``: the replayed schedules in KV pools too small for the workload under
    ``kv_pressure_mode="offload"``. A stalled victim's blocks are swapped to a host pool of
    ``num_cpu_blocks`` blocks and restored (admitted ahead of fresh prompts) once blocks free up;
    a victim that does not fit the host pool falls back to recompute. Host pools of 64 blocks
    (every victim fits), 2 and 1 (offload and recompute mixed), refill and no-refill; and under
    ``last_exited`` (4 KV slots per layer, every slot's blocks swapped; no recompute fallback); and
    both loops in the delayed (default) timing, into ``ouro_cfg0_offload.json``.
    The host pool is given in GiB, as the reference's config takes it: ``num_cpu_blocks`` times
    the bytes of one block over all cache layers (K and V) in the cache dtype."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gold = json.loads((HERE / "ouro_cfg0.json").read_text())
    block_bytes = 2 * CFG0.num_hidden_layers * 16 * CFG0.num_key_value_heads * CFG0.head_dim * 4
    runs = []
    for refill, nb, cpu_blocks, policy in (
        (True, 48, 64, "single"), (True, 40, 2, "single"), (True, 48, 1, "single"), (False, 40, 64, "single"),
        (False, 48, 2, "single"), (True, 40, 64, "last_exited"), (False, 40, 64, "last_exited"),
    ):
        tag = "refill" if refill else "norefill"
        src = "replay_last_exited" if policy == "last_exited" else f"replay_{tag}"
        depths = next(r for r in gold["runs"] if r["name"] == src)["exit_depths"]
        slots = CFG0.total_ut_steps if policy == "last_exited" else 1
        name = f"replay_{tag}_blocks{nb}_host{cpu_blocks}" + ("_last_exited" if policy == "last_exited" else "")
        res, _ = run_case(
            name, kv_policy=policy, refill=refill, live_gate=False, exit_depths=depths, num_blocks=nb,
            pressure_mode="offload", cpu_offload_space=cpu_blocks * block_bytes * slots / 1024**3,
        )
        assert res["stats"]["num_cpu_blocks"] == cpu_blocks, res["stats"]
        res["num_blocks"] = nb
        res["num_cpu_blocks"] = cpu_blocks
        runs.append(res)
    # the reference's default timing (delayed gate consumption)
    agold = json.loads((HERE / "ouro_cfg0_async.json").read_text())
    for refill, nb, cpu_blocks in ((True, 40, 2), (False, 40, 64)):
        tag = "refill" if refill else "norefill"
        depths = next(r for r in agold["runs"] if r["name"] == f"replay_{tag}_async")["exit_depths"]
        res, _ = run_case(
            f"replay_{tag}_blocks{nb}_host{cpu_blocks}_async", kv_policy="single", refill=refill, live_gate=False,
            exit_depths=depths, num_blocks=nb, pressure_mode="offload", async_mode=True,
            cpu_offload_space=cpu_blocks * block_bytes / 1024**3,
        )
        res["num_blocks"] = nb
        res["num_cpu_blocks"] = cpu_blocks
        runs.append(res)
    prompts, max_new = config0_workload()
    payload = {
        "generator": "tests/golden/make_golden.py --offload",
        "shape": CFG0.__dict__,
        "gate_std": GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "runs": runs,
    }
    (HERE / "ouro_cfg0_offload.json").write_text(json.dumps(payload, separators=(",", ":")))
    for r in runs:
        print(r["name"], r["stats"])


def knobs_main() -> None:
    """``--knobs``: the replayed schedule under non-default scheduler settings, into
    ``ouro_cfg0_knobs.json``: a 48-token prefill budget (prompts are chunked and a request is
    PREFILLING across several batches), refill synchronous and delayed and no-refill; at most 6
    resident requests (admission waits for open slots); and a coda minimum of 4 exited tokens."""

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gold = json.loads((HERE / "ouro_cfg0.json").read_text())
    runs = []
    for name, refill, async_mode, extra in (
        ("replay_refill_chunked48", True, False, {"max_num_batched_tokens": 48}),
        ("replay_refill_chunked48_async", True, True, {"max_num_batched_tokens": 48}),
        ("replay_norefill_chunked48", False, False, {"max_num_batched_tokens": 48}),
        ("replay_refill_seqs6", True, False, {"max_num_seqs": 6}),
        ("replay_refill_coda4", True, False, {"min_coda_batch_size": 4}),
    ):
        tag = "refill" if refill else "norefill"
        src = next(r for r in gold["runs"] if r["name"] == f"replay_{tag}")["exit_depths"]
        if async_mode:
            src = json.loads((HERE / "ouro_cfg0_async.json").read_text())
            src = next(r for r in src["runs"] if r["name"] == "replay_refill_async")["exit_depths"]
        res, _ = run_case(
            name, kv_policy="single", refill=refill, live_gate=False, exit_depths=src, async_mode=async_mode,
            extra_cfg=extra,
        )
        res["config"] = extra
        runs.append(res)
    prompts, max_new = config0_workload()
    payload = {
        "generator": "tests/golden/make_golden.py --knobs",
        "shape": CFG0.__dict__,
        "gate_std": GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "num_blocks": 4096,
        "runs": runs,
    }
    (HERE / "ouro_cfg0_knobs.json").write_text(json.dumps(payload, separators=(",", ":")))
    for r in runs:
        print(r["name"], r["stats"]["prefill_batches"], r["stats"]["coda_batches"], len(r["launches"]))


if __name__ == "__main__":
    if "--knobs" in sys.argv[1:]:
        knobs_main()
    elif "--offload" in sys.argv[1:]:
        offload_main()
    elif "--policies" in sys.argv[1:]:
        policies_main()
    elif "--finish" in sys.argv[1:]:
        finish_main()
    elif "--pressure" in sys.argv[1:]:
        pressure_main()
    else:
        main()
