"""The engine's host scheduler, run on the CPU against the reference's recorded schedules.

The B200 engine keeps its queues, block allocator and request lifecycle on the host and launches
device work through its runner. Here the runner is replaced by a host stand-in that launches
nothing: it hands out the same block pool and KV layout, and each LM-head row it would sample
gets a deterministic token. Everything else, from admission and chunked prefill through the
recurrent queue, exit routing, codas, stalls and recompute preemption, is the engine's own code.
With the replayed exit schedules of the reference runs, its launch trace (each launch's kind,
items and block-table rows) must equal the trace recorded from the reference engine. The GPU tests
repeat these comparisons through the real runner.
"""

from __future__ import annotations

import json
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from continuous_depth_batching_b200 import ContinuousDepthBatchingConfig, ContinuousDepthBatchingEngine, OuroShape
from continuous_depth_batching_b200.kv_cache import BlockPool, LoopedKvLayout

GOLDEN = Path(__file__).resolve().parent / "golden"


def _token(log_row: int, vocab: int) -> int:
    return (7 * log_row + 3) % vocab


class _HostRunner:
    """The runner surface the engine drives, with no device work behind it."""

    def __init__(self, cfg: ContinuousDepthBatchingConfig, shape: OuroShape) -> None:
        self.vocab = shape.vocab_size
        self.pool = SimpleNamespace(
            pool=BlockPool(cfg.num_blocks, cfg.block_size, cfg.decode_block_table_width()),
            num_host_blocks=0,
            host_copies=[],
            host_copy=lambda dev, host, to_host, stream: self.pool.host_copies.append((list(dev), list(host), to_host)),
        )
        self.rebinds: list[tuple[int, int]] = []
        self.layout = LoopedKvLayout(
            num_prelude_layers=0, num_core_layers=shape.num_hidden_layers, num_coda_layers=0,
            total_recurrent_steps=cfg.max_recurrent_steps, policy=cfg.kv_policy,
            requested_slots=cfg.kv_slots_per_layer,
        )
        self.bank_slots = 2 * cfg.max_num_seqs + 8
        self.stats = SimpleNamespace(recurrent_graph_hits=0, recurrent_graph_captures=0)
        self.stream = SimpleNamespace(synchronize=lambda: None)
        self.prefill_ids: list[list[int]] = []
        self.token_log = torch.zeros(1, dtype=torch.int64)

    def reset(self, log_len: int) -> None:
        self.pool.pool.reset()
        self.token_log = torch.zeros(log_len, dtype=torch.int64)
        self.prefill_ids = []

    def _sample(self, log_rows) -> None:
        for row in log_rows:
            self.token_log[row] = _token(row, self.vocab)

    def prefill(self, ids, slots, pos, logit_rows, log_rows, req_slots, kv_slots, keep_logits=False):
        self.prefill_ids.append(list(ids))
        self._sample(log_rows)
        return None

    def coda(self, hidden, log_rows, slots, keep_logits=False, positions=None):
        self._sample(log_rows)
        return None

    def prelude(self, *args, **kwargs) -> None:
        pass

    def recurrent(self, *args, **kwargs) -> None:
        pass

    def exit_kv_copy(self, rows, pairs) -> None:
        pass

    def rebind_token(self, req_slot: int, log_row: int) -> None:
        self.rebinds.append((req_slot, log_row))

    def read_tokens(self, n: int) -> list[int]:
        return self.token_log[:n].tolist()

    def check_status(self) -> None:
        pass


def _engine(data: dict, run: dict, num_blocks: int, host_blocks: int = 0) -> ContinuousDepthBatchingEngine:
    shape = OuroShape(**data["shape"])
    kv_policy = run.get("kv_policy", "single")
    pressure = run.get("kv_pressure_mode") or (
        "offload" if host_blocks else ("reserve" if kv_policy == "last_exited" else "recompute")
    )
    cfg = ContinuousDepthBatchingConfig(
        block_size=16,
        num_blocks=num_blocks,
        max_recurrent_steps=shape.total_ut_steps,
        synthetic_exit_replay=True,
        use_async_batching=run.get("async", False),
        refill=run["refill"],
        kv_policy=kv_policy,
        kv_pressure_mode=pressure,
        cpu_offload_space=1.0 if host_blocks else None,
        max_model_len=run.get("max_model_len", 2048),
    ).get_resolved()
    runner = _HostRunner(cfg, shape)
    runner.pool.num_host_blocks = host_blocks
    eng = ContinuousDepthBatchingEngine(None, cfg, runner, shape)
    eng.record_trace = True
    return eng


def _check_prefill_contents(eng: ContinuousDepthBatchingEngine, prompts, outs) -> None:
    """Every prefill chunk holds the request's prompt followed by its generated tokens at the
    chunk's positions, so a re-prefill after a preemption recomputes exactly the tokens it had."""

    prefills = [t for t in eng.launch_trace if t["kind"] == "prefill"]
    assert len(prefills) == len(eng.runner.prefill_ids)
    for trace, ids in zip(prefills, eng.runner.prefill_ids, strict=True):
        k = 0
        for idx, past, qlen, _ in trace["items"]:
            seq = list(prompts[idx]) + list(outs[idx].generated_tokens)
            assert ids[k : k + qlen] == seq[past : past + qlen]
            k += qlen
        assert k == len(ids)


def _run(data: dict, run: dict, num_blocks: int, forced=None, eos=None, stops=None, host_blocks: int = 0):
    eng = _engine(data, run, num_blocks, host_blocks)
    outs = eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=eos, stop_sequences=stops,
        exit_depths=run["exit_depths"], forced_tokens=forced,
    )
    return eng, outs


def _load(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


PRESSURE = [
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
]


@pytest.mark.parametrize("name,preemptions", PRESSURE)
def test_kv_pressure_schedule_matches_reference(name, preemptions):
    """Recompute mode in pools too small for the workload: stalls, restaging, preemption of the
    shortest stalled request, its re-prefill and the admission hold equal the reference's."""

    data = _load("ouro_cfg0_pressure.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng, outs = _run(data, run, run["num_blocks"])
    assert eng.launch_trace == run["launches"]
    assert eng.last_stats.recompute_preemptions == run["stats"]["recompute_preemptions"] == preemptions
    assert [len(o.generated_tokens) for o in outs] == data["max_new_tokens"]
    assert [o.generated_tokens for o in outs] == [
        [_token(r_base + g, OuroShape(**data["shape"]).vocab_size) for g in range(m)]
        for r_base, m in zip(_log_bases(data["max_new_tokens"]), data["max_new_tokens"], strict=True)
    ]
    _check_prefill_contents(eng, data["prompts"], outs)
    assert not eng.stalled and not eng.block_new


OFFLOAD = [
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


@pytest.mark.parametrize("name,counts", OFFLOAD)
def test_kv_offload_schedule_matches_reference(name, counts):
    """Offload mode: victims' blocks go to the host pool (recompute when it is full) and return
    ahead of fresh prompts; the launch trace, block tables and counters equal the reference's. Each
    restore copies back exactly the host blocks its offload filled, into the first of the request's
    new blocks, and rebinds its pending token to its new block-table row."""

    data = _load("ouro_cfg0_offload.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng, outs = _run(data, run, run["num_blocks"], host_blocks=run["num_cpu_blocks"])
    assert eng.launch_trace == run["launches"]
    st = eng.last_stats
    assert (st.recompute_preemptions, st.offload_preemptions, st.restores) == counts
    assert [len(o.generated_tokens) for o in outs] == data["max_new_tokens"]
    _check_prefill_contents(eng, data["prompts"], outs)
    copies = eng.runner.pool.host_copies
    outs_ = [c for c in copies if c[2]]
    ins = [c for c in copies if not c[2]]
    assert len(outs_) == counts[1] and len(ins) == counts[2]
    for (dev_out, host_out, _), (dev_in, host_in, _) in zip(outs_, ins, strict=True):
        assert host_in == host_out and len(dev_in) == len(dev_out)
        assert max(host_out) < run["num_cpu_blocks"]
    assert len(eng.runner.rebinds) == counts[2]
    assert not eng.host_tables and len(eng.host_free) == run["num_cpu_blocks"]


def _log_bases(max_new: list[int]) -> list[int]:
    out, base = [], 0
    for m in max_new:
        out.append(base)
        base += m
    return out


@pytest.mark.parametrize("name", ["replay_refill", "replay_norefill", "replay_last_exited"])
def test_schedule_matches_reference(name):
    data = _load("ouro_cfg0.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng, _ = _run(data, run, data["num_blocks"])
    assert eng.launch_trace == run["launches"]
    assert eng.last_stats.scheduler_refills == run["stats"]["scheduler_refills"]
    assert eng.last_stats.recompute_preemptions == 0


@pytest.mark.parametrize("name", ["replay_refill_async", "replay_norefill_async", "replay_last_exited_async"])
def test_async_schedule_matches_reference(name):
    data = _load("ouro_cfg0_async.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng, _ = _run(data, run, data["num_blocks"])
    assert eng.launch_trace == run["launches"]


@pytest.mark.parametrize("name", ["replay_first_then_shared", "replay_first_then_shared_async", "replay_depth_indexed_full"])
def test_kv_policy_schedule_matches_reference(name):
    data = _load("ouro_cfg0_policies.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng, _ = _run(data, run, data["num_blocks"])
    assert eng.launch_trace == run["launches"]


@pytest.mark.parametrize("name", ["replay_refill_eos_stop", "replay_norefill_eos_stop"])
def test_early_finish_schedule_matches_reference(name):
    data = _load("ouro_cfg0_finish.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng, outs = _run(
        data, run, data["num_blocks"], forced=run["tokens"], eos=run["eos_token_id"], stops=run["stop_sequences"]
    )
    assert eng.launch_trace == run["launches"]
    assert [len(o.generated_tokens) for o in outs] == [len(t) for t in run["tokens"]]


CB_RUNS = [
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
]


@pytest.mark.parametrize("name,preemptions", CB_RUNS)
def test_cb_schedule_matches_reference(name, preemptions):
    """The full-depth continuous-batching baseline: its FIFO prefill-or-decode ticks, pipelined
    (batch k+1 launched before batch k is consumed) and serialized, with the recompute eviction
    under a short KV pool, equal the reference CB engine's batches and block tables."""

    from continuous_depth_batching_b200 import ContinuousBatchingConfig, ContinuousBatchingEngine
    from continuous_depth_batching_b200.config import ContinuousDepthBatchingConfig as CDBConfig

    data = _load("ouro_cfg0_cb.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    shape = OuroShape(**data["shape"])
    host = run.get("num_cpu_blocks") or 0
    cfg = CDBConfig(
        block_size=16, num_blocks=run["num_blocks"], max_recurrent_steps=shape.total_ut_steps,
        use_async_batching=run["async"], kv_policy="single", max_model_len=run["max_model_len"],
        kv_pressure_mode=run["kv_pressure_mode"], cpu_offload_space=1.0 if host else None,
        max_num_batched_tokens=run["max_num_batched_tokens"],
    ).get_resolved()
    runner = _HostRunner(cfg, shape)
    runner.pool.num_host_blocks = host
    eng = ContinuousBatchingEngine(None, cfg, runner, shape)
    eng.cb_config = ContinuousBatchingConfig(num_blocks=run["num_blocks"], use_async_batching=run["async"])
    eng.record_trace = True
    finish = run["eos_token_id"] is not None
    outs = eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=run["eos_token_id"],
        stop_sequences=run["stop_sequences"], forced_tokens=run["tokens"] if finish else None,
    )
    assert eng.launch_trace == run["launches"]
    st, ref = eng.last_stats, run["stats"]
    assert st.recompute_preemptions == ref["recompute_preemptions"] == preemptions
    for k in ("prefill_batches", "prefill_requests", "prefill_query_tokens", "decode_batches", "decode_tokens"):
        assert getattr(st, k) == ref[k], k
    if host:
        assert (st.offload_preemptions, st.restores) == (ref["offload_preemptions"], ref["restores"])
        assert not eng.host_tables and len(eng.host_free) == host
    assert [len(o.generated_tokens) for o in outs] == [len(t) for t in run["tokens"]]
    _check_prefill_contents(eng, data["prompts"], outs)


KNOBS = [
    "replay_refill_chunked48",
    "replay_refill_chunked48_async",
    "replay_norefill_chunked48",
    "replay_refill_seqs6",
    "replay_refill_coda4",
]


@pytest.mark.parametrize("name", KNOBS)
def test_scheduler_settings_match_reference(name):
    """Non-default scheduler settings (``tests/golden/ouro_cfg0_knobs.json``): a 48-token prefill
    budget, so prompts are chunked over several batches (refill in both timings, and no-refill);
    at most 6 resident requests; a coda minimum of 4 exited tokens."""

    data = _load("ouro_cfg0_knobs.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    eng = _engine(data, {**run, "kv_policy": "single"}, data["num_blocks"])
    for key, value in run["config"].items():
        setattr(eng.cdb_config, key, value)
    eng.generate_batch(
        data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, exit_depths=run["exit_depths"]
    )
    assert eng.launch_trace == run["launches"]
    assert eng.last_stats.scheduler_refills == run["stats"]["scheduler_refills"]


def test_resident_cap_resolves_to_the_token_budget():
    """``resolve_max_num_seqs``: a prefill budget below ``max_num_seqs`` caps the resident set,
    and the default ``min_free_slots`` follows the resolved cap."""

    data = _load("ouro_cfg0_knobs.json")
    run = next(r for r in data["runs"] if r["name"] == "replay_refill_chunked48")
    eng = _engine(data, {**run, "kv_policy": "single"}, data["num_blocks"])
    eng.cdb_config.max_num_batched_tokens = 48
    eng._reset_state()
    assert (eng.max_num_seqs, eng.min_free, len(eng.free_slots)) == (48, 6, 48)


@pytest.mark.parametrize("name", ["replay_refill_eos_stop_async", "replay_norefill_eos_stop_async"])
def test_early_finish_lengths_in_delayed_timing(name):
    """Early finishes in the delayed timing, teacher-forced on the reference's tokens: every request
    ends where the reference's does (the launches differ by the successors the reference stages and
    cancels)."""

    data = _load("ouro_cfg0_finish.json")
    run = next(r for r in data["runs"] if r["name"] == name)
    _eng, outs = _run(
        data, run, data["num_blocks"], forced=run["tokens"], eos=run["eos_token_id"], stops=run["stop_sequences"]
    )
    assert [len(o.generated_tokens) for o in outs] == [len(t) for t in run["tokens"]]


def test_single_request_that_cannot_fit_raises():
    """With one active request left and no block for its next token, preemption cannot help: the
    reference raises ``CacheFullError`` (``continuous_api.py:1640-1646``)."""

    from continuous_depth_batching_b200.engine import CacheFullError

    data = _load("ouro_cfg0_pressure.json")
    run = {"refill": True, "exit_depths": [[0] * 63]}
    one = {**data, "prompts": [list(range(30))], "max_new_tokens": [64]}
    eng = _engine(one, run, 2)
    with pytest.raises(CacheFullError, match="single request's KV cache does not fit"):
        eng.generate_batch(one["prompts"], max_new_tokens=[64], eos_token_id=None, exit_depths=run["exit_depths"])


def test_pressure_none_mode_raises_instead_of_stalling():
    data = _load("ouro_cfg0_pressure.json")
    run = next(r for r in data["runs"] if r["name"] == "replay_refill_blocks48")
    eng = _engine(data, run, run["num_blocks"])
    eng.cdb_config.kv_pressure_mode = "none"
    from continuous_depth_batching_b200.engine import CacheFullError

    with pytest.raises(CacheFullError, match="kv_pressure_mode='none' does no preemption"):
        eng.generate_batch(
            data["prompts"], max_new_tokens=data["max_new_tokens"], eos_token_id=None, exit_depths=run["exit_depths"]
        )


class _FakeEvent:
    """CUDA-event stand-in: every timed window reads 10 ms."""

    def __init__(self, enable_timing=False):
        self.recorded = False

    def record(self, stream=None):
        self.recorded = True

    def elapsed_time(self, other):
        assert self.recorded and other.recorded
        return 10.0


def test_cb_decode_step_latency_window(monkeypatch):
    """``measure_decode_step_latency``: with every prompt prefilled first (``safety_margin=0``),
    the window opens after ``warmup`` full-batch decode ticks and closes after ``timed`` more, at a
    uniform context (prompt length + warm-up tokens). Events are faked: the control flow is what is
    checked here."""

    from continuous_depth_batching_b200 import ContinuousBatchingEngine
    from continuous_depth_batching_b200.config import ContinuousDepthBatchingConfig as CDBConfig

    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "Event", _FakeEvent)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    shape = OuroShape(**_load("ouro_cfg0_cb.json")["shape"])
    cfg = CDBConfig(block_size=16, num_blocks=256, max_recurrent_steps=4, kv_policy="single", max_model_len=512,
                    safety_margin=0.0).get_resolved()
    eng = ContinuousBatchingEngine(None, cfg, _HostRunner(cfg, shape), shape)
    eng.record_trace = True
    prompts = [[(7 * i + j) % shape.vocab_size for j in range(20)] for i in range(6)]
    t = eng.measure_decode_step_latency(prompts, max_new_tokens=16, warmup_decode_steps=2, timed_decode_steps=5)
    assert (t.batch_size, t.context_length, t.context_min, t.context_max) == (6, 20, 22, 22)
    assert t.gpu_elapsed_ms == 10.0 and t.gpu_per_step_ms == 2.0 and t.per_step_ms >= 0
    kinds = [launch["kind"] for launch in eng.launch_trace]
    assert kinds == ["prefill"] + ["decode"] * 7
    with pytest.raises(ValueError, match="must exceed"):
        eng.measure_decode_step_latency(prompts, max_new_tokens=7, warmup_decode_steps=2, timed_decode_steps=5)
    with pytest.raises(ValueError, match="equal-length"):
        eng.measure_decode_step_latency([[1, 2], [3]], max_new_tokens=16, warmup_decode_steps=2, timed_decode_steps=5)
