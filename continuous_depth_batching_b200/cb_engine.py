"""Full-depth continuous batching (CB) on the B200 kernels: the baseline CDB is measured against.

Mirror of the reference's ``ContinuousBatchingEngine`` (``continuous_batching/continuous_api.py:133-489``)
and ``FIFOScheduler`` (``continuous_batching/scheduler.py:45-267``): the same
``from_model`` / ``generate_batch`` / ``last_stats`` surface and the same schedule. Every token
is served at the model's full recurrent depth. Each tick runs one batch:
either prompt work (whole or chunked prompts, packed under the token and KV budgets while prefill
is admitted) or one decode token for every decoding request that its pending token will not
finish, up to ``max_num_seqs``. With ``use_async_batching`` (the default) the tick launches batch
k+1 before it consumes batch k, so the scheduler sees the resident set and the free blocks one
tick late, exactly as the reference's pipelined loop does. When nothing fits and nothing is in
flight, the active request with the fewest cached tokens is soft-reset and re-queued, and
admission is held until a request finishes (``kv_pressure_mode="recompute"``); under ``"offload"``
its blocks go to the pinned host pool when they fit and come back, ahead of fresh prompts, at
the start of a later tick.

The device work is the CDB engine's, on the same runner, graphs and kernels:
* a prompt batch is one full-depth prefill launch (``OuroRunner.prefill``: tiled prefill
  attention over every recurrent step, then the fused LM head and argmax on the sampling rows);
* a decode batch is the prelude, ``max_recurrent_steps`` recurrent launches over the same rows
  (one per step, each on its KV slot, through the captured recurrent graphs), and one coda.
Only the schedule differs from CDB: no token leaves the loop early and no slot is refilled.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass

import torch

from .config import DEFAULT_MAX_NUM_SEQS, ContinuousDepthBatchingConfig
from .engine import CacheFullError, ContinuousDepthBatchingEngine, GenerationOutput, RequestStatus, _Req

__all__ = ["ContinuousBatchingConfig", "ContinuousBatchingEngine", "ContinuousBatchingStats", "DecodeStepTiming"]


@dataclass
class ContinuousBatchingConfig:
    """Fields of the reference ``ContinuousBatchingConfig`` (``continuous_batching/config.py:42-86``)."""

    block_size: int = 16
    num_blocks: int | None = None
    mem_fraction_static: float | None = None
    max_num_batched_tokens: int = 8192
    max_num_seqs: int = DEFAULT_MAX_NUM_SEQS
    min_free_slots: int | None = None
    safety_margin: float = 0.2
    replay_eos_finishes: bool = False
    kv_pressure_mode: str = "recompute"
    cpu_offload_space: float | None = None
    max_model_len: int = 16384
    use_async_batching: bool = True
    use_cuda_graph: bool = True
    use_cuda_graph_prefill: bool = True


@dataclass
class ContinuousBatchingStats:
    """The reference ``ContinuousBatchingStats`` counters (``continuous_api.py:53-86``) plus the
    engine's own (preemptions, host synchronisations, generated tokens)."""

    prefill_batches: int = 0
    decode_batches: int = 0
    prefill_requests: int = 0
    prefill_query_tokens: int = 0
    decode_tokens: int = 0
    generated_tokens: int = 0
    recompute_preemptions: int = 0
    offload_preemptions: int = 0
    restores: int = 0
    host_syncs: int = 0
    kv_peak_blocks: int = 0

    @property
    def mean_prefill_batch_size(self) -> float:
        return self.prefill_requests / self.prefill_batches if self.prefill_batches else 0.0

    @property
    def mean_prefill_query_tokens(self) -> float:
        return self.prefill_query_tokens / self.prefill_batches if self.prefill_batches else 0.0

    @property
    def mean_decode_batch_size(self) -> float:
        return self.decode_tokens / self.decode_batches if self.decode_batches else 0.0


@dataclass
class DecodeStepTiming:
    """One steady-state decode step at full batch, prefill excluded (the reference's
    ``DecodeStepTiming``, ``continuous_api.py:106-131``). ``per_step_ms`` is host wall clock over the
    timed window (opened and closed by a device synchronisation) per step; ``gpu_per_step_ms`` the
    same window in CUDA events on the engine stream. ``context_min`` / ``context_max`` bracket the
    requests' KV lengths when the window opened."""

    batch_size: int
    context_length: int
    context_min: int
    context_max: int
    warmup_decode_steps: int
    timed_decode_steps: int
    wall_elapsed_ms: float
    gpu_elapsed_ms: float
    per_step_ms: float
    gpu_per_step_ms: float


class ContinuousBatchingEngine(ContinuousDepthBatchingEngine):
    """Full-depth continuous batching over the CDB engine's runner (Ouro and Huginn models)."""

    @classmethod
    def from_model(  # type: ignore[override]
        cls,
        model,
        cb_config: ContinuousBatchingConfig,
        *,
        dtype: torch.dtype | None = None,
        device: torch.device | str | None = None,
        kv_policy: str | None = None,
        fused_lm_head: bool = True,
    ) -> ContinuousBatchingEngine:
        """Build the engine for an Ouro or Huginn causal LM (reference parameter names).

        Every token runs the model's configured recurrent depth (``total_ut_steps`` /
        ``mean_recurrence``). ``kv_policy`` is the recurrent KV layout; by default the model
        config's ``_cdb_kv_policy``, else ``depth_indexed`` (one KV slot per recurrent step), which
        is what the reference's paged cache assumes for a model that does not name one
        (``continuous_batching/cache.py:160-163``)."""

        config = getattr(model, "config", None)
        steps = getattr(config, "total_ut_steps", None) or getattr(config, "mean_recurrence", None)
        if steps is None:
            raise TypeError(f"Continuous batching on the B200 kernels needs an Ouro or Huginn model; got {type(model)!r}")
        policy = kv_policy or getattr(config, "_cdb_kv_policy", None) or "depth_indexed"
        cdb = ContinuousDepthBatchingConfig(
            block_size=cb_config.block_size,
            num_blocks=cb_config.num_blocks,
            mem_fraction_static=cb_config.mem_fraction_static,
            max_num_batched_tokens=cb_config.max_num_batched_tokens,
            safety_margin=cb_config.safety_margin,
            replay_eos_finishes=cb_config.replay_eos_finishes,
            max_model_len=cb_config.max_model_len,
            use_async_batching=cb_config.use_async_batching,
            use_cuda_graph=cb_config.use_cuda_graph,
            use_cuda_graph_prefill=cb_config.use_cuda_graph_prefill,
            max_recurrent_steps=int(steps),
            max_num_seqs=cb_config.max_num_seqs,
            min_free_slots=cb_config.min_free_slots,
            kv_policy=policy,
            kv_pressure_mode=cb_config.kv_pressure_mode,
            cpu_offload_space=cb_config.cpu_offload_space,
        )
        eng = super().from_model(model, cdb, dtype=dtype, device=device, fused_lm_head=fused_lm_head)
        eng.cb_config = cb_config
        return eng

    # ------------------------------------------------------------------ public API
    @torch.no_grad()
    def generate_batch(  # type: ignore[override]
        self,
        input_ids: list[list[int]],
        *,
        max_new_tokens: int | list[int],
        eos_token_id: int | list[int] | None,
        stop_sequences: list[list[int]] | None = None,
        warmup: bool = True,
        model_kwargs: dict | None = None,
        arrival_offsets_s: list[float] | None = None,
        record_token_times: bool = False,
        record_queue_samples: bool = False,
        forced_tokens: list[list[int]] | None = None,
    ) -> list[GenerationOutput]:
        """Generate from tokenized prompts at full depth (``continuous_api.py:223-304``).

        ``forced_tokens`` (parity harness) continues each request with the given tokens instead of
        its own samples; the engine still records its own argmax at every position."""

        del warmup, record_queue_samples
        caps = self._validate(input_ids, max_new_tokens, None, model_kwargs)
        eos = set()
        if eos_token_id is not None:
            for t in [eos_token_id] if isinstance(eos_token_id, int) else eos_token_id:
                if t >= 0:
                    eos.add(int(t))
        stops = [list(s) for s in stop_sequences] if stop_sequences else []
        self._content_finish = bool(eos or stops)
        self._forced = forced_tokens
        self._gate_live = False
        self._delayed = False
        reqs: list[_Req] = []
        base = 0
        for i, (p, m) in enumerate(zip(input_ids, caps, strict=True)):
            r = _Req(i, list(p), m, [], eos, stops, record_token_times)
            r.log_base = base
            base += m
            reqs.append(r)
        self.runner.reset(max(base, 1))
        self._reset_state()
        self.last_stats = ContinuousBatchingStats()
        self._log_total = base
        arrivals = None
        if arrival_offsets_s is None:
            for r in reqs:
                self.waiting[r.idx] = r
        else:
            if len(arrival_offsets_s) != len(reqs):
                raise ValueError("arrival_offsets_s needs one offset per request")
            arrivals = deque(sorted(zip(arrival_offsets_s, range(len(reqs))), key=lambda x: (x[0], x[1])))
        self._reqs = reqs
        self._t0 = time.perf_counter()
        in_flight = None
        while arrivals or self.active or self.waiting or in_flight is not None:
            if arrivals:
                self._release_arrivals(arrivals)
                if not (self.active or self.waiting) and in_flight is None:
                    self._wait_next_arrival(arrivals)
                    continue
            in_flight = self._tick(in_flight)
        tokens = self.runner.read_tokens(base) if base else []
        self.runner.check_status()
        outs = [
            GenerationOutput(
                request_id=r.request_id,
                prompt_ids=r.prompt,
                generated_tokens=tokens[r.log_base : r.log_base + r.generated],
                status=r.status,
                created_time=r.created,
                lifespan=(r.start, r.finish),
                first_token_time=r.first_token,
                token_ready_times=r.token_times,
            )
            for r in reqs
        ]
        st = self.last_stats
        st.generated_tokens = sum(len(o.generated_tokens) for o in outs)
        st.kv_peak_blocks = self.runner.pool.pool.peak
        return outs

    @torch.no_grad()
    def measure_decode_step_latency(
        self,
        input_ids: list[list[int]],
        *,
        max_new_tokens: int,
        warmup_decode_steps: int,
        timed_decode_steps: int,
        model_kwargs: dict | None = None,
    ) -> DecodeStepTiming:
        """Time one full-batch decode step at full depth, isolated from prefill
        (``continuous_api.py:491-624``).

        ``B`` equal-length prompts are submitted; once all ``B`` decode together (a decode batch of
        ``B`` with nothing waiting) the next ``warmup_decode_steps`` such ticks settle, and the
        following ``timed_decode_steps`` are timed. Build the engine with ``safety_margin=0`` so every
        prompt prefills before decoding starts; ``max_new_tokens`` must outlast the window. Raises
        if the batch drops below ``B`` inside the window or never reaches it."""

        del model_kwargs
        if warmup_decode_steps < 1:
            raise ValueError("warmup_decode_steps must be >= 1 to settle the decode graph before timing")
        if timed_decode_steps < 1:
            raise ValueError("timed_decode_steps must be >= 1")
        if max_new_tokens <= warmup_decode_steps + timed_decode_steps:
            raise ValueError(
                f"max_new_tokens ({max_new_tokens}) must exceed warmup+timed decode steps "
                f"({warmup_decode_steps + timed_decode_steps})"
            )
        if not torch.cuda.is_available():
            raise RuntimeError("measure_decode_step_latency requires CUDA for event timing")
        self._validate_generate_inputs(input_ids, max_new_tokens)
        batch = len(input_ids)
        context = len(input_ids[0])
        if any(len(p) != context for p in input_ids):
            raise ValueError("measure_decode_step_latency expects equal-length prompts")
        caps = self._validate(input_ids, max_new_tokens, None, None)
        self._content_finish = False
        self._forced = None
        self._gate_live = False
        self._delayed = False
        reqs = []
        for i, (p, m) in enumerate(zip(input_ids, caps, strict=True)):
            r = _Req(i, list(p), m, [], set(), [], False)
            r.log_base = i * m
            reqs.append(r)
        self.runner.reset(max(sum(caps), 1))
        self._reset_state()
        self.last_stats = ContinuousBatchingStats()
        self._reqs = reqs
        for r in reqs:
            self.waiting[r.idx] = r
        stream = self.runner.stream
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        full_ticks = 0
        timing = False
        wall0 = 0.0
        ctx_min = ctx_max = context
        in_flight = None
        while self.active or self.waiting or in_flight is not None:
            self._last_launch = None
            try:
                in_flight = self._tick(in_flight)
            except CacheFullError as exc:
                raise CacheFullError(
                    f"could not assemble the full batch of {batch} requests at context {context}: the KV cache "
                    "is exhausted before all requests are resident. Increase num_blocks, or reduce the batch "
                    "size or context length."
                ) from exc
            launch = self._last_launch
            if not (launch is not None and launch[0] and launch[1] == batch and not self.waiting):
                if timing:
                    raise RuntimeError("decode batch dropped below B inside the timed window")
                continue
            full_ticks += 1
            if full_ticks < warmup_decode_steps:
                continue
            if full_ticks == warmup_decode_steps:
                torch.cuda.synchronize()
                lengths = [r.position for r in reqs]
                ctx_min, ctx_max = min(lengths), max(lengths)
                wall0 = time.perf_counter()
                start.record(stream)
                timing = True
                continue
            if full_ticks == warmup_decode_steps + timed_decode_steps:
                stop.record(stream)
                torch.cuda.synchronize()
                wall_ms = (time.perf_counter() - wall0) * 1e3
                gpu_ms = start.elapsed_time(stop)
                return DecodeStepTiming(
                    batch_size=batch, context_length=context, context_min=ctx_min, context_max=ctx_max,
                    warmup_decode_steps=warmup_decode_steps, timed_decode_steps=timed_decode_steps,
                    wall_elapsed_ms=wall_ms, gpu_elapsed_ms=gpu_ms, per_step_ms=wall_ms / timed_decode_steps,
                    gpu_per_step_ms=gpu_ms / timed_decode_steps,
                )
        raise RuntimeError(
            f"generation ended after {full_ticks} full-batch decode ticks before timing completed (need "
            f"{warmup_decode_steps + timed_decode_steps}); the batch may never reach B={batch} at this context, "
            "or max_new_tokens / the block budget is too small"
        )

    # ------------------------------------------------------------------ scheduling
    def _will_finish(self, r: _Req) -> bool:
        """``will_finish_on_pending_token`` (``continuous_batching/requests.py:196-206``)."""

        if self.cdb_config.replay_eos_finishes:
            return False
        return r.in_flight_tokens > 0 and r.generated + r.in_flight_tokens >= r.max_new

    def _cb_prefill_candidates(self) -> list[_Req]:
        """``get_prefill_candidates`` (``scheduler_base.py:473-516``); CB continues a chunked prompt
        whether or not its previous chunk is still in flight."""

        prefilling = [r for r in self.active.values() if r.status == RequestStatus.PREFILLING]
        free_res = max(0, self.max_num_seqs - len(self.active))
        fresh = [r for r in self.waiting.values() if not r.offloaded]  # offloaded ones return by restore
        admissible = [] if self.block_new else fresh[:free_res]
        if self.cdb_config.kv_pressure_mode == "reserve":
            committed = sum(self._reserved_peak(r) for r in self.active.values())
            kept = []
            for r in admissible:
                need = self._reserved_peak(r)
                if committed + need > self.cdb_config.num_blocks:
                    break
                committed += need
                kept.append(r)
            admissible = kept
        cands = prefilling + admissible
        if not cands:
            return []
        if any(r.status == RequestStatus.PREFILLING for r in cands):
            return cands
        return cands if free_res >= self.min_free else []

    def _cb_process(self, cands: list[_Req], token_budget: int, margin_frac: float):
        """``FIFOScheduler._process_candidates`` (``scheduler.py:183-267``) with
        ``_schedule_request`` (``:158-181``): ``([(req, q_len, samples)], allocation_failed)``."""

        cfg = self.cdb_config
        bs = cfg.block_size
        cache_budget = cfg.num_blocks * bs
        margin = margin_frac * cfg.num_blocks
        fast = True
        failed = False
        out = []
        for r in cands:
            n_free = self.pool.num_free
            decoding = r.status == RequestStatus.DECODING
            if n_free < margin and out and not decoding:
                break
            n_tokens = 1 if decoding else len(r.remaining)
            qlen = min(n_tokens, token_budget)
            if qlen == 0:
                continue
            eligible = qlen == 1 and r.position < self.width * bs
            read_needed = r.position
            if not (fast and eligible) and cache_budget < read_needed:
                continue
            bound_here = False
            if r.status == RequestStatus.PENDING and r.slot < 0:
                r.slot = self.free_slots.pop()
                bound_here = True
            if not self._alloc_if_needed(r, qlen):
                if bound_here:
                    self.free_slots.append(r.slot)
                    r.slot = -1
                failed = True
                if n_free == 0 and r.idx in self.waiting:
                    break
                continue
            if not decoding:
                if r.status == RequestStatus.PENDING:
                    self.active[r.idx] = r
                    if r.start < 0:
                        r.start = time.perf_counter()
                if n_tokens <= token_budget:
                    r.chunk, r.remaining = r.remaining, []
                    r.status = RequestStatus.DECODING
                else:
                    r.chunk, r.remaining = r.remaining[:token_budget], r.remaining[token_budget:]
                    r.status = RequestStatus.PREFILLING
                qlen = len(r.chunk)
            fast = fast and qlen == 1 and r.position < self.width * bs
            token_budget -= qlen
            cache_budget -= read_needed
            out.append((r, qlen, not r.remaining))
            self.waiting.pop(r.idx, None)
            if token_budget == 0 or (cache_budget <= 0 and not fast):
                break
        return out, failed

    def _schedule_batch(self):
        """``FIFOScheduler.schedule_batch`` (``scheduler.py:82-141``): ``(entries, cache_exhausted)``."""

        cfg = self.cdb_config
        # offloaded requests come back first, into new blocks with their KV (``scheduler.py:97-100``)
        self._restore_offloaded()
        decode = [r for r in self.active.values() if r.status == RequestStatus.DECODING and not self._will_finish(r)]
        prefill = self._cb_prefill_candidates()
        if prefill and (not decode or self.pool.num_free > self.safety * cfg.num_blocks):
            out, failed = self._cb_process(prefill, cfg.max_num_batched_tokens, self.safety)
            if out:
                return out, False
            if not decode:
                return [], failed
        if not decode:
            return [], False
        out, failed = self._cb_process(decode, self.max_num_seqs, 0.0)
        return out, (not out and failed)

    # ------------------------------------------------------------------ launches
    def _launch(self, entries) -> list[tuple[_Req, int]]:
        """Run one batch (``prepare_batch_tensors``, ``input_outputs.py:285-352``, then the model).
        Returns the sampling rows as ``(request, token-log row)``."""

        st = self.last_stats
        bs = self.cdb_config.block_size
        is_decode = all(q == 1 and r.status == RequestStatus.DECODING for r, q, _s in entries)
        self._last_launch = (is_decode, len(entries))
        if self.record_trace:
            self.launch_trace.append(
                {
                    "kind": "decode" if is_decode else "prefill",
                    "items": [[r.idx, r.position, q, int(s)] for r, q, s in entries],
                    "blocks": [list(self.pool.tables[r.idx][: -(-(r.position + q) // bs)]) for r, q, _s in entries],
                }
            )
        if is_decode:
            st.decode_batches += 1
            st.decode_tokens += len(entries)
            return self._launch_decode(entries)
        st.prefill_batches += 1
        st.prefill_requests += len(entries)
        st.prefill_query_tokens += sum(q for _r, q, _s in entries)
        ids, slots, pos, logit_rows, log_rows, req_slots, sampled = [], [], [], [], [], [], []
        for r, qlen, samples in entries:
            past = r.position
            ids.extend(r.chunk)
            slots.extend([r.slot] * qlen)
            pos.extend(range(past, past + qlen))
            r.position = past + qlen
            r.chunk = []
            if samples:
                row = r.log_base + r.generated + r.in_flight_tokens
                logit_rows.append(len(ids) - 1)
                log_rows.append(row)
                req_slots.append(r.slot)
                sampled.append((r, row))
                r.in_flight_tokens += 1
        logits = self.runner.prefill(
            ids, slots, pos, logit_rows, log_rows, req_slots, [self._slot_of_step(s) for s in range(self.steps)],
            keep_logits=self.keep_logits,
        )
        if logits is not None:
            self.lm_logits.append(("prefill", logits))
        return sampled

    def _launch_decode(self, entries) -> list[tuple[_Req, int]]:
        """Prelude, one recurrent launch per step over the same rows, coda."""

        n = len(entries)
        tokens, req_slots, positions, log_rows, sampled = [], [], [], [], []
        hidden = [self.free_hidden.pop() for _ in range(n)]
        for r, _q, _s in entries:
            if r.chunk:  # a prompt's last token: its id is on the host
                tokens.append(int(r.chunk[0]))
                r.chunk = []
            elif self._forced is not None:
                tokens.append(int(self._forced[r.idx][r.generated + r.in_flight_tokens - 1]))
            else:
                tokens.append(-1)  # the request's latest sampled token, from the device token table
            req_slots.append(r.slot)
            positions.append(r.position)
            row = r.log_base + r.generated + r.in_flight_tokens
            log_rows.append(row)
            sampled.append((r, row))
            r.position += 1
            r.in_flight_tokens += 1
        self.runner.prelude(tokens, req_slots, hidden, positions=positions)
        for step in range(self.steps):
            self.runner.recurrent(req_slots, positions, hidden, self._slot_of_step(step), False, steps=[step] * n)
        logits = self.runner.coda(hidden, log_rows, req_slots, keep_logits=self.keep_logits, positions=positions)
        if logits is not None:
            self.lm_logits.append(("decode", logits))
        self.free_hidden.extend(hidden)
        return sampled

    # ------------------------------------------------------------------ consumption
    def _consume(self, sampled: list[tuple[_Req, int]]) -> None:
        """``_consume_batch`` (``continuous_api.py:450-489``): rows of requests that finished (or
        were preempted) while the row was in flight are dropped."""

        live = [(r, row) for r, row in sampled if r.status not in (RequestStatus.FINISHED, RequestStatus.PENDING)]
        if self._content_finish and live:
            if self._forced is not None:
                for r, row in live:
                    r.pending_token = int(self._forced[r.idx][row - r.log_base])
            else:
                self.last_stats.host_syncs += 1
                self.runner.stream.synchronize()
                for r, row in live:
                    r.pending_token = int(self.runner.token_log[row].item())
        for r, _row in live:
            r.in_flight_tokens = max(0, r.in_flight_tokens - 1)
            if self._record_token(r):
                self._retire(r)

    def _evict(self) -> None:
        """``offload_one_request`` (``offloading_manager.py:165-214``): the active request with the
        fewest cached tokens (ties: the latest admitted) gives up its KV. Under ``offload`` its blocks
        are copied to the host pool if they fit there, and it waits with its status, position and
        pending token until it is restored. Otherwise it is soft-reset (``requests.py:290-315``) and
        re-queued as prompt + generated tokens."""

        victim = min(reversed(list(self.active)), key=lambda i: self.active[i].position)
        r = self.active.pop(victim)
        offloaded = self._offload(r)
        if not offloaded:
            if self._forced is None:
                self.last_stats.host_syncs += 1
                self.runner.stream.synchronize()
            generated = self._host_tokens(r)
        self.pool.release(r.idx)
        self.free_slots.append(r.slot)
        r.slot = -1
        r.allocated = 0
        r.chunk = []
        if offloaded:
            if r.status == RequestStatus.DECODING:
                r.remaining = []
            self.last_stats.offload_preemptions += 1
        else:
            r.remaining = list(r.prompt) + generated
            r.position = 0
            r.in_flight_tokens = 0
            r.status = RequestStatus.PENDING
            self.last_stats.recompute_preemptions += 1
        self.waiting[r.idx] = r
        self.block_new = True

    def _tick(self, in_flight):
        """``_execute_tick`` (``continuous_api.py:306-448``)."""

        entries, cache_full = [], False
        if self.active or self.waiting:
            entries, cache_full = self._schedule_batch()
            if not entries and not cache_full and in_flight is None:
                raise RuntimeError(
                    "No request could be scheduled: a pending prefill request's KV read exceeds the cache budget "
                    "(the prompt is too long for the KV cache)."
                )
        launched = self._launch(entries) if entries else None
        pipelined = self.cdb_config.use_async_batching
        to_consume = in_flight if pipelined else launched
        if to_consume is not None:
            self._consume(to_consume)
        if cache_full and to_consume is None:
            mode = self.cdb_config.kv_pressure_mode
            if mode == "none":
                raise CacheFullError(
                    "KV cache full and kv_pressure_mode='none' does no preemption. Increase num_blocks, reduce "
                    "load, or select kv_pressure_mode='reserve'/'recompute'."
                )
            if mode == "reserve":
                raise CacheFullError(
                    "Reserve admission over-committed the KV cache: an admitted request could not allocate. "
                    "This is a bug in reservation accounting."
                )
            if len(self.active) > 1:
                self._evict()
                return None
            raise CacheFullError(
                "No request could be scheduled and no request can be preempted: a single request's KV cache "
                "does not fit (increase num_blocks or reduce max_model_len)."
            )
        return launched if pipelined else None
