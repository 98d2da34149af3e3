"""``ContinuousDepthBatchingEngine``: the reference's engine surface over the B200 runner.

Public surface (kept verbatim from ``continuous_depth_batching/continuous_api.py``):
``from_model(model, cdb_config, *, dtype=None, model_adapter=None)`` (``:275-376``),
``generate_batch(input_ids, *, max_new_tokens, eos_token_id, stop_sequences=None, warmup=True,
model_kwargs=None, exit_depths=None, arrival_offsets_s=None, record_token_times=False,
record_queue_samples=False)`` (``:379-452``) and ``last_stats`` (``:114-228``).

Scheduling follows the reference's synchronous decision timing exactly, so every launch, block
table and per-step depth assignment is bit-identical to the reference run on the same inputs:

* refill loop ``:503-606`` with ``CDBScheduler.schedule_next`` (``scheduler.py:101-140``):
  coda when >= ``min_coda_batch_size`` -> prefill when admitted (``scheduler_base.py:129-201``)
  -> recurrent FIFO (slot-homogeneous under multi-slot KV, ``scheduler.py:322-346``) -> coda flush;
* recurrent routing ``:1090-1203``: exits go to the coda queue, survivors return to the queue
  head in order; coda re-entry ``:1378-1448`` puts each successor at the queue head;
* no-refill lockstep waves ``:608-944``; ``last_exited`` copy-on-exit ``:1205-1245``.

What differs is where the work runs. Token ids stay on the device (the coda's argmax feeds the
next prelude through the device token table), block tables live on the device and are patched
with new block ids only, and the host never waits for the device unless a decision needs device
data (a live exit gate, EOS or stop sequences): with replayed exits it schedules ahead while the
GPU executes, and reads every sampled token back once at the end.
"""

from __future__ import annotations

import time
from collections import Counter, OrderedDict, deque
from dataclasses import dataclass, field
from enum import IntEnum

import torch

from .config import ContinuousDepthBatchingConfig, validate_exit_threshold
from .huginn import HuginnShape
from .huginn_runner import HuginnRunner
from .kv_cache import copies_exit_kv, kv_slot_for_step, resolve_kv_slots_per_layer
from .model_adapter import resolve_cdb_model_adapter
from .ouro import OuroShape
from .runner import OuroRunner


class CacheFullError(RuntimeError):
    """Raised when the KV cache cannot place any work and nothing can relieve the pressure."""


class RequestStatus(IntEnum):
    PENDING = 0
    PREFILLING = 1
    DECODING = 2
    FINISHED = 3


@dataclass
class GenerationOutput:
    """Mirror of the reference ``GenerationOutput`` (``continuous_batching/requests.py:44-70``)."""

    request_id: str
    prompt_ids: list[int] = field(default_factory=list)
    generated_tokens: list[int] = field(default_factory=list)
    status: RequestStatus = RequestStatus.PENDING
    created_time: float = field(default_factory=time.perf_counter)
    lifespan: tuple[float, float] = (-1, -1)
    first_token_time: float = -1.0
    token_ready_times: list[float] = field(default_factory=list)
    exit_depths: list[int] = field(default_factory=list)

    def is_finished(self) -> bool:
        return self.status == RequestStatus.FINISHED


@dataclass
class ContinuousDepthBatchingStats:
    """Runtime counters (the reference ``ContinuousDepthBatchingStats`` fields this engine produces)."""

    prefill_batches: int = 0
    prefill_requests: int = 0
    recurrent_batches: int = 0
    coda_batches: int = 0
    recurrent_steps: int = 0
    coda_tokens: int = 0
    generated_tokens: int = 0
    prefill_recurrent_steps: int = 0
    prefill_coda_tokens: int = 0
    fixed_depth_recurrent_steps: int = 0
    exit_depth_histogram: Counter = field(default_factory=Counter)
    recurrent_step_histogram: Counter = field(default_factory=Counter)
    mixed_recurrent_batches: int = 0
    mixed_recurrent_depth_histogram: Counter = field(default_factory=Counter)
    max_mixed_depths_per_batch: int = 0
    scheduler_refills: int = 0
    max_depth_queue_size: int = 0
    recurrent_graph_hits: int = 0
    recurrent_graph_captures: int = 0
    scheduler_ticks: int = 0
    prefill_tokens: int = 0
    exit_kv_copies: int = 0
    host_syncs: int = 0
    kv_peak_blocks: int = 0
    recompute_preemptions: int = 0
    offload_preemptions: int = 0
    restores: int = 0

    @property
    def skipped_recurrent_steps(self) -> int:
        return max(0, self.fixed_depth_recurrent_steps - self.recurrent_steps)

    @property
    def mean_recurrent_batch_size(self) -> float:
        return self.recurrent_steps / self.recurrent_batches if self.recurrent_batches else 0.0

    @property
    def mean_coda_batch_size(self) -> float:
        return self.coda_tokens / self.coda_batches if self.coda_batches else 0.0


class _Req:
    __slots__ = (
        "idx", "request_id", "prompt", "max_new", "depths", "cursor", "status", "remaining", "chunk",
        "position", "allocated", "generated", "slot", "log_base", "exit_depths", "eos", "stops",
        "created", "start", "finish", "first_token", "token_times", "record_times", "pending_token", "offloaded",
        "in_flight_tokens",
    )

    def __init__(self, idx: int, prompt: list[int], max_new: int, depths: list[int], eos: set[int], stops, rec: bool):
        self.idx = idx
        self.request_id = f"request-{idx}"
        self.prompt = prompt
        self.max_new = max_new
        self.depths = depths
        self.cursor = 0
        self.status = RequestStatus.PENDING
        self.remaining = list(prompt)
        self.chunk: list[int] = []
        self.position = 0
        self.allocated = 0
        self.generated = 0
        self.slot = -1
        self.log_base = 0
        self.exit_depths: list[int] = []
        self.eos = eos
        self.stops = stops
        self.created = time.perf_counter()
        self.start = -1.0
        self.finish = -1.0
        self.first_token = -1.0
        self.token_times: list[float] = []
        self.record_times = rec
        self.pending_token = -1
        self.offloaded = False
        self.in_flight_tokens = 0  # sampled tokens launched but not yet consumed (CB pipelining)

    def next_depth(self) -> int | None:
        if not self.depths:
            return None
        if self.cursor >= len(self.depths):
            raise RuntimeError(f"Request {self.request_id}: synthetic exit-depth schedule exhausted")
        d = self.depths[self.cursor]
        self.cursor += 1
        return d


class _Item:
    __slots__ = ("req", "position", "step", "depth", "hidden", "token", "pending")

    def __init__(self, req: _Req, position: int, depth: int | None, hidden: int, token: int):
        self.req = req
        self.position = position
        self.step = 0
        self.depth = depth
        self.hidden = hidden
        self.token = token
        # Delayed gate consumption: the live decision of the item's previous step, as
        # (staged launch decisions, row), consumed at the routing after the following launch.
        self.pending: tuple[_StagedDecisions, int] | None = None


class _StagedDecisions:
    """One recurrent launch's live exit decisions, copied to pinned host memory on the engine
    stream without waiting (``stage_delayed_exit_signals``, ``continuous_api.py:1117-1122``).
    The host reads them one launch later, by which time the copy has normally landed."""

    def __init__(self, values: torch.Tensor, stream: torch.cuda.Stream, decide) -> None:
        self.host = torch.empty(values.shape, dtype=values.dtype, pin_memory=True)
        with torch.cuda.stream(stream):
            self.host.copy_(values, non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(stream)
        self.decide = decide  # (row, host values) -> bool
        self._vals: list | None = None

    def get(self, row: int) -> bool:
        if self._vals is None:
            self.event.synchronize()
            self._vals = self.host.tolist()
        return self.decide(row, self._vals)


class ContinuousDepthBatchingEngine:
    """Continuous depth batching over the B200 CUDA library (one engine per GPU)."""

    def __init__(
        self, model, cdb_config: ContinuousDepthBatchingConfig, runner: OuroRunner, shape: OuroShape | HuginnShape
    ):
        self.model = model
        self.cdb_config = cdb_config
        self.runner = runner
        self.shape = shape
        self.last_stats = ContinuousDepthBatchingStats()
        self.record_trace = False
        self.launch_trace: list[dict] = []
        self.lm_logits: list[tuple[str, torch.Tensor]] = []
        self.keep_logits = False

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_model(
        cls,
        model,
        cdb_config: ContinuousDepthBatchingConfig,
        *,
        dtype: torch.dtype | None = None,
        model_adapter=None,
        device: torch.device | str | None = None,
        fused_lm_head: bool = True,
    ) -> ContinuousDepthBatchingEngine:
        """Build an engine for an Ouro or Huginn causal LM given by its parameters (reference names).

        ``model`` is the reference's ``OuroForCausalLM`` / ``HuginnForCausalLM`` or any module with
        its state-dict layout (e.g. :class:`~.ouro.OuroForCausalLM`,
        :class:`~.huginn.HuginnForCausalLM`); ``config.model_type`` picks the family, as
        ``resolve_cdb_model_adapter`` does (``model_adapter.py:105-122``). Weights are packed to bf16 on ``device``
        (default: the model's device if CUDA, else ``cuda``). ``dtype`` other than bf16 is rejected:
        the kernels compute in bf16 with fp32 accumulation; every projection runs on the library's
        tcgen05 GEMM (SwiGLU fused into the gate/up projection). ``fused_lm_head`` runs the LM head
        and the greedy argmax as one tcgen05 GEMM with no logits in HBM (``cdb_lm_head_argmax``)
        instead of a GEMM followed by ``cdb_argmax``.
        """

        # The reference's plugin seam: no adapter (inferred from the model), the reference's Ouro /
        # Huginn adapters, or this package's; see model_adapter.py for what is rejected and why.
        adapter = resolve_cdb_model_adapter(model, model_adapter)
        if dtype not in (None, torch.bfloat16):
            raise NotImplementedError(f"the B200 kernels run bf16; got dtype={dtype}")
        config = getattr(model, "config", None)
        model_type = adapter.family
        cfg = cdb_config.get_resolved()
        # ``resolve_max_num_seqs`` (``scheduler_base.py:49-66``, applied at ``continuous_api.py:328``):
        # a decode launch writes one row per resident request into buffers sized by the prefill
        # token budget, so the resident cap is at most that budget
        cfg.max_num_seqs = min(cfg.max_num_seqs, cfg.max_num_batched_tokens)
        if model_type == "huginn":
            hshape = HuginnShape.from_config(config)
            shape = HuginnShape(**{**hshape.__dict__, "total_recurrent_steps": cfg.max_recurrent_steps})
            runner_cls = HuginnRunner
        else:
            oshape = OuroShape.from_config(config)
            shape = OuroShape(**{**oshape.__dict__, "total_ut_steps": cfg.max_recurrent_steps})
            runner_cls = OuroRunner
        # The adapters' exit specs: Ouro's gate is a cumulative hazard, Huginn's a direct threshold
        # on the latent difference (adapters/ouro.py:293-299, adapters/huginn.py:63-66).
        validate_exit_threshold(cfg.exit_threshold, "direct" if model_type == "huginn" else "hazard")
        if shape.num_key_value_heads != shape.num_attention_heads:
            raise NotImplementedError("the paged decode kernel serves MHA (num_key_value_heads == num_attention_heads)")
        if device is None:
            p = next(model.parameters())
            device = p.device if p.device.type == "cuda" else torch.device("cuda")
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if cfg.num_blocks is None:
            cfg.num_blocks = _auto_num_blocks(shape, cfg, device)
        state = {k: v for k, v in model.state_dict().items()}
        runner = runner_cls(
            shape,
            state,
            device=device,
            kv_policy=cfg.kv_policy,
            kv_slots_per_layer=cfg.kv_slots_per_layer,
            num_blocks=cfg.num_blocks,
            block_size=cfg.block_size,
            max_model_len=cfg.max_model_len,
            max_num_seqs=cfg.max_num_seqs,
            max_num_batched_tokens=cfg.max_num_batched_tokens,
            use_cuda_graph=cfg.use_cuda_graph,
            fused_lm_head=fused_lm_head,
        )
        if cfg.kv_pressure_mode == "offload" and cfg.cpu_offload_space:
            # ``OffloadingManager._compute_num_cpu_blocks`` (``offloading_manager.py:134-144``)
            runner.pool.attach_host_pool(int(cfg.cpu_offload_space * 1024**3) // runner.pool.block_bytes)
        adapter.configure_recurrent_steps(cfg.max_recurrent_steps)
        adapter.configure_kv_policy(cfg.kv_policy, cfg.kv_slots_per_layer)
        eng = cls(model, cfg, runner, shape)
        eng.model_adapter = adapter
        return eng

    # ------------------------------------------------------------------ public API
    @torch.no_grad()
    def generate_batch(
        self,
        input_ids: list[list[int]],
        *,
        max_new_tokens: int | list[int],
        eos_token_id: int | list[int] | None,
        stop_sequences: list[list[int]] | None = None,
        warmup: bool = True,
        model_kwargs: dict | None = None,
        exit_depths: list[list[int]] | None = None,
        arrival_offsets_s: list[float] | None = None,
        record_token_times: bool = False,
        record_queue_samples: bool = False,
        forced_tokens: list[list[int]] | None = None,
    ) -> list[GenerationOutput]:
        """Generate from tokenized prompts with decode-time CDB (see the module docstring).

        ``forced_tokens`` (parity harness) continues each request with the given tokens instead of
        its own samples; the engine still records its own argmax at every position.
        """

        del warmup, record_queue_samples
        cfg = self.cdb_config
        caps = self._validate(input_ids, max_new_tokens, exit_depths, model_kwargs)
        eos = set()
        if eos_token_id is not None:
            for t in [eos_token_id] if isinstance(eos_token_id, int) else eos_token_id:
                if t >= 0:
                    eos.add(int(t))
        stops = [list(s) for s in stop_sequences] if stop_sequences else []
        self._content_finish = bool(eos or stops)
        self._forced = forced_tokens
        self._gate_live = cfg.exit_threshold is not None and (
            model_kwargs is None or model_kwargs.get("use_early_exit_gate", True)
        )
        # The reference's default timing (use_async_batching with delay_gate_consumption): a step's
        # exit decision is applied at the routing after the item's next launch
        # (ExitPolicy.delayed_transport_enabled, exit_policy.py:76-80).
        self._delayed = bool(cfg.use_async_batching and cfg.delay_gate_consumption)
        reqs: list[_Req] = []
        base = 0
        for i, (p, m) in enumerate(zip(input_ids, caps, strict=True)):
            r = _Req(i, list(p), m, list(exit_depths[i]) if exit_depths else [], eos, stops, record_token_times)
            r.log_base = base
            base += m
            reqs.append(r)
        self.runner.reset(max(base, 1))
        self._reset_state()
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
        if cfg.refill:
            self._refill_loop(arrivals)
        else:
            self._no_refill_loop(arrivals)
        tokens = self.runner.read_tokens(base) if base else []
        self.runner.check_status()
        outs = []
        for r in reqs:
            gen = tokens[r.log_base : r.log_base + r.generated]
            outs.append(
                GenerationOutput(
                    request_id=r.request_id,
                    prompt_ids=r.prompt,
                    generated_tokens=gen,
                    status=r.status,
                    created_time=r.created,
                    lifespan=(r.start, r.finish),
                    first_token_time=r.first_token,
                    token_ready_times=r.token_times,
                    exit_depths=r.exit_depths,
                )
            )
        st = self.last_stats
        st.generated_tokens = sum(len(o.generated_tokens) for o in outs)
        st.scheduler_refills = self.refills
        st.max_depth_queue_size = self.max_queue
        st.recurrent_graph_hits = self.runner.stats.recurrent_graph_hits
        st.recurrent_graph_captures = self.runner.stats.recurrent_graph_captures
        st.fixed_depth_recurrent_steps = st.coda_tokens * cfg.max_recurrent_steps
        st.kv_peak_blocks = self.runner.pool.pool.peak
        return outs

    # ------------------------------------------------------------------ state
    def _reset_state(self) -> None:
        cfg = self.cdb_config
        self.last_stats = ContinuousDepthBatchingStats()
        self.launch_trace = []
        self.lm_logits = []
        self.waiting: OrderedDict[int, _Req] = OrderedDict()
        self.active: OrderedDict[int, _Req] = OrderedDict()
        self.in_flight: set[int] = set()
        self.ready: deque[_Item] = deque()
        self.coda_q: deque[_Item] = deque()
        self.backlog: list[tuple[_Item, int]] = []
        self.stalled: OrderedDict[int, _Req] = OrderedDict()
        self.block_new = False
        self.num_host_blocks = self.runner.pool.num_host_blocks if cfg.kv_pressure_mode == "offload" else 0
        self.host_free: deque[int] = deque(range(self.num_host_blocks))
        self.host_tables: dict[int, list[int]] = {}
        self.refills = 0
        self.max_queue = 0
        seqs = min(cfg.max_num_seqs, cfg.max_num_batched_tokens)  # as from_model resolves it
        self.free_slots = list(range(seqs - 1, -1, -1))
        self.free_hidden = list(range(self.runner.bank_slots - 1, -1, -1))
        self.pool = self.runner.pool.pool
        self.max_num_seqs = seqs
        self.min_free = max(1, seqs // 8) if cfg.min_free_slots is None else min(cfg.min_free_slots, seqs)
        self.safety = 0.0 if cfg.kv_pressure_mode == "reserve" else cfg.safety_margin
        self.width = cfg.decode_block_table_width()
        self.slots = cfg.kv_slots_per_layer
        self.steps = cfg.max_recurrent_steps

    def _slot_of_step(self, step: int) -> int:
        return kv_slot_for_step(step, policy=self.cdb_config.kv_policy, slots_per_layer=self.slots)

    # ------------------------------------------------------------------ block allocation
    def _alloc(self, r: _Req, n: int) -> bool:
        if n <= 0:
            return True
        if not self.pool.allocate(r.idx, r.slot, n):
            return False
        r.allocated += n
        return True

    def _alloc_if_needed(self, r: _Req, n_next: int) -> bool:
        bs = self.cdb_config.block_size
        if r.allocated * bs - r.position < n_next:
            return self._alloc(r, -(-(r.position + n_next) // bs) - r.allocated)
        return True

    def _alloc_one_decode(self, r: _Req) -> bool:
        bs = self.cdb_config.block_size
        if r.allocated * bs - r.position >= 1 and r.allocated > 0:
            return True
        return self._alloc(r, -(-(r.position + 1) // bs) - r.allocated)

    # ------------------------------------------------------------------ request lifecycle
    def _retire(self, r: _Req) -> None:
        r.status = RequestStatus.FINISHED
        r.finish = time.perf_counter()
        self.pool.release(r.idx)
        self.active.pop(r.idx, None)
        self.in_flight.discard(r.idx)
        self.stalled.pop(r.idx, None)
        self.free_slots.append(r.slot)
        # a finish frees blocks, so admission resumes (``continuous_api.py:1436-1448``)
        self.block_new = False

    def _record_token(self, r: _Req) -> bool:
        """Count one sampled token; True when the request is finished (length, EOS or stop)."""

        now = time.perf_counter()
        if r.first_token < 0:
            r.first_token = now
        if r.record_times:
            r.token_times.append(now)
        r.generated += 1
        if r.generated >= r.max_new:
            return True
        if self._content_finish:
            tok = r.pending_token
            if tok in r.eos:
                return True
            if r.stops:
                gen = self._host_tokens(r)
                for s in r.stops:
                    if s and len(gen) >= len(s) and gen[-len(s):] == s:
                        return True
        return False

    def _host_tokens(self, r: _Req) -> list[int]:
        """The tokens the request has continued with so far (the forced ones under teacher forcing)."""

        if self._forced is not None:
            return list(self._forced[r.idx][: r.generated])
        return self.runner.token_log[r.log_base : r.log_base + r.generated].cpu().tolist()

    def _next_token_id(self, r: _Req) -> int:
        """Host-known input id of the request's next decode token, or -1 (device token table)."""

        if self._forced is not None:
            return int(self._forced[r.idx][r.generated - 1])
        return -1

    def _stage_decode(self, r: _Req) -> _Item | None:
        """``_stage_decode_token`` (``continuous_api.py:1584-1610``): the request's next decode
        item, or None when no KV block is free for its token: the request then stalls at a token
        boundary, is retried each tick and is preempted only when nothing else can run."""

        if not self._alloc_one_decode(r):
            mode = self.cdb_config.kv_pressure_mode
            if mode == "none":
                raise CacheFullError(
                    f"KV cache full staging a decode block for request {r.request_id} and "
                    "kv_pressure_mode='none' does no preemption. Increase num_blocks, reduce load, or select "
                    "kv_pressure_mode='reserve'/'recompute'."
                )
            if mode == "reserve":
                raise CacheFullError(
                    f"Reserve admission over-committed the KV cache: request {r.request_id} could not "
                    "allocate a decode block. This is a bug in reservation accounting."
                )
            self.stalled[r.idx] = r
            return None
        self.stalled.pop(r.idx, None)
        hidden = self.free_hidden.pop()
        return _Item(r, r.position, r.next_depth(), hidden, self._next_token_id(r))

    def _restage_stalled(self) -> list[_Item]:
        """``_restage_stalled_decoders`` (``continuous_api.py:1612-1623``): retry the stalled
        requests in stall order; every one needs one new block, so the first failure ends the scan."""

        items = []
        for r in list(self.stalled.values()):
            it = self._stage_decode(r)
            if it is None:
                break
            items.append(it)
        return items

    def _preempt_stalled(self) -> None:
        """``_preempt_stalled_decoder`` (``continuous_api.py:1625-1652``) and
        ``OffloadingManager._preempt`` (``offloading_manager.py:180-214``).

        The victim is the stalled request with the fewest cached tokens, ties going to the latest
        staller. Under ``offload`` its blocks are first copied to the host pool if they fit there;
        it then waits, still decoding, until :meth:`_restore_offloaded` brings it back. Otherwise
        (``recompute``, or a full host pool) it is soft-reset (``create_equivalent_initial_request``,
        ``requests.py:290-315``): its generated tokens are appended to its prompt for a full-depth
        re-prefill, and the depth its pending token would have replayed is skipped. Either way its
        blocks and block-table row are released, it re-enters the waiting queue at the back, and no
        new prompt is admitted until a request finishes."""

        if len(self.active) <= 1:
            rid = next(iter(self.stalled.values())).request_id
            raise CacheFullError(
                f"A single request's KV cache does not fit: request {rid} could not allocate a decode block "
                "and no other request can be preempted (increase num_blocks or reduce max_model_len)."
            )
        victim = min(reversed(list(self.stalled)), key=lambda i: self.stalled[i].position)
        r = self.stalled.pop(victim)
        offloaded = self._offload(r)
        if not offloaded:
            if self.num_host_blocks and copies_exit_kv(self.cdb_config.kv_policy):
                raise RuntimeError(
                    f"CPU swap pool cannot hold request {r.request_id} ({r.allocated} blocks needed, "
                    f"{len(self.host_free)} free) and the soft-reset fallback is disabled: re-prefilling at "
                    "full depth would replace the KV this cache policy rewrote on early exit. Increase "
                    "cpu_offload_space or reduce load."
                )
            if self._forced is None:
                self.last_stats.host_syncs += 1
                self.runner.stream.synchronize()
            generated = self._host_tokens(r)
        self.pool.release(r.idx)
        self.active.pop(r.idx, None)
        self.in_flight.discard(r.idx)
        self.waiting.pop(r.idx, None)
        self.free_slots.append(r.slot)
        r.slot = -1
        r.allocated = 0
        if offloaded:
            # ``prepare_for_offload_requeue`` (``requests.py:275-288``): still decoding, with its
            # position and pending token; only the blocks are given up
            self.last_stats.offload_preemptions += 1
        else:
            r.remaining = list(r.prompt) + generated
            r.chunk = []
            r.position = 0
            r.status = RequestStatus.PENDING
            r.cursor += 1
            self.last_stats.recompute_preemptions += 1
        self.waiting[r.idx] = r
        self.block_new = True

    def _offload(self, r: _Req) -> bool:
        """``OffloadingManager._offload_to_cpu`` (``offloading_manager.py:269-306``): queue the copy of
        every block of ``r`` into free host blocks; False when the host pool has too few."""

        if not self.num_host_blocks:
            return False
        blocks = self.pool.tables.get(r.idx, [])
        if not blocks or len(self.host_free) < len(blocks):
            return False
        host = [self.host_free.popleft() for _ in blocks]
        self.runner.pool.host_copy(blocks, host, True, self.runner.stream)
        self.host_tables[r.idx] = host
        r.offloaded = True
        return True

    def _restore_offloaded(self) -> list[_Req]:
        """``admit_offloaded_restores`` (``scheduler_base.py:434-460``) and
        ``restore_scheduled_requests`` (``offloading_manager.py:216-267``).

        Offloaded waiting requests return to the active set in queue order, ahead of fresh prompts,
        while a resident slot and blocks for their cached tokens plus the pending one are free (the
        first that does not fit ends the scan; nothing returns while admission is held). Each gets a
        block-table row, its host blocks are copied into its new blocks, and its pending token is
        rebound to the new row."""

        if self.block_new or not self.num_host_blocks:
            return []
        admitted = []
        for i in list(self.waiting):
            r = self.waiting[i]
            if not r.offloaded:
                continue
            if max(0, self.max_num_seqs - len(self.active)) == 0:
                break
            r.slot = self.free_slots.pop()
            if not self._alloc_if_needed(r, 1):
                self.free_slots.append(r.slot)
                r.slot = -1
                break
            self.active[i] = r
            del self.waiting[i]
            admitted.append(r)
        for r in admitted:
            host = self.host_tables.pop(r.idx)
            self.runner.pool.host_copy(self.pool.tables[r.idx][: len(host)], host, False, self.runner.stream)
            self.host_free.extend(host)
            if r.generated:  # a request offloaded mid-prompt has no sampled token to carry
                self.runner.rebind_token(r.slot, r.log_base + r.generated - 1)
            r.offloaded = False
            self.last_stats.restores += 1
        return admitted

    def _prelude(self, items: list[_Item]) -> None:
        if items:
            self.runner.prelude(
                [it.token for it in items],
                [it.req.slot for it in items],
                [it.hidden for it in items],
                positions=[it.position for it in items],
            )

    def _enqueue(self, item: _Item, front: bool = False) -> None:
        self.in_flight.add(item.req.idx)
        if item.step == 0 and self.ready:
            self.refills += 1
        if front:
            self.ready.appendleft(item)
        else:
            self.ready.append(item)
        if len(self.ready) > self.max_queue:
            self.max_queue = len(self.ready)

    def _enqueue_front(self, items: list[_Item]) -> None:
        for it in reversed(items):
            self._enqueue(it, front=True)

    # ------------------------------------------------------------------ admission
    def _has_pending(self) -> bool:
        return bool(self.coda_q or self.ready or self.active or self.waiting)

    def _has_decode_work(self) -> bool:
        return any(r.status == RequestStatus.DECODING for r in self.active.values())

    def _admit_prefill(self) -> bool:
        return not self._has_decode_work() or self.pool.num_free > self.safety * self.cdb_config.num_blocks

    def _reserved_peak(self, r: _Req) -> int:
        total = min(len(r.prompt) + r.max_new, self.cdb_config.max_model_len)
        return -(-total // self.cdb_config.block_size)

    def _prefill_candidates(self) -> list[_Req]:
        prefilling = [r for r in self.active.values() if r.status == RequestStatus.PREFILLING and r.idx not in self.in_flight]
        free_res = max(0, self.max_num_seqs - len(self.active))
        admissible = []
        for key in self.waiting:
            # after a preemption no new prompt is admitted until a request finishes
            if self.block_new or len(admissible) >= free_res:
                break
            if not self.waiting[key].offloaded:  # offloaded requests return through the restore path
                admissible.append(self.waiting[key])
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

    def _schedule_prefill(self):
        """``CDBScheduler.schedule_prefill_batch`` (``scheduler.py:190-320``)."""

        cands = self._prefill_candidates()
        if not cands:
            return None
        cfg = self.cdb_config
        bs = cfg.block_size
        token_budget = cfg.max_num_batched_tokens
        cache_budget = cfg.num_blocks * bs
        margin = self.safety * cfg.num_blocks
        fast = True
        out = []
        for r in cands:
            n_free = self.pool.num_free
            if n_free < margin and out:
                break
            toks = r.remaining
            qlen = min(len(toks), token_budget)
            if qlen == 0:
                continue
            eligible = qlen == 1 and r.position < self.width * bs
            read_needed = r.position
            if not (fast and eligible) and cache_budget < read_needed:
                continue
            if r.status == RequestStatus.PENDING and r.slot < 0:
                # A resident slot (block-table row) is bound at admission; undone if allocation fails.
                r.slot = self.free_slots.pop()
                bound_here = True
            else:
                bound_here = False
            if not self._alloc_if_needed(r, qlen):
                if bound_here:
                    self.free_slots.append(r.slot)
                    r.slot = -1
                if n_free == 0 and r.idx in self.waiting:
                    break
                continue
            past = r.position
            if len(toks) <= qlen:
                if r.status == RequestStatus.PENDING:
                    self.active[r.idx] = r
                    if r.start < 0:
                        r.start = time.perf_counter()
                r.chunk = toks
                r.remaining = []
                r.status = RequestStatus.DECODING
            else:
                if r.status == RequestStatus.PENDING:
                    self.active[r.idx] = r
                    if r.start < 0:
                        r.start = time.perf_counter()
                    r.status = RequestStatus.PREFILLING
                r.remaining = toks[qlen:]
                r.chunk = toks[:qlen]
            self.in_flight.add(r.idx)
            qlen = len(r.chunk)
            fast = fast and qlen == 1 and r.position < self.width * bs
            token_budget -= qlen
            cache_budget -= read_needed
            out.append((r, past, qlen, not r.remaining))
            self.waiting.pop(r.idx, None)
            if token_budget == 0 or (cache_budget <= 0 and not fast):
                break
        return out or None

    # ------------------------------------------------------------------ launches
    def _run_prefill(self, batch) -> list[_Req]:
        st = self.last_stats
        st.prefill_batches += 1
        st.prefill_requests += len(batch)
        ids, slots, pos, logit_rows, log_rows, req_slots, sampled = [], [], [], [], [], [], []
        for r, past, qlen, has in batch:
            ids.extend(r.chunk)
            slots.extend([r.slot] * qlen)
            pos.extend(range(past, past + qlen))
            r.position = past + qlen
            if has:
                logit_rows.append(len(ids) - 1)
                log_rows.append(r.log_base + r.generated)
                req_slots.append(r.slot)
                sampled.append(r)
        st.prefill_tokens += len(ids)
        st.prefill_recurrent_steps += len(ids) * self.steps
        if self.record_trace:
            bs = self.cdb_config.block_size
            self.launch_trace.append(
                {
                    "kind": "prefill",
                    "items": [[r.idx, past, qlen, int(has)] for r, past, qlen, has in batch],
                    "blocks": [list(self.pool.tables[r.idx][: -(-r.position // bs)]) for r, *_ in batch],
                }
            )
        logits = self.runner.prefill(
            ids, slots, pos, logit_rows, log_rows, req_slots, [self._slot_of_step(s) for s in range(self.steps)],
            keep_logits=self.keep_logits,
        )
        if logits is not None:
            self.lm_logits.append(("prefill", logits))
        st.prefill_coda_tokens += len(sampled)
        if self._content_finish and sampled:
            self._sync_tokens(sampled)
        return sampled

    def _sync_tokens(self, reqs: list[_Req]) -> None:
        """Host copies of the tokens about to be recorded, for the EOS / stop-sequence checks. Under
        teacher forcing the sequence continues with the forced token, so that one decides."""

        if self._forced is not None:
            for r in reqs:
                r.pending_token = int(self._forced[r.idx][r.generated])
            return
        self.last_stats.host_syncs += 1
        self.runner.stream.synchronize()
        for r in reqs:
            r.pending_token = int(self.runner.token_log[r.log_base + r.generated].item())

    def _run_recurrent(self, items: list[_Item]) -> list[bool] | None:
        st = self.last_stats
        kv_slot = self._slot_of_step(items[0].step)
        if self.record_trace:
            bs = self.cdb_config.block_size
            self.launch_trace.append(
                {
                    "kind": "recurrent",
                    "items": [[it.req.idx, it.position, it.step] for it in items],
                    "blocks": [list(self.pool.tables[it.req.idx][: -(-(it.position + 1) // bs)]) for it in items],
                }
            )
        self.runner.recurrent(
            [it.req.slot for it in items], [it.position for it in items], [it.hidden for it in items], kv_slot,
            self._gate_live, steps=[it.step for it in items],
        )
        st.recurrent_batches += 1
        st.recurrent_steps += len(items)
        st.mixed_recurrent_batches += 1
        depths = Counter(it.step for it in items)
        st.max_mixed_depths_per_batch = max(st.max_mixed_depths_per_batch, len(depths))
        for k, v in depths.items():
            st.mixed_recurrent_depth_histogram[k] += v
        if not self._gate_live:
            return None
        if self._delayed:
            return self._stage_live_decisions(items)
        return self._live_decisions(items)

    def _live_flags(self, items: list[_Item]) -> torch.Tensor:
        """This launch's live exit decisions on device (``cdb_exit_gate_route``, synchronous rule):
        Ouro's cumulative hazard of the gate logit, Huginn's direct threshold on the latent
        difference. Policy state (fp64 cdf/survival) lives per hidden-bank slot on the device."""

        r = self.runner
        cfg = self.cdb_config
        n = len(items)
        meta = r.upload([[it.hidden for it in items], [it.step for it in items], [int(it.step == 0) for it in items]])
        meta = meta.view(3, n)
        if not hasattr(self, "_route"):
            m = cfg.max_num_seqs
            self._route = (
                torch.zeros(r.bank_slots, dtype=torch.float64, device=r.device),
                torch.ones(r.bank_slots, dtype=torch.float64, device=r.device),
                torch.zeros(m, dtype=torch.int8, device=r.device),
                torch.zeros(2, m, dtype=torch.int32, device=r.device),
                torch.zeros(2, dtype=torch.int32, device=r.device),
            )
        cdf, surv, flags, lists, counts = self._route
        policy = 2 if isinstance(self.shape, HuginnShape) else 1
        from . import _lib

        with torch.cuda.stream(r.stream):
            reset = meta[2].to(torch.int8)
            _lib.call(
                "cdb_exit_gate_route", _lib.ptr(r.gate_out), r.gate_out.stride(0), _lib.ptr(meta[0]),
                _lib.ptr(meta[1]), None, _lib.ptr(reset), _lib.ptr(cdf), _lib.ptr(surv), None, n, policy, 0,
                cfg.min_recurrent_steps, self.steps, float(cfg.exit_threshold), _lib.ptr(flags), _lib.ptr(lists[0]),
                _lib.ptr(lists[1]), _lib.ptr(counts), r.stream.cuda_stream,
            )
        return flags[:n]

    def _stage_live_decisions(self, items: list[_Item]) -> _StagedDecisions:
        """Delayed consumption: decide this launch's signals on device now (the per-token policy
        state advances in step order, as the reference's deferred ``should_exit`` calls advance
        it) and stage the flags to the host; routing reads them after the next launch."""

        return _StagedDecisions(self._live_flags(items), self.runner.stream, lambda i, v: bool(v[i]))

    def _live_decisions(self, items: list[_Item]) -> list[bool]:
        """Live exit decisions (``ExitPolicy.should_exit``, ``exit_policy.py:150-169``) decided on
        device and read back with one synchronisation (the synchronous timing)."""

        self.last_stats.host_syncs += 1
        with torch.cuda.stream(self.runner.stream):
            host = self._live_flags(items).cpu()
        return [bool(x) for x in host.tolist()]

    def _should_exit(self, it: _Item, step: int, live, i: int) -> bool:
        if self._delayed:
            # Delayed consumption (continuous_api.py:1124-1160, 1250-1280): route on the decision
            # of the item's previous step; this step's live decision is kept for the next routing.
            pend, it.pending = it.pending, None
            if isinstance(live, _StagedDecisions):
                it.pending = (live, i)
            if step == self.steps - 1:
                return True
            if it.depth is not None:
                return step >= it.depth + 1  # the pending replay step (step - 1) reached the depth
            return pend is not None and pend[0].get(pend[1])
        if step == self.steps - 1:
            return True
        if it.depth is not None:
            return step >= it.depth
        if live is None:
            return False
        return live[i]

    def _record_exit(self, it: _Item, step: int) -> None:
        it.req.exit_depths.append(step)
        self.last_stats.exit_depth_histogram[step] += 1
        if copies_exit_kv(self.cdb_config.kv_policy) and step < self.steps - 1:
            self.backlog.append((it, step))

    def _flush_exit_copies(self) -> None:
        if not self.backlog:
            return
        backlog, self.backlog = self.backlog, []
        by_step: dict[int, list[_Item]] = {}
        for it, step in backlog:
            by_step.setdefault(step, []).append(it)
        bs = self.cdb_config.block_size
        layout = self.runner.layout
        for step, items in sorted(by_step.items()):
            rows = [self.pool.tables[it.req.idx][it.position // bs] * bs + it.position % bs for it in items]
            pairs = [(src_layer, t) for src_layer, targets in layout.exit_copy_layer_groups(step) for t in targets]
            self.runner.exit_kv_copy(rows, pairs)
            self.last_stats.exit_kv_copies += len(rows)

    def _run_coda(self, items: list[_Item]) -> None:
        st = self.last_stats
        if self.record_trace:
            self.launch_trace.append({"kind": "coda", "items": [[it.req.idx, it.position, it.step] for it in items]})
        logits = self.runner.coda(
            [it.hidden for it in items],
            [it.req.log_base + it.req.generated for it in items],
            [it.req.slot for it in items],
            keep_logits=self.keep_logits,
            positions=[it.position for it in items],
        )
        if logits is not None:
            self.lm_logits.append(("coda", logits))
        st.coda_batches += 1
        st.coda_tokens += len(items)
        if self._content_finish:
            self._sync_tokens([it.req for it in items])

    # ------------------------------------------------------------------ consumption
    def _consume_prefill(self, sampled: list[_Req], stage: bool) -> None:
        new_items = []
        for r in sampled:
            if r.status == RequestStatus.FINISHED:
                continue
            if self._record_token(r):
                self._retire(r)
                continue
            if stage and (it := self._stage_decode(r)) is not None:
                new_items.append(it)
        self._prelude(new_items)
        for it in new_items:
            self._enqueue(it)

    def _consume_coda(self, items: list[_Item], stage: bool) -> None:
        new_items = []
        for it in items:
            r = it.req
            self.free_hidden.append(it.hidden)
            if r.status == RequestStatus.FINISHED:
                continue
            r.position += 1
            if self._record_token(r):
                self._retire(r)
                continue
            if stage and (nxt := self._stage_decode(r)) is not None:
                new_items.append(nxt)
        self._prelude(new_items)
        self._enqueue_front(new_items)

    def _release_arrivals(self, arrivals) -> None:
        if not arrivals:
            return
        self.runner.stream.synchronize()
        now = time.perf_counter() - self._t0
        while arrivals and arrivals[0][0] <= now:
            _, i = arrivals.popleft()
            self.waiting[i] = self._reqs[i]

    def _wait_next_arrival(self, arrivals) -> None:
        delay = arrivals[0][0] - (time.perf_counter() - self._t0)
        if delay > 0:
            time.sleep(delay)

    # ------------------------------------------------------------------ loops
    def _refill_loop(self, arrivals) -> None:
        cfg = self.cdb_config
        pending_prefill: list[list[_Req]] = []
        pending_coda: list[list[_Item]] = []
        while arrivals or self._has_pending() or pending_prefill or pending_coda:
            self._release_arrivals(arrivals)
            for sampled in pending_prefill:
                self._consume_prefill(sampled, stage=True)
            pending_prefill = []
            for items in pending_coda:
                self._consume_coda(items, stage=True)
            pending_coda = []
            if not self._has_pending():
                if arrivals:
                    self._wait_next_arrival(arrivals)
                continue
            # restored requests, then decode tokens that found no KV block last tick, go first, at
            # the queue head
            resumed = [it for r in self._restore_offloaded() if (it := self._stage_decode(r)) is not None]
            if self.stalled:
                resumed += self._restage_stalled()
            if resumed:
                self._prelude(resumed)
                self._enqueue_front(resumed)
            self.last_stats.scheduler_ticks += 1
            if len(self.coda_q) >= cfg.min_coda_batch_size:
                batch = [self.coda_q.popleft() for _ in range(min(self.max_num_seqs, len(self.coda_q)))]
                self._run_coda(batch)
                pending_coda.append(batch)
                continue
            if self._admit_prefill():
                pb = self._schedule_prefill()
                if pb is not None:
                    pending_prefill.append(self._run_prefill(pb))
                    for r, _past, _q, has in pb:
                        if not has:
                            self.in_flight.discard(r.idx)
                    continue
            items = self._pop_recurrent()
            if items:
                live = self._run_recurrent(items)
                refills = []
                for i, it in enumerate(items):
                    step = it.step
                    self.last_stats.recurrent_step_histogram[step] += 1
                    if self._should_exit(it, step, live, i):
                        self._record_exit(it, step)
                        self.in_flight.add(it.req.idx)
                        self.coda_q.append(it)
                    else:
                        it.step = step + 1
                        refills.append(it)
                self._enqueue_front(refills)
                self._flush_exit_copies()
                continue
            if self.coda_q:
                batch = [self.coda_q.popleft() for _ in range(min(self.max_num_seqs, len(self.coda_q)))]
                self._run_coda(batch)
                pending_coda.append(batch)
                continue
            if self.stalled:
                self._preempt_stalled()
                continue
            if arrivals:
                self._wait_next_arrival(arrivals)
                continue
            raise CacheFullError(
                "The CDB scheduler could place no work: the KV cache cannot admit the next prompt "
                "(increase num_blocks or reduce max_model_len)"
            )

    def _pop_recurrent(self) -> list[_Item]:
        n = min(self.max_num_seqs, len(self.ready))
        if n == 0:
            return []
        first = self.ready.popleft()
        batch = [first]
        if self.slots > 1:
            target = self._slot_of_step(first.step)
            deferred: deque[_Item] = deque()
            while self.ready and len(batch) < n:
                it = self.ready.popleft()
                if self._slot_of_step(it.step) == target:
                    batch.append(it)
                else:
                    deferred.append(it)
            deferred.extend(self.ready)
            self.ready = deferred
        else:
            while self.ready and len(batch) < n:
                batch.append(self.ready.popleft())
        return batch

    def _carry_successor(self, r: _Req, token: int | None = None) -> _Item | None:
        """Stage the next decode token of ``r`` ahead of its wave (eager re-entry,
        ``_select_eager_reentries``, ``continuous_api.py:1304-1327``): allocate its KV block now;
        None when no block is free (a later wave's cohort scan picks it up). ``token`` is the input
        id when the host knows it (-1: the request's device token)."""

        if not self._alloc_one_decode(r):
            return None
        tok = self._next_token_id(r) if token is None else token
        return _Item(r, r.position, r.next_depth(), self.free_hidden.pop(), tok)

    def _would_finish(self, r: _Req) -> bool:
        """Whether recording the request's pending token will finish it (length, EOS, stop)."""

        if r.generated + 1 >= r.max_new:
            return True
        if not self._content_finish:
            return False
        tok = r.pending_token
        if tok in r.eos:
            return True
        gen = self._host_tokens(r) + [tok]
        return any(s and len(gen) >= len(s) and gen[-len(s):] == s for s in r.stops)

    def _consume_carried_coda(self, pending: list[_Req]) -> None:
        """``_consume_no_refill_coda``: the boundary coda's tokens are recorded, and finished
        requests retired (their blocks freed), once the next wave's first launch is queued."""

        for r in pending:
            if r.status == RequestStatus.FINISHED:
                continue
            if self._record_token(r):
                self._retire(r)

    def _carry_after_prefill(self, sampled: list[_Req], budget: int) -> list[_Item]:
        """Delayed no-refill path: each prefilled request's first decode token is carried into
        this iteration's wave, up to ``budget`` items (``continuous_api.py:763-781``)."""

        carried = []
        for r in sampled:
            if r.status == RequestStatus.FINISHED:
                continue
            if self._record_token(r):
                self._retire(r)
                continue
            if len(carried) < budget and (it := self._carry_successor(r)) is not None:
                carried.append(it)
        return carried

    def _carry_after_coda(self, items: list[_Item]) -> tuple[list[_Item], list[_Req]]:
        """Delayed no-refill path: the wave's exiters' successors, staged at the boundary coda in
        exit order, lead the next wave (``continuous_api.py:929-940``). The coda's tokens are
        recorded during that wave (:meth:`_consume_carried_coda`); a request the token finishes
        gets no successor, and one whose successor finds no KV block sits out a wave. Returns the
        carried successors and the requests whose tokens are pending."""

        carried, pending = [], []
        for it in items:
            r = it.req
            self.free_hidden.append(it.hidden)
            if r.status == RequestStatus.FINISHED:
                continue
            r.position += 1
            pending.append(r)
            if self._would_finish(r):
                continue
            tok = int(self._forced[r.idx][r.generated]) if self._forced is not None else -1
            if (nxt := self._carry_successor(r, tok)) is not None:
                carried.append(nxt)
        return carried, pending

    def _no_refill_loop(self, arrivals) -> None:
        carried: list[_Item] = []  # delayed path: successors staged before their wave
        coda_ids: set[int] = set()  # delayed path: the previous wave's exiters (its coda is in flight)
        pending_coda: list[_Req] = []  # that coda's requests, whose tokens are recorded during the next wave
        while arrivals or self._has_pending():
            self._release_arrivals(arrivals)
            if not self._has_pending():
                if arrivals:
                    self._wait_next_arrival(arrivals)
                continue
            self.last_stats.scheduler_ticks += 1
            # offloaded requests come back before admission, so the prefill gate counts them as
            # decoders, and join this wave's cohort (``continuous_api.py:656-658``)
            self._restore_offloaded()
            did_prefill = False
            while self._admit_prefill():
                pb = self._schedule_prefill()
                if pb is None:
                    break
                sampled = self._run_prefill(pb)
                for r, *_ in pb:
                    self.in_flight.discard(r.idx)
                if self._delayed:
                    carried += self._carry_after_prefill(sampled, max(0, self.max_num_seqs - len(carried)))
                else:
                    self._consume_prefill(sampled, stage=False)
                did_prefill = True
            # every request of the in-flight boundary coda sits out this wave's scan
            # (``continuous_api.py:829-834``)
            carried_ids = {it.req.idx for it in carried} | coda_ids
            coda_ids = set()
            cohort = [
                r
                for r in self.active.values()
                if r.status == RequestStatus.DECODING and r.generated > 0 and r.idx not in carried_ids
            ]
            cohort = cohort[: max(0, self.max_num_seqs - len(carried))]
            # a request whose token finds no KV block stalls out of this wave (``continuous_api.py:840-843``)
            items = carried + [it for r in cohort if (it := self._stage_decode(r)) is not None]
            carried = []
            if not items:
                if pending_coda:  # nothing launches: recording the carried coda is this wave's work
                    self._consume_carried_coda(pending_coda)
                    pending_coda = []
                    continue
                if not did_prefill and self.stalled:
                    self._preempt_stalled()
                    continue
                if not did_prefill and self._has_pending() and not arrivals:
                    raise CacheFullError("No-refill loop stalled with pending work (over-subscribed KV cache)")
                if arrivals and not did_prefill:
                    self._wait_next_arrival(arrivals)
                continue
            self._prelude(items)
            survivors, exited = items, []
            for step in range(self.steps):
                for it in survivors:
                    it.step = step
                live = self._run_recurrent(survivors)
                if pending_coda:  # the previous wave's coda is recorded after this wave's first launch
                    self._consume_carried_coda(pending_coda)
                    pending_coda = []
                forced = step == self.steps - 1
                cont = []
                for i, it in enumerate(survivors):
                    self.last_stats.recurrent_step_histogram[step] += 1
                    if forced or self._should_exit(it, step, live, i):
                        self._record_exit(it, step)
                        exited.append(it)
                    else:
                        cont.append(it)
                self._flush_exit_copies()
                survivors = cont
                if not survivors:
                    break
            self._run_coda(exited)
            if self._delayed:
                coda_ids = {it.req.idx for it in exited}
                carried, pending_coda = self._carry_after_coda(exited)
            else:
                self._consume_coda(exited, stage=False)

    # ------------------------------------------------------------------ validation
    def _validate(self, input_ids, max_new_tokens, exit_depths, model_kwargs) -> list[int]:
        """All checks of generate_batch's arguments; returns the per-request token caps."""

        cfg = self.cdb_config
        self._validate_generate_inputs(input_ids, max_new_tokens)
        if cfg.exit_threshold is not None and model_kwargs is not None and model_kwargs.get("use_early_exit_gate") is False:
            raise ValueError("exit_threshold CDB requires use_early_exit_gate to stay enabled")
        mnt = max_new_tokens if isinstance(max_new_tokens, list) else [max_new_tokens] * len(input_ids)
        caps = cap_max_new_tokens_to_model_len(input_ids, mnt, cfg.max_model_len)
        self._validate_exit_depths(input_ids, caps, exit_depths)
        return caps

    @staticmethod
    def _validate_generate_inputs(input_ids: list[list[int]], max_new_tokens: int | list[int]) -> None:
        """Token-level input checks before scheduling (``continuous_api.py:1766-1785``)."""

        if not input_ids:
            raise ValueError("input_ids must contain at least one prompt")
        if isinstance(max_new_tokens, list):
            if len(max_new_tokens) != len(input_ids):
                raise ValueError(
                    f"max_new_tokens has {len(max_new_tokens)} entries but there are {len(input_ids)} prompts"
                )
            bad = [i for i, v in enumerate(max_new_tokens) if v < 1]
            if bad:
                raise ValueError(f"max_new_tokens must be >= 1 for every request, but got <1 at indices {bad}")
        elif max_new_tokens <= 0:
            raise ValueError(f"max_new_tokens must be positive, but got {max_new_tokens}")
        empty = [i for i, p in enumerate(input_ids) if not p]
        if empty:
            raise ValueError(f"input_ids contains empty prompts at indices {empty}")

    def _validate_exit_depths(self, input_ids, max_new_tokens: list[int], exit_depths) -> None:
        """A replay schedule against the config and lengths (``continuous_api.py:1787-1836``);
        ``max_new_tokens`` is per request, already capped by ``max_model_len``."""

        cfg = self.cdb_config
        if exit_depths is None:
            return
        if not cfg.synthetic_exit_replay:
            raise ValueError("exit_depths requires cdb_config.synthetic_exit_replay=True")
        if cfg.exit_threshold is not None:
            raise ValueError("exit_depths cannot be combined with exit_threshold")
        if len(exit_depths) != len(input_ids):
            raise ValueError(f"exit_depths has {len(exit_depths)} entries but there are {len(input_ids)} requests")
        steps = cfg.max_recurrent_steps
        for idx, depths in enumerate(exit_depths):
            if len(depths) != max_new_tokens[idx] - 1:
                raise ValueError(
                    f"exit_depths[{idx}] has {len(depths)} entries but the request stages {max_new_tokens[idx] - 1} "
                    "decode tokens (max_new_tokens - 1)"
                )
            for d in depths:
                if not 0 <= d < steps:
                    raise ValueError(
                        f"exit_depths[{idx}] value {d} is out of range [0, {steps}); values are 0-based "
                        "recurrent steps"
                    )
        if copies_exit_kv(cfg.kv_policy):
            # copy-on-exit routing fills the deeper slots at exit time, so any replay depth is safe
            return
        slots = resolve_kv_slots_per_layer(
            cfg.kv_policy, total_recurrent_steps=steps, requested_slots=cfg.kv_slots_per_layer
        )
        extra = int(cfg.use_async_batching and cfg.delay_gate_consumption)  # continuous_api.py:1826
        for depths in exit_depths:
            for d in depths:
                if d + 1 + extra < slots:
                    raise ValueError(
                        "Every replay exit depth must write all static KV slots before exit: "
                        f"kv_slots_per_layer={slots}, exit step {d + 1 + extra}"
                    )


def cap_max_new_tokens_to_model_len(input_ids: list[list[int]], max_new_tokens: list[int],
                                    max_model_len: int | None) -> list[int]:
    """Prompt + generation within ``max_model_len`` (``utils.py:70-97``): a prompt with no room for
    a single generated token is refused (the whole batch), every other request's budget is clamped
    to ``max_model_len - len(prompt)`` (a length finish); no-op without a limit."""

    if max_model_len is None:
        return max_new_tokens
    over = [(i, len(p)) for i, p in enumerate(input_ids) if len(p) >= max_model_len]
    if over:
        shown = ", ".join(f"request {i} (len {n})" for i, n in over[:5])
        more = " ..." if len(over) > 5 else ""
        raise ValueError(
            f"{len(over)} prompt(s) have length >= max_model_len ({max_model_len}) and leave no room "
            f"for a generated token: {shown}{more}. Filter or truncate them before serving."
        )
    return [min(m, max_model_len - len(p)) for m, p in zip(max_new_tokens, input_ids, strict=True)]


def _auto_num_blocks(shape: OuroShape | HuginnShape, cfg: ContinuousDepthBatchingConfig, device: torch.device) -> int:
    """Fill the post-load budget (``kv_cache_sizing.py:34-80``; default static fraction 0.8)."""

    free, total = torch.cuda.mem_get_info(device)
    frac = 0.8 if cfg.mem_fraction_static is None else cfg.mem_fraction_static
    assert cfg.kv_slots_per_layer is not None
    h, i = shape.hidden_size, shape.intermediate_size
    # Reserve room for the packed weights, the work buffers and the logits the runner allocates.
    if isinstance(shape, HuginnShape):
        extra = shape.n_layers_in_prelude + shape.n_layers_in_coda
        weights = 2 * (shape.param_count_core_step() + extra * (4 * h * h + 3 * h * i) + shape.vocab_size * h)
        cache_layers = extra + cfg.kv_slots_per_layer * shape.n_layers_in_recurrent_block
    else:
        weights = 2 * (shape.param_count_recurrent() + 2 * shape.vocab_size * h)
        cache_layers = cfg.kv_slots_per_layer * shape.num_hidden_layers
    work = 2 * cfg.max_num_batched_tokens * (9 * h + 3 * i)
    budget = int(free - total * (1 - frac)) - weights - work
    per_block = 2 * cache_layers * cfg.block_size * shape.num_key_value_heads * shape.head_dim * 2
    blocks = budget // per_block - 2
    if blocks <= 0:
        raise ValueError("No usable KV blocks fit in device memory")
    return int(blocks)
