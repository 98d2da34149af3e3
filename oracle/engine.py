"""CPU restatement of the reference CDB engine (synchronous and delayed-gate timing).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA engine's schedules, block tables and
logits. Nothing in the product imports this module.

It restates ``ContinuousDepthBatchingEngine`` with ``use_async_batching=False`` (every
stage synchronous), and with ``OracleConfig.delayed`` the reference's default timing
(``use_async_batching`` + ``delay_gate_consumption``: decisions applied one launch late):

* refill loop ``continuous_depth_batching/continuous_api.py:503-606`` with
  ``CDBScheduler.schedule_next`` ``scheduler.py:101-140`` (coda >= min -> prefill if admitted
  -> recurrent FIFO -> coda flush);
* prefill admission/packing ``scheduler_base.py:129-201,466-515`` and ``scheduler.py:211-320``;
* recurrent routing ``continuous_api.py:1090-1203`` (survivors return to the queue head in
  order, ``scheduler.py:164-180``), exits to the coda queue;
* coda + re-entry ``continuous_api.py:1378-1448`` (sampled token -> next decode item at the
  head of the queue);
* no-refill lockstep waves ``continuous_api.py:608-944`` (``refill=False``);
* FIFO block ids ``continuous_batching/cache_manager.py:33-91`` with exact-ceil allocation
  ``scheduler_base.py:416-433`` / ``continuous_api.py:1654-1669``;
* exit policies ``exit_policy.py:150-169`` (cumulative hazard) and replay
  ``continuous_api.py:1671-1697``; ``last_exited`` copy-on-exit ``:1205-1245``.

Every launch is appended to ``launches`` in the golden-fixture format:
``{"kind": "prefill", "items": [[req, past, q_len, has_new], ...], "blocks": [...]}``,
``{"kind": "recurrent", "items": [[req, pos, step], ...], "blocks": [[block ids], ...]}``,
``{"kind": "coda", "items": [[req, pos, step], ...]}``.

``forced_tokens`` (teacher forcing) makes the engine continue every request with the given
tokens instead of its own argmax, so a second engine's per-position predictions can be
compared against these without autoregressive divergence.

Two model families: Ouro (:class:`OuroOracle`; prelude = embedding, coda = LM head, exit
signal = gate logit under the cumulative-hazard rule) and Huginn (:class:`HuginnOracle`;
``HuginnCDBAdapter`` ``adapters/huginn.py``: prelude and coda are attention blocks writing
their own cache layers, the hidden vector is ``[state | injection]``, the exit signal is the
latent difference under the direct-threshold rule ``exit_policy.py:167-168``).
"""

from __future__ import annotations

from collections import Counter, OrderedDict, deque
from dataclasses import dataclass, field

import torch

from continuous_depth_batching_b200.huginn import HuginnShape
from continuous_depth_batching_b200.ouro import OuroShape

from .huginn_math import HuginnOracle, HuginnWeights
from .ouro_math import OracleKVCache, OuroOracle, OuroWeights

PENDING, PREFILLING, DECODING, FINISHED = 0, 1, 2, 3
KV_POLICIES = ("depth_indexed", "last_exited", "single", "first_then_shared")


def slots_per_layer(policy: str, steps: int, requested: int | None = None) -> int:
    """``resolve_kv_slots_per_layer`` (``kv_cache_policy.py:52-79``)."""

    fixed = {"depth_indexed": steps, "last_exited": steps, "single": 1}
    if policy in fixed:
        return fixed[policy]
    return 2 if requested is None else requested


def slot_for_step(policy: str, step: int, slots: int) -> int:
    """``kv_slot_for_step`` (``kv_cache_policy.py:82-103``)."""

    if policy in ("depth_indexed", "last_exited"):
        return step
    if policy == "single":
        return 0
    return min(step, slots - 1)


@dataclass
class OracleConfig:
    block_size: int = 16
    num_blocks: int = 4096
    max_num_batched_tokens: int = 8192
    safety_margin: float = 0.2
    max_model_len: int = 16384
    max_recurrent_steps: int = 4
    exit_threshold: float | None = None
    synthetic_exit_replay: bool = False
    min_recurrent_steps: int = 1
    min_coda_batch_size: int = 1
    max_num_seqs: int = 256
    min_free_slots: int | None = None
    refill: bool = True
    kv_policy: str = "single"
    kv_slots_per_layer: int | None = None
    kv_pressure_mode: str = "recompute"
    # host swap pool for kv_pressure_mode="offload", in blocks (the reference sizes it from
    # cpu_offload_space GiB over the bytes of one block in every cache layer)
    num_cpu_blocks: int = 0
    # use_async_batching and delay_gate_consumption both on (the reference's defaults): every
    # exit decision is applied at the routing after the item's next launch.
    delayed: bool = False


@dataclass
class Req:
    idx: int
    prompt: list[int]
    max_new: int
    depths: list[int]
    status: int = PENDING
    remaining: list[int] = field(default_factory=list)
    to_process: list[int] = field(default_factory=list)
    generated: list[int] = field(default_factory=list)
    position: int = 0
    allocated: int = 0
    in_flight_tokens: int = 0
    cursor: int = 0
    exit_depths: list[int] = field(default_factory=list)
    offloaded: bool = False

    def next_depth(self) -> int | None:
        if not self.depths:
            return None
        d = self.depths[self.cursor]
        self.cursor += 1
        return d


@dataclass
class Item:
    req: Req
    token: int
    position: int
    step: int
    depth: int | None
    hidden: torch.Tensor | None = None
    cdf: float = 0.0
    survival: float = 1.0
    pending_step: int | None = None  # delayed: the step whose decision is still to be applied
    pending_signal: torch.Tensor | None = None


class OracleEngine:
    """Synchronous-mode CDB engine on CPU over :class:`OuroOracle` math."""

    def __init__(
        self, shape: OuroShape | HuginnShape, state_dict: dict, cfg: OracleConfig, dtype: torch.dtype = torch.float32
    ):
        if cfg.kv_policy not in KV_POLICIES:
            raise ValueError(f"unknown kv_policy {cfg.kv_policy!r}")
        self.shape = shape
        self.cfg = cfg
        self.dtype = dtype
        self.huginn = isinstance(shape, HuginnShape)
        self.slots = slots_per_layer(cfg.kv_policy, cfg.max_recurrent_steps, cfg.kv_slots_per_layer)
        if self.huginn:
            self.core_layers = shape.n_layers_in_recurrent_block
            self.num_cache_layers = shape.n_layers_in_prelude + self.slots * self.core_layers + shape.n_layers_in_coda
            self.weights = HuginnWeights.from_state_dict(shape, state_dict, dtype)
        else:
            self.core_layers = shape.num_hidden_layers
            self.num_cache_layers = self.slots * shape.num_hidden_layers
            self.weights = OuroWeights.from_state_dict(shape, state_dict, dtype)
        self.max_num_seqs = min(cfg.max_num_seqs, cfg.max_num_batched_tokens)
        self.min_free = (
            max(1, self.max_num_seqs // 8) if cfg.min_free_slots is None else min(cfg.min_free_slots, self.max_num_seqs)
        )
        self.safety = 0.0 if cfg.kv_pressure_mode == "reserve" else cfg.safety_margin
        self.width = -(-cfg.max_model_len // cfg.block_size)

    # ------------------------------------------------------------------ block pool
    def _alloc(self, r: Req, n: int) -> bool:
        if n > len(self.free):
            return False
        got = [self.free.popleft() for _ in range(n)]
        self.tables.setdefault(r.idx, []).extend(got)
        r.allocated += n
        return True

    def _free(self, r: Req) -> None:
        self.free.extend(self.tables.pop(r.idx, []))

    def _alloc_if_needed(self, r: Req, n_next: int) -> bool:
        bs = self.cfg.block_size
        if r.allocated * bs - r.position < n_next:
            need = -(-(r.position + n_next) // bs) - r.allocated
            return self._alloc(r, need)
        return True

    def _alloc_one_decode(self, r: Req) -> bool:
        bs = self.cfg.block_size
        if r.allocated * bs - r.position >= 1 and r.allocated > 0:
            return True
        need = -(-(r.position + 1) // bs) - r.allocated
        return self._alloc(r, need)

    # ------------------------------------------------------------------ request bookkeeping
    def _update(self, r: Req, token: int) -> bool:
        """``RequestState.update_and_check_completion`` (``continuous_batching/requests.py:209-250``):
        an EOS id is kept and finishes the request, as does the length limit or a generated tail
        equal to a stop sequence."""

        r.in_flight_tokens = max(0, r.in_flight_tokens - 1)
        is_eos = token in self.eos
        if is_eos or len(r.generated) < r.max_new:
            r.generated.append(token)
            r.to_process = [token]
        stop = any(len(q) and len(r.generated) >= len(q) and r.generated[-len(q):] == q for q in self.stops)
        if is_eos or len(r.generated) >= r.max_new or stop:
            r.status = FINISHED
            return True
        return False

    def _retire(self, r: Req) -> None:
        self._free(r)
        self.active.pop(r.idx, None)
        self.in_flight.discard(r.idx)
        self.stalled.pop(r.idx, None)
        self.finished[r.idx] = list(r.generated)
        self.block_new = False  # a finish frees blocks: admission resumes (continuous_api.py:1436-1448)

    def _stage_decode(self, r: Req) -> Item | None:
        """``_stage_decode_token`` (``continuous_api.py:1584-1610``): a request whose next token
        cannot get a KV block stalls (retried each tick, preempted only when nothing can run)."""

        if not self._alloc_one_decode(r):
            if self.cfg.kv_pressure_mode in ("none", "reserve"):
                raise RuntimeError("oracle: KV cache full (size num_blocks to fit the workload)")
            self.stalled[r.idx] = r
            return None
        self.stalled.pop(r.idx, None)
        return Item(req=r, token=r.to_process[0], position=r.position, step=0, depth=r.next_depth())

    def _restage_stalled(self) -> list[Item]:
        """``_restage_stalled_decoders`` (``:1612-1623``): retry in stall order, stop at the first
        request that still cannot allocate."""

        items = []
        for r in list(self.stalled.values()):
            it = self._stage_decode(r)
            if it is None:
                break
            items.append(it)
        return items

    def _preempt_stalled(self) -> None:
        """``_preempt_stalled_decoder`` (``:1625-1652``) with recompute (soft reset,
        ``create_equivalent_initial_request``, ``requests.py:290-315`` and the CDB slice of the replay
        schedule): the stalled request with the fewest cached tokens (ties: the latest staller)
        gives up its KV; its generated tokens join its prompt for a full-depth re-prefill; it waits
        behind every other waiting prompt, and no new prompt is admitted until a request finishes."""

        if len(self.active) <= 1:
            raise RuntimeError("oracle: a single request's KV cache does not fit")
        victim = min(reversed(list(self.stalled)), key=lambda i: self.stalled[i].position)
        r = self.stalled.pop(victim)
        offloaded = self._offload(r)
        if not offloaded and self.cfg.kv_pressure_mode == "offload" and self.cfg.kv_policy == "last_exited":
            raise RuntimeError("oracle: host pool full and the recompute fallback is off under last_exited")
        self._free(r)
        self.active.pop(r.idx, None)
        self.in_flight.discard(r.idx)
        self.waiting.pop(r.idx, None)
        if offloaded:
            # ``prepare_for_offload_requeue`` (``requests.py:275-288``): still decoding, same
            # position and pending token; only the block allocation is dropped
            r.allocated = 0
            self.stats["offload_preemptions"] += 1
        else:
            r.remaining = list(r.prompt) + list(r.generated)
            r.to_process = []
            r.position = 0
            r.allocated = 0
            r.status = PENDING
            r.cursor += 1  # the pending token's depth is spent: it is recomputed at full depth
            self.stats["recompute_preemptions"] += 1
        self.waiting[r.idx] = r
        self.block_new = True

    def _offload(self, r: Req) -> bool:
        """``OffloadingManager._offload_to_cpu`` (``offloading_manager.py:269-306``): copy every
        block of the request (all cache layers, K and V) into the host pool; False when the pool
        has too few free blocks (the caller then soft-resets instead)."""

        if self.cfg.kv_pressure_mode != "offload" or self.cfg.num_cpu_blocks <= 0:
            return False
        blocks = self.tables.get(r.idx, [])
        if not blocks or len(self.cpu_free) < len(blocks):
            return False
        host = [self.cpu_free.popleft() for _ in blocks]
        rows = self.cache.rows_for(blocks, 0, len(blocks) * self.cfg.block_size)
        saved = ([k[rows].clone() for k in self.cache.k], [v[rows].clone() for v in self.cache.v])
        self.host_store[r.idx] = (host, saved)
        r.offloaded = True
        return True

    def _restore_offloaded(self) -> list[Req]:
        """``admit_offloaded_restores`` (``scheduler_base.py:434-460``) then
        ``restore_scheduled_requests`` (``offloading_manager.py:216-267``): offloaded waiting
        requests return to the active set in queue order, ahead of fresh prompts, while a resident
        slot and blocks for their cached tokens plus the pending one are free; their KV is copied
        into the new blocks and their host blocks are released."""

        if self.block_new or self.cfg.kv_pressure_mode != "offload" or self.cfg.num_cpu_blocks <= 0:
            return []
        admitted = []
        for i in list(self.waiting):
            r = self.waiting[i]
            if not r.offloaded:
                continue
            if max(0, self.max_num_seqs - len(self.active)) == 0 or not self._alloc_if_needed(r, 1):
                break
            self.active[i] = r
            del self.waiting[i]
            admitted.append(r)
        for r in admitted:
            host, (ks, vs) = self.host_store.pop(r.idx)
            blocks = self.tables[r.idx][: len(host)]
            rows = self.cache.rows_for(blocks, 0, len(blocks) * self.cfg.block_size)
            for k, v, sk, sv in zip(self.cache.k, self.cache.v, ks, vs, strict=True):
                k[rows] = sk
                v[rows] = sv
            self.cpu_free.extend(host)
            r.offloaded = False
            self.stats["restores"] += 1
        return admitted

    def _next_token(self, r: Req, computed: int) -> int:
        if self.forced is not None:
            return self.forced[r.idx][len(r.generated)]
        return computed

    # ------------------------------------------------------------------ queues
    def _enqueue(self, item: Item, front: bool = False) -> None:
        self.in_flight.add(item.req.idx)
        if item.step == 0 and self.ready:
            self.refills += 1
        if front:
            self.ready.appendleft(item)
        else:
            self.ready.append(item)

    def _enqueue_front(self, items: list[Item]) -> None:
        for item in reversed(items):
            self._enqueue(item, front=True)

    def _has_pending(self) -> bool:
        return bool(self.coda_q or self.ready or self.active or self.waiting)

    def _has_decode_work(self) -> bool:
        return any(r.status == DECODING for r in self.active.values())

    def _admit_prefill(self) -> bool:
        return not self._has_decode_work() or len(self.free) > self.safety * self.cfg.num_blocks

    def _reserved_peak(self, r: Req) -> int:
        total = min(len(r.prompt) + r.max_new, self.cfg.max_model_len)
        return -(-total // self.cfg.block_size)

    def _prefill_candidates(self) -> list[Req]:
        prefilling = [r for r in self.active.values() if r.status == PREFILLING and r.idx not in self.in_flight]
        free_slots = max(0, self.max_num_seqs - len(self.active))
        # fresh prompts only: offloaded requests come back through the restore path
        fresh = [r for r in self.waiting.values() if not r.offloaded]
        admissible = [] if self.block_new else fresh[:free_slots]
        if self.cfg.kv_pressure_mode == "reserve":
            committed = sum(self._reserved_peak(r) for r in self.active.values())
            kept = []
            for r in admissible:
                need = self._reserved_peak(r)
                if committed + need > self.cfg.num_blocks:
                    break
                committed += need
                kept.append(r)
            admissible = kept
        cands = prefilling + admissible
        if not cands:
            return []
        if any(r.status == PREFILLING for r in cands):
            return cands
        return cands if free_slots >= self.min_free else []

    def _schedule_prefill(self) -> list[tuple[Req, int, int, bool]] | None:
        cands = self._prefill_candidates()
        if not cands:
            return None
        bs = self.cfg.block_size
        token_budget = self.cfg.max_num_batched_tokens
        cache_budget = self.cfg.num_blocks * bs
        margin = self.safety * self.cfg.num_blocks
        fast = True
        out = []
        for r in cands:
            n_free = len(self.free)
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
            if not self._alloc_if_needed(r, qlen):
                if n_free == 0 and r.idx in self.waiting:
                    break
                continue
            past = r.position
            if len(toks) <= qlen:
                if r.status == PENDING:
                    self.active[r.idx] = r
                if r.status <= PREFILLING:
                    r.to_process = toks
                    r.remaining = []
                    r.status = DECODING
            else:
                if r.status == PENDING:
                    self.active[r.idx] = r
                    r.status = PREFILLING
                r.remaining = toks[qlen:]
                r.to_process = toks[:qlen]
            self.in_flight.add(r.idx)
            qlen = len(r.to_process)
            fast = fast and qlen == 1 and r.position < self.width * bs
            token_budget -= qlen
            cache_budget -= read_needed
            has_new = not r.remaining
            out.append((r, past, qlen, has_new))
            self.waiting.pop(r.idx, None)
            if token_budget == 0 or (cache_budget <= 0 and not fast):
                break
        return out or None

    # ------------------------------------------------------------------ launches
    def _run_prefill(self, batch: list[tuple[Req, int, int, bool]]) -> list[tuple[Req, int]]:
        """Full-depth prefill; returns ``(req, sampled token)`` for prompts that finished."""

        chunks = []
        for r, past, qlen, _has in batch:
            chunks.append((list(r.to_process), past, self.tables[r.idx]))
        steps = [slot_for_step(self.cfg.kv_policy, s, self.slots) for s in range(self.cfg.max_recurrent_steps)]
        hidden = self.model.prefill(chunks, steps)
        rows, offset = [], 0
        for r, past, qlen, has in batch:
            r.position = past + qlen
            offset += qlen
            if has:
                rows.append(offset - 1)
                r.to_process = [-1]
                r.in_flight_tokens += 1
        self.launches.append(
            {
                "kind": "prefill",
                "items": [[r.idx, past, qlen, int(has)] for r, past, qlen, has in batch],
                "blocks": [list(self.tables[r.idx][: -(-r.position // self.cfg.block_size)]) for r, *_ in batch],
            }
        )
        if not rows:
            return []
        logits = self.model.lm_head(hidden[torch.tensor(rows)])
        self.logits.append(("prefill", logits))
        toks = torch.argmax(logits, dim=-1).tolist()
        sampled = [r for r, _p, _q, has in batch if has]
        return list(zip(sampled, toks, strict=True))

    def _run_recurrent(self, items: list[Item]) -> torch.Tensor | None:
        bs = self.cfg.block_size
        slot = slot_for_step(self.cfg.kv_policy, items[0].step, self.slots)
        blocks = [self.tables[it.req.idx][: -(-(it.position + 1) // bs)] for it in items]
        self.launches.append(
            {
                "kind": "recurrent",
                "items": [[it.req.idx, it.position, it.step] for it in items],
                "blocks": [list(b) for b in blocks],
            }
        )
        hidden = torch.stack([it.hidden for it in items])
        if self.huginn:
            out, gate = self.model.recurrent_step(hidden, [it.position for it in items], blocks, slot)
        else:
            out, gate = self.model.recurrent_step(
                hidden, [it.position for it in items], blocks, slot * self.shape.num_hidden_layers
            )
        for i, it in enumerate(items):
            it.hidden = out[i]
        self.stats["recurrent_batches"] += 1
        self.stats["recurrent_steps"] += len(items)
        return gate

    def _should_exit(self, item: Item, step: int, gate: torch.Tensor | None, i: int) -> bool:
        if self.cfg.delayed:
            return self._should_exit_delayed(item, step, gate, i)
        if step == self.cfg.max_recurrent_steps - 1:
            return True
        if item.depth is not None:
            return step >= item.depth
        if self.cfg.exit_threshold is None:
            return False
        return self._policy(item, step, gate[i])

    def _policy(self, item: Item, source_step: int, signal: torch.Tensor) -> bool:
        """``ExitPolicy.should_exit`` (``exit_policy.py:150-169``) for one signal of ``source_step``."""

        can_exit = source_step + 1 >= self.cfg.min_recurrent_steps
        if self.huginn:
            return can_exit and float(signal.float().item()) < self.cfg.exit_threshold
        hazard = float(torch.sigmoid(signal).float().item())
        item.cdf += hazard * item.survival
        item.survival *= 1.0 - hazard
        return can_exit and item.cdf >= self.cfg.exit_threshold

    def _should_exit_delayed(self, item: Item, step: int, gate: torch.Tensor | None, i: int) -> bool:
        """Delayed consumption: ``_consume_delayed_gate`` / ``_consume_delayed_synthetic_exit``
        (``continuous_api.py:1699-1724``) route on the previous step's pending decision, then
        ``_schedule_after_delayed_*_step`` (``:1250-1280``) keep this step's for the next routing."""

        pend_step, pend_sig = item.pending_step, item.pending_signal
        item.pending_step = step
        item.pending_signal = gate[i] if gate is not None else None
        if step == self.cfg.max_recurrent_steps - 1:
            return True
        if item.depth is not None:
            return pend_step is not None and pend_step >= item.depth
        if self.cfg.exit_threshold is None or pend_sig is None:
            return False
        return self._policy(item, pend_step, pend_sig)

    def _record_exit(self, item: Item, step: int) -> None:
        item.req.exit_depths.append(step)
        self.hist[step] += 1
        if self.cfg.kv_policy == "last_exited" and step < self.cfg.max_recurrent_steps - 1:
            self.backlog.append((item, step))

    def _flush_exit_copies(self) -> None:
        """``_flush_exit_kv_copies`` + ``LoopedKvLayout.exit_copy_layer_groups`` (``kv_cache_policy.py:235-258``)."""

        if not self.backlog:
            return
        backlog, self.backlog = self.backlog, []
        by_step: dict[int, list[Item]] = {}
        for item, step in backlog:
            by_step.setdefault(step, []).append(item)
        bs, layers = self.cfg.block_size, self.core_layers
        first = self.shape.n_layers_in_prelude if self.huginn else 0
        for step, items in sorted(by_step.items()):
            rows = torch.tensor(
                [self.tables[it.req.idx][it.position // bs] * bs + it.position % bs for it in items], dtype=torch.long
            )
            src_slot = slot_for_step(self.cfg.kv_policy, step, self.slots)
            for layer in range(layers):
                dst = [first + t * layers + layer for t in range(src_slot + 1, self.slots)]
                if dst:
                    self.model.copy_rows(first + src_slot * layers + layer, dst, rows)

    def _item_blocks(self, it: Item) -> list[int]:
        return self.tables[it.req.idx][: -(-(it.position + 1) // self.cfg.block_size)]

    def _prelude(self, items: list[Item]) -> None:
        if not items:
            return
        if self.huginn:
            emb = self.model.prelude(
                [it.token for it in items], [it.position for it in items], [self._item_blocks(it) for it in items]
            )
        else:
            emb = self.model.embed([it.token for it in items])
        for i, it in enumerate(items):
            it.hidden = emb[i]

    def _run_coda(self, items: list[Item]) -> list[int]:
        self.launches.append({"kind": "coda", "items": [[it.req.idx, it.position, it.step] for it in items]})
        for it in items:
            it.req.in_flight_tokens += 1
        hidden = torch.stack([it.hidden for it in items])
        if self.huginn:
            hidden = self.model.coda(hidden, [it.position for it in items], [self._item_blocks(it) for it in items])
        logits = self.model.lm_head(hidden)
        self.logits.append(("coda", logits))
        self.stats["coda_batches"] += 1
        self.stats["coda_tokens"] += len(items)
        return torch.argmax(logits, dim=-1).tolist()

    # ------------------------------------------------------------------ loops
    def _consume_prefill(self, results: list[tuple[Req, int]], stage: bool) -> None:
        new_items = []
        for r, tok in results:
            if r.status == FINISHED:
                continue
            if self._update(r, self._next_token(r, tok)):
                self._retire(r)
                continue
            if stage and (it := self._stage_decode(r)) is not None:
                new_items.append(it)
        self._prelude(new_items)
        for it in new_items:
            self._enqueue(it)

    def _consume_coda(self, items: list[Item], toks: list[int], stage: bool) -> None:
        new_items = []
        for it, tok in zip(items, toks, strict=True):
            r = it.req
            if r.status == FINISHED:
                continue
            r.position += 1
            if self._update(r, self._next_token(r, tok)):
                self._retire(r)
                continue
            if stage and (it := self._stage_decode(r)) is not None:
                new_items.append(it)
        self._prelude(new_items)
        self._enqueue_front(new_items)

    def _refill_loop(self) -> None:
        pending_prefill: list[list[tuple[Req, int]]] = []
        pending_coda: list[tuple[list[Item], list[int]]] = []
        while self._has_pending() or pending_prefill or pending_coda:
            for res in pending_prefill:
                self._consume_prefill(res, stage=True)
            pending_prefill = []
            for items, toks in pending_coda:
                self._consume_coda(items, toks, stage=True)
            pending_coda = []
            if not self._has_pending():
                continue
            # restored requests, then decode tokens that could not get a KV block last tick, go
            # first, at the queue head
            resumed = [it for r in self._restore_offloaded() if (it := self._stage_decode(r)) is not None]
            resumed += self._restage_stalled()
            self._prelude(resumed)
            self._enqueue_front(resumed)
            self.stats["ticks"] += 1
            if len(self.coda_q) >= self.cfg.min_coda_batch_size:
                batch = [self.coda_q.popleft() for _ in range(min(self.max_num_seqs, len(self.coda_q)))]
                pending_coda.append((batch, self._run_coda(batch)))
                continue
            if self._admit_prefill():
                pb = self._schedule_prefill()
                if pb is not None:
                    self.stats["prefill_batches"] += 1
                    pending_prefill.append(self._run_prefill(pb))
                    for r, _past, _q, has in pb:
                        if not has:
                            self.in_flight.discard(r.idx)
                    continue
            items = self._pop_recurrent()
            if items:
                gate = self._run_recurrent(items)
                refills = []
                for i, it in enumerate(items):
                    if self._should_exit(it, it.step, gate, i):
                        self._record_exit(it, it.step)
                        self.in_flight.add(it.req.idx)
                        self.coda_q.append(it)
                    else:
                        it.step += 1
                        refills.append(it)
                self._enqueue_front(refills)
                self._flush_exit_copies()
                continue
            if self.coda_q:
                batch = [self.coda_q.popleft() for _ in range(min(self.max_num_seqs, len(self.coda_q)))]
                pending_coda.append((batch, self._run_coda(batch)))
                continue
            if self.stalled:
                self._preempt_stalled()
                continue
            raise RuntimeError("oracle: scheduler stalled (KV cache too small for the workload)")

    def _pop_recurrent(self) -> list[Item]:
        n = min(self.max_num_seqs, len(self.ready))
        if n == 0:
            return []
        first = self.ready.popleft()
        batch = [first]
        if self.slots > 1:
            target = slot_for_step(self.cfg.kv_policy, first.step, self.slots)
            deferred: deque[Item] = deque()
            while self.ready and len(batch) < n:
                it = self.ready.popleft()
                if slot_for_step(self.cfg.kv_policy, it.step, self.slots) == target:
                    batch.append(it)
                else:
                    deferred.append(it)
            deferred.extend(self.ready)
            self.ready = deferred
        else:
            while self.ready and len(batch) < n:
                batch.append(self.ready.popleft())
        return batch

    def _carry_successor(self, r: Req, token: int | None = None) -> Item | None:
        """Eager re-entry (``_select_eager_reentries``, ``continuous_api.py:1304-1327``)."""

        if not self._alloc_one_decode(r):
            return None
        tok = r.to_process[0] if token is None else token
        return Item(req=r, token=tok, position=r.position, step=0, depth=r.next_depth())

    def _finishes_on(self, r: Req, token: int) -> bool:
        """Whether consuming ``token`` will finish ``r`` (length limit, EOS id, stop sequence)."""

        gen = list(r.generated) + [token]
        stop = any(len(q) and len(gen) >= len(q) and gen[-len(q):] == q for q in self.stops)
        return token in self.eos or len(gen) >= r.max_new or stop

    def _consume_carried_coda(self, pending: list[tuple[Req, int]]) -> None:
        """``_consume_no_refill_coda``: the boundary coda's tokens are applied (and finished
        requests retired, freeing their blocks) once the next wave's first launch is queued."""

        for r, tok in pending:
            if r.status == FINISHED:
                continue
            if self._update(r, tok):
                self._retire(r)

    def _no_refill_loop(self) -> None:
        # Delayed mode carries a wave's exiters' successors (staged at its boundary coda, in exit
        # order) and each prefilled request's first decode token (up to the launch width) into
        # the next wave ahead of the cohort scan (``continuous_api.py:721-790, 815-944``).
        carried: list[Item] = []
        coda_ids: set[int] = set()  # delayed path: the previous wave's exiters (its coda is in flight)
        pending_coda: list[tuple[Req, int]] = []  # that coda's tokens, applied during the next wave
        while self._has_pending():
            # offloaded requests come back before admission, so the prefill gate sees them as
            # decoders, and join this wave's cohort (``continuous_api.py:656-658``)
            self._restore_offloaded()
            did_prefill = False
            while self._admit_prefill():
                pb = self._schedule_prefill()
                if pb is None:
                    break
                self.stats["prefill_batches"] += 1
                res = self._run_prefill(pb)
                for r, *_ in pb:
                    self.in_flight.discard(r.idx)
                if self.cfg.delayed:
                    budget = max(0, self.max_num_seqs - len(carried))
                    for r, tok in res:
                        if r.status == FINISHED:
                            continue
                        if self._update(r, self._next_token(r, tok)):
                            self._retire(r)
                            continue
                        if budget > 0 and (it := self._carry_successor(r)) is not None:
                            carried.append(it)
                            budget -= 1
                else:
                    self._consume_prefill(res, stage=False)
                did_prefill = True
            # every request of the in-flight boundary coda sits out this wave's scan, so one whose
            # successor found no KV block joins a wave later (continuous_api.py:829-834, 929-940)
            carried_ids = {it.req.idx for it in carried} | coda_ids
            coda_ids = set()
            cohort = [
                r
                for r in self.active.values()
                if r.status == DECODING and r.to_process and r.to_process[0] >= 0 and r.idx not in carried_ids
            ]
            cohort = cohort[: max(0, self.max_num_seqs - len(carried))]
            # a token that finds no KV block stalls its request out of this wave
            # (continuous_api.py:840-843); a wave-less pass preempts one staller (:672-677)
            items = carried + [it for r in cohort if (it := self._stage_decode(r)) is not None]
            carried = []
            if not items:
                if pending_coda:  # nothing launches: consuming the carried coda is this wave's work
                    self._consume_carried_coda(pending_coda)
                    pending_coda = []
                    continue
                if not did_prefill and self.stalled:
                    self._preempt_stalled()
                    continue
                if not did_prefill and self._has_pending():
                    raise RuntimeError("oracle: no-refill loop stalled")
                continue
            self._prelude(items)
            survivors, exited = items, []
            for step in range(self.cfg.max_recurrent_steps):
                for it in survivors:
                    it.step = step
                gate = self._run_recurrent(survivors)
                if pending_coda:  # the previous wave's coda is consumed after this wave's first launch
                    self._consume_carried_coda(pending_coda)
                    pending_coda = []
                forced = step == self.cfg.max_recurrent_steps - 1
                cont = []
                for i, it in enumerate(survivors):
                    if forced or self._should_exit(it, step, gate, i):
                        self._record_exit(it, step)
                        exited.append(it)
                    else:
                        cont.append(it)
                self._flush_exit_copies()
                survivors = cont
                if not survivors:
                    break
            toks = self._run_coda(exited)
            if self.cfg.delayed:
                coda_ids = {it.req.idx for it in exited}
                for it, tok in zip(exited, toks, strict=True):
                    r = it.req
                    if r.status == FINISHED:
                        continue
                    tok = self._next_token(r, tok)
                    r.position += 1
                    pending_coda.append((r, tok))
                    # no successor for a token that finishes its request (the length limit, as the
                    # reference predicts it; an EOS id or stop sequence, which this restatement reads
                    # before staging); a successor that finds no KV block waits a wave
                    if not self._finishes_on(r, tok) and (nxt := self._carry_successor(r, tok)) is not None:
                        carried.append(nxt)
            else:
                self._consume_coda(exited, toks, stage=False)

    def generate(
        self,
        prompts: list[list[int]],
        max_new_tokens: list[int],
        exit_depths: list[list[int]] | None = None,
        forced_tokens: list[list[int]] | None = None,
        eos_token_ids: list[int] | None = None,
        stop_sequences: list[list[int]] | None = None,
    ) -> list[list[int]]:
        cfg = self.cfg
        self.eos = set(eos_token_ids or [])
        self.stops = [list(q) for q in (stop_sequences or [])]
        caps = [min(m, cfg.max_model_len - len(p)) for m, p in zip(max_new_tokens, prompts, strict=True)]
        self.free: deque[int] = deque(range(cfg.num_blocks))
        self.tables: dict[int, list[int]] = {}
        cache = OracleKVCache(self.shape, self.num_cache_layers, cfg.num_blocks, cfg.block_size, self.dtype)
        self.cache = cache
        self.cpu_free: deque[int] = deque(range(cfg.num_cpu_blocks))
        self.host_store: dict[int, tuple[list[int], tuple[list[torch.Tensor], list[torch.Tensor]]]] = {}
        if self.huginn:
            self.model = HuginnOracle(self.weights, cache, self.slots)
        else:
            self.model = OuroOracle(self.weights, cache)
        self.waiting: OrderedDict[int, Req] = OrderedDict()
        self.active: OrderedDict[int, Req] = OrderedDict()
        self.in_flight: set[int] = set()
        self.ready: deque[Item] = deque()
        self.coda_q: deque[Item] = deque()
        self.backlog: list[tuple[Item, int]] = []
        self.stalled: OrderedDict[int, Req] = OrderedDict()
        self.block_new = False
        self.finished: dict[int, list[int]] = {}
        self.launches: list[dict] = []
        self.logits: list[tuple[str, torch.Tensor]] = []
        self.refills = 0
        self.hist: Counter[int] = Counter()
        self.stats = Counter()
        self.forced = forced_tokens
        reqs = []
        for i, (p, m) in enumerate(zip(prompts, caps, strict=True)):
            r = Req(idx=i, prompt=list(p), max_new=m, depths=list(exit_depths[i]) if exit_depths else [])
            r.remaining = list(p)
            reqs.append(r)
            self.waiting[i] = r
        with torch.no_grad():
            if cfg.refill:
                self._refill_loop()
            else:
                self._no_refill_loop()
        self.requests = reqs
        self.stats["generated_tokens"] = sum(len(v) for v in self.finished.values())
        self.stats["scheduler_refills"] = self.refills
        return [self.finished[i] for i in range(len(prompts))]


def exit_depth_histogram(engine: OracleEngine) -> dict[str, int]:
    return {str(k): v for k, v in sorted(engine.hist.items())}


def isclose_tokens(a: list[list[int]], b: list[list[int]]) -> float:
    """Fraction of equal token positions between two generations (same shapes)."""

    total = sum(len(x) for x in a)
    same = sum(int(p == q) for x, y in zip(a, b, strict=True) for p, q in zip(x, y, strict=True))
    return same / total if total else 1.0


__all__ = ["OracleConfig", "OracleEngine", "exit_depth_histogram", "isclose_tokens"]
