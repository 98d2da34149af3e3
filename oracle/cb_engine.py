"""CPU restatement of the reference's full-depth continuous-batching (CB) engine.

TEST INFRASTRUCTURE ONLY: the checker for the B200 CB baseline's schedules, block tables and
logits. Nothing in the product imports this module.

``ContinuousBatchingEngine`` (``continuous_batching/continuous_api.py:133-489``) serves every
token at the model's full recurrent depth. Each tick schedules one batch with
``FIFOScheduler.schedule_batch`` (``continuous_batching/scheduler.py:82-141``). The batch is
either prompt work (whole or chunked prompts, packed by ``_process_candidates`` ``:183-267`` under
the token and cache budgets while prefill is admitted, ``scheduler_base.py:171-201,473-516``) or
one decode token for each decoding request that its pending token will not finish, up to
``max_num_seqs``. With ``use_async_batching`` (the default) the tick launches batch k+1 before it
consumes batch k's tokens (``_execute_tick`` ``:306-448``), so the resident set and the free blocks
the scheduler sees lag one tick. When nothing fits and nothing is in flight, the active request
with the fewest cached tokens (ties: the latest) is soft-reset and re-queued
(``pop_request_to_evict`` ``scheduler_base.py:406-414``), and admission is held until a request
finishes.

A batch runs the whole model over its query rows (:meth:`OuroOracle.prefill` /
:meth:`HuginnOracle.prefill`: every recurrent step, each with its KV slot, then the LM head on the
rows that sample). A decode batch is the same
computation with one row per request. Launches are recorded as
``{"kind": "prefill" | "decode", "items": [[req, past, q_len, has_new], ...], "blocks": [...]}``.
"""

from __future__ import annotations

from collections import Counter, OrderedDict, deque

import torch

from continuous_depth_batching_b200.huginn import HuginnShape
from continuous_depth_batching_b200.ouro import OuroShape

from .engine import DECODING, FINISHED, PENDING, PREFILLING, OracleConfig, OracleEngine, Req, slot_for_step
from .huginn_math import HuginnOracle
from .ouro_math import OracleKVCache, OuroOracle


class OracleCBEngine(OracleEngine):
    """The reference CB engine on CPU over :class:`OuroOracle` or :class:`HuginnOracle` math."""

    def __init__(self, shape: OuroShape | HuginnShape, state_dict: dict, cfg: OracleConfig,
                 dtype: torch.dtype = torch.float32, async_mode: bool = True):
        super().__init__(shape, state_dict, cfg, dtype)
        self.async_mode = async_mode

    # ------------------------------------------------------------------ scheduling
    def _will_finish(self, r: Req) -> bool:
        """``will_finish_on_pending_token`` (``continuous_batching/requests.py:196-206``)."""

        return r.in_flight_tokens > 0 and len(r.generated) + r.in_flight_tokens >= r.max_new

    def _cb_prefill_candidates(self) -> list[Req]:
        """``get_prefill_candidates`` (``scheduler_base.py:473-516``); CB continues a chunked
        prefill whether or not its previous chunk is still in flight."""

        prefilling = [r for r in self.active.values() if r.status == PREFILLING]
        free_slots = max(0, self.max_num_seqs - len(self.active))
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

    def _process(self, cands: list[Req], token_budget: int, margin_frac: float):
        """``FIFOScheduler._process_candidates`` (``scheduler.py:183-267``). Returns the scheduled
        ``(req, q_len, has_new_token)`` entries and whether an allocation failed."""

        bs = self.cfg.block_size
        cache_budget = self.cfg.num_blocks * bs
        margin = margin_frac * self.cfg.num_blocks
        fast = True
        failed = False
        out = []
        for r in cands:
            n_free = len(self.free)
            if n_free < margin and out and r.status != DECODING:
                break
            toks = r.to_process if r.status == DECODING else r.remaining
            qlen = min(len(toks), token_budget)
            if qlen == 0:
                continue
            eligible = qlen == 1 and r.position < self.width * bs
            read_needed = r.position
            if not (fast and eligible) and cache_budget < read_needed:
                continue
            if not self._alloc_if_needed(r, qlen):
                failed = True
                if n_free == 0 and r.idx in self.waiting:
                    break
                continue
            # ``_schedule_request`` (``scheduler.py:158-181``)
            if len(toks) <= token_budget:
                if r.status == PENDING:
                    self.active[r.idx] = r
                if r.status <= PREFILLING:
                    r.to_process = r.remaining
                    r.remaining = []
                    r.status = DECODING
            else:
                if r.status == PENDING:
                    self.active[r.idx] = r
                    r.status = PREFILLING
                r.remaining = toks[token_budget:]
                r.to_process = toks[:token_budget]
            qlen = len(r.to_process)
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

        # offloaded requests come back first, with their KV (``scheduler.py:97-100``)
        self._restore_offloaded()
        decode = [r for r in self.active.values() if r.status == DECODING and not self._will_finish(r)]
        prefill = self._cb_prefill_candidates()
        if prefill and (not decode or len(self.free) > self.safety * self.cfg.num_blocks):
            out, failed = self._process(prefill, self.cfg.max_num_batched_tokens, self.safety)
            if out:
                return out, False
            if not decode:
                return [], failed
        if not decode:
            return [], False
        out, failed = self._process(decode, self.max_num_seqs, 0.0)
        return out, (not out and failed)

    # ------------------------------------------------------------------ launch and consume
    def _launch(self, entries) -> tuple[list[tuple[Req, int]], list[Req]]:
        """Prepare (``prepare_batch_tensors`` ``input_outputs.py:285-352``) and run one batch."""

        bs = self.cfg.block_size
        is_decode = all(q == 1 and r.status == DECODING for r, q, _h in entries)
        self.stats["decode_batches" if is_decode else "prefill_batches"] += 1
        chunks, rows, sampled, items, blocks = [], [], [], [], []
        offset = 0
        for r, qlen, has in entries:
            past = r.position
            # the device feeds a decode row the request's latest sampled token; on the host that
            # token is still in flight (pipelined mode) or already consumed into ``to_process``
            ids = [r.last_sampled] if r.in_flight_tokens > 0 else [r.last_sampled if t < 0 else t for t in r.to_process]
            chunks.append((ids, past, self.tables[r.idx]))
            items.append([r.idx, past, qlen, int(has)])
            blocks.append(list(self.tables[r.idx][: -(-(past + qlen) // bs)]))
            r.position = past + qlen
            offset += qlen
            if has:
                rows.append(offset - 1)
                sampled.append((r, len(r.generated) + r.in_flight_tokens))
                r.to_process = [-1]
                r.in_flight_tokens += 1
        self.launches.append({"kind": "decode" if is_decode else "prefill", "items": items, "blocks": blocks})
        steps = [slot_for_step(self.cfg.kv_policy, s, self.slots) for s in range(self.cfg.max_recurrent_steps)]
        hidden = self.model.prefill(chunks, steps)
        if not rows:
            return [], [r for r, *_ in entries]
        logits = self.model.lm_head(hidden[torch.tensor(rows)])
        self.logits.append(("decode" if is_decode else "prefill", logits))
        toks = torch.argmax(logits, dim=-1).tolist()
        out = []
        for (r, gen_idx), tok in zip(sampled, toks, strict=True):
            if self.forced is not None and gen_idx < len(self.forced[r.idx]):
                # (a row past the forced sequence is the extra token of a request whose finish the
                # pipelined loop has not seen yet; it is dropped when consumed)
                tok = self.forced[r.idx][gen_idx]
            r.last_sampled = tok
            out.append((r, tok))
        return out, [r for r, *_ in entries]

    def _consume(self, results: list[tuple[Req, int]]) -> None:
        """``_consume_batch`` (``continuous_api.py:450-489``)."""

        for r, tok in results:
            # a row whose request finished (EOS seen one tick late) or was evicted is dropped
            if r.status in (FINISHED, PENDING):
                continue
            if self._update(r, tok):
                self._free(r)
                self.active.pop(r.idx, None)
                self.finished[r.idx] = list(r.generated)
                self.block_new = False

    def _evict(self) -> None:
        """``offload_one_request`` (``offloading_manager.py:165-214``): the victim's blocks go to the
        host pool when they fit (``offload`` mode; it keeps its status, position and pending token),
        otherwise it is soft-reset to prompt + generated tokens."""

        victim = min(reversed(list(self.active)), key=lambda i: self.active[i].position)
        r = self.active.pop(victim)
        offloaded = self._offload(r)
        self._free(r)
        r.allocated = 0
        if offloaded:
            if r.status == DECODING:
                r.remaining = []
            self.stats["offload_preemptions"] += 1
        else:
            r.remaining = list(r.prompt) + list(r.generated)
            r.to_process = []
            r.position = 0
            r.in_flight_tokens = 0
            r.status = PENDING
            self.stats["recompute_preemptions"] += 1
        self.waiting[r.idx] = r
        self.block_new = True

    def _tick(self, in_flight):
        entries, cache_full = ([], False)
        if self.active or self.waiting:
            entries, cache_full = self._schedule_batch()
            if not entries and not cache_full and in_flight is None:
                raise RuntimeError("oracle CB: a pending prompt's KV read exceeds the cache budget")
        launched = self._launch(entries)[0] if entries else None
        to_consume = in_flight if self.async_mode else launched
        carried = launched if self.async_mode else None
        if to_consume is not None:
            self._consume(to_consume)
        if cache_full and to_consume is None:
            if self.cfg.kv_pressure_mode in ("none", "reserve"):
                raise RuntimeError("oracle CB: KV cache full")
            if len(self.active) <= 1:
                raise RuntimeError("oracle CB: a single request's KV cache does not fit")
            self._evict()
            return None
        return carried

    def generate(self, prompts, max_new_tokens, exit_depths=None, forced_tokens=None, eos_token_ids=None,
                 stop_sequences=None) -> list[list[int]]:
        if exit_depths is not None:
            raise NotImplementedError("the CB engine serves every token at full depth")
        cfg = self.cfg
        self.eos = set(eos_token_ids or [])
        self.stops = [list(q) for q in (stop_sequences or [])]
        caps = [min(m, cfg.max_model_len - len(p)) for m, p in zip(max_new_tokens, prompts, strict=True)]
        self.free = deque(range(cfg.num_blocks))
        self.tables = {}
        self.cache = OracleKVCache(self.shape, self.num_cache_layers, cfg.num_blocks, cfg.block_size, self.dtype)
        if self.huginn:
            self.model = HuginnOracle(self.weights, self.cache, self.slots)
        else:
            self.model = OuroOracle(self.weights, self.cache)
        self.waiting: OrderedDict[int, Req] = OrderedDict()
        self.active: OrderedDict[int, Req] = OrderedDict()
        self.block_new = False
        self.finished: dict[int, list[int]] = {}
        self.launches: list[dict] = []
        self.logits: list[tuple[str, torch.Tensor]] = []
        self.stats = Counter()
        self.cpu_free = deque(range(cfg.num_cpu_blocks))
        self.host_store = {}
        self.forced = forced_tokens
        for i, (p, m) in enumerate(zip(prompts, caps, strict=True)):
            r = Req(idx=i, prompt=list(p), max_new=m, depths=[])
            r.remaining = list(p)
            r.last_sampled = -1
            self.waiting[i] = r
        in_flight = None
        with torch.no_grad():
            while self.active or self.waiting or in_flight is not None:
                in_flight = self._tick(in_flight)
        return [self.finished[i] for i in range(len(prompts))]
