"""Device scheduling primitives (``cdb_exit_gate_route``, the FIFO block allocator, the per-launch
table build) against the host rules they restate, through the C ABI. All integer / decision
outputs must match exactly.

* Routing: a population of tokens in policy-state slots runs through many launches (random
  subsets, random order, padding rows). Each launch's exit flags, the ordered survivor and exit
  lists and the counts equal what the CPU oracle's ``_should_exit`` (synchronous) or its delayed
  consumption path decides for the same rows, for replay, cumulative hazard and direct threshold.
* Allocator: a random sequence of allocations (including ones that cannot be granted) and
  releases gives the same block-table rows, free count and peak as the host ``BlockPool`` (the
  order-exact FIFO deque pinned by the reference traces).
* Tables: block rows, ``cu_seq_lens_q/k`` and padding equal the reference's host construction.
"""

from __future__ import annotations

import math
import random
from types import SimpleNamespace

import pytest
import torch

from continuous_depth_batching_b200 import _lib
from continuous_depth_batching_b200.kv_cache import BlockPool
from oracle.engine import Item, OracleEngine

pytestmark = pytest.mark.gpu
DEV = "cuda"

# Gate logits whose fp32 sigmoid is far from a bf16 rounding midpoint, so host and device hazards
# are the same bf16 value (the hazard rounding itself is covered by test_exit_hazard_matches_host_policy).
LOGITS = [-3.0, -2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0]


def _oracle_router(policy: int, delayed: bool, steps: int, min_steps: int, tau: float | None) -> OracleEngine:
    eng = OracleEngine.__new__(OracleEngine)
    eng.cfg = SimpleNamespace(
        delayed=delayed, max_recurrent_steps=steps, exit_threshold=tau, min_recurrent_steps=min_steps
    )
    eng.huginn = policy == 2
    return eng


def _sp() -> int:
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("delayed", [False, True])
@pytest.mark.parametrize("policy", [0, 1, 2])
def test_exit_gate_route_matches_oracle_rules(policy, delayed):
    rng = random.Random(100 * policy + int(delayed))
    S, min_steps = 4, 2
    tau = {0: None, 1: 0.5, 2: 0.4}[policy]
    slots = 48
    router = _oracle_router(policy, delayed, S, min_steps, tau)
    for x in LOGITS:
        h32 = 1.0 / (1.0 + math.exp(-x))
        b = float(torch.tensor(h32).to(torch.bfloat16).float())
        ulp = 2.0 ** (math.floor(math.log2(b)) - 7)
        assert abs(abs(h32 - b) - ulp / 2) > 1e-4 * ulp
    cdf = torch.zeros(slots, dtype=torch.float64, device=DEV)
    surv = torch.ones(slots, dtype=torch.float64, device=DEV)
    pending = torch.full((slots,), -1, dtype=torch.int8, device=DEV)

    def new_token(slot):
        depth = rng.randrange(S) if policy == 0 else None
        return Item(req=None, token=0, position=0, step=0, depth=depth)

    tokens = {s: new_token(s) for s in range(slots)}
    fresh = set(range(slots))
    launches = 0
    for _ in range(60):
        rows = rng.sample(range(slots), rng.randrange(1, slots + 1))
        n_pad = rng.randrange(0, 4)
        hidden = rows + [-1] * n_pad
        rng.shuffle(hidden)
        n = len(hidden)
        if policy == 2:
            sig = [rng.random() for _ in range(n)]
        else:
            sig = [rng.choice(LOGITS) for _ in range(n)]
        signal = torch.tensor(sig).to(torch.bfloat16)
        step = [tokens[h].step if h >= 0 else 0 for h in hidden]
        depth = [(tokens[h].depth if tokens[h].depth is not None else -1) if h >= 0 else -1 for h in hidden]
        reset = [int(h >= 0 and h in fresh) for h in hidden]
        d = lambda v, dt: torch.tensor(v, dtype=dt, device=DEV)  # noqa: E731
        hid_d, step_d, dep_d, reset_d = d(hidden, torch.int32), d(step, torch.int32), d(depth, torch.int32), d(reset, torch.int8)
        sig_d = signal.to(DEV)
        flags = torch.zeros(n, dtype=torch.int8, device=DEV)
        surv_l = torch.full((n,), -7, dtype=torch.int32, device=DEV)
        exit_l = torch.full((n,), -7, dtype=torch.int32, device=DEV)
        counts = torch.zeros(2, dtype=torch.int32, device=DEV)
        _lib.call(
            "cdb_exit_gate_route", _lib.ptr(sig_d), 1, _lib.ptr(hid_d), _lib.ptr(step_d), _lib.ptr(dep_d),
            _lib.ptr(reset_d), _lib.ptr(cdf), _lib.ptr(surv), _lib.ptr(pending), n, policy, int(delayed), min_steps, S,
            float(tau) if tau is not None else 0.0, _lib.ptr(flags), _lib.ptr(surv_l), _lib.ptr(exit_l),
            _lib.ptr(counts), _sp(),
        )
        torch.cuda.synchronize()
        want_flags, want_s, want_e = [], [], []
        for i, h in enumerate(hidden):
            if h < 0:
                want_flags.append(-1)
                continue
            it = tokens[h]
            gate = signal if policy != 0 else None
            ex = router._should_exit(it, it.step, gate, i)
            want_flags.append(int(ex))
            (want_e if ex else want_s).append(i)
        assert flags.tolist() == want_flags
        ns, ne = counts.tolist()
        assert (ns, ne) == (len(want_s), len(want_e))
        assert surv_l[:ns].tolist() == want_s
        assert exit_l[:ne].tolist() == want_e
        for i, h in enumerate(hidden):
            if h < 0:
                continue
            fresh.discard(h)
            if want_flags[i]:
                tokens[h] = new_token(h)
                fresh.add(h)
            else:
                tokens[h].step += 1
        launches += 1
    assert launches == 60


def _alloc_buffers(num_blocks, rows, width):
    ring = torch.zeros(max(num_blocks, 1), dtype=torch.int32, device=DEV)
    state = torch.zeros(4, dtype=torch.int32, device=DEV)
    row_len = torch.zeros(rows, dtype=torch.int32, device=DEV)
    table = torch.full((rows, width), -1, dtype=torch.int32, device=DEV)
    _lib.call("cdb_block_pool_init", _lib.ptr(ring), _lib.ptr(state), _lib.ptr(row_len), rows, num_blocks, _sp())
    return ring, state, row_len, table


def test_block_allocator_matches_host_fifo_pool():
    rng = random.Random(7)
    num_blocks, rows, width = 300, 24, 40
    ring, state, row_len, table = _alloc_buffers(num_blocks, rows, width)
    host = BlockPool(num_blocks, 16, width)
    live: set[int] = set()
    for _ in range(200):
        if live and rng.random() < 0.3:
            frees = rng.sample(sorted(live), rng.randrange(1, len(live) + 1))
            for s in frees:
                host.release(s)
                live.discard(s)
            f = torch.tensor(frees, dtype=torch.int32, device=DEV)
            _lib.call("cdb_block_free", _lib.ptr(ring), _lib.ptr(state), _lib.ptr(row_len), _lib.ptr(table),
                      table.stride(0), _lib.ptr(f), len(frees), _sp())
        else:
            reqs = [rng.randrange(rows) for _ in range(rng.randrange(1, 8))]
            counts = [rng.randrange(0, 30) for _ in reqs]
            want = []
            for s, c in zip(reqs, counts, strict=True):
                have = len(host.tables.get(s, []))
                ok = c <= host.num_free and have + c <= width
                if ok:
                    assert host.allocate(s, s, c)
                    live.add(s)
                want.append(int(ok))
            s_d = torch.tensor(reqs, dtype=torch.int32, device=DEV)
            c_d = torch.tensor(counts, dtype=torch.int32, device=DEV)
            granted = torch.full((len(reqs),), -1, dtype=torch.int32, device=DEV)
            _lib.call("cdb_block_alloc", _lib.ptr(ring), _lib.ptr(state), _lib.ptr(row_len), _lib.ptr(table),
                      table.stride(0), width, _lib.ptr(s_d), _lib.ptr(c_d), len(reqs), _lib.ptr(granted), _sp())
            torch.cuda.synchronize()
            assert granted.tolist() == want
        torch.cuda.synchronize()
        tab = table.cpu().tolist()
        for s in range(rows):
            blocks = host.tables.get(s, [])
            assert tab[s] == blocks + [-1] * (width - len(blocks)), s
        assert row_len.tolist() == [len(host.tables.get(s, [])) for s in range(rows)]
        assert int(state[1]) == host.num_free
    assert int(state[3]) == host.peak


def test_build_tables_matches_reference_layout():
    rng = random.Random(3)
    num_blocks, rows, width, bs = 512, 16, 12, 16
    ring, state, row_len, table = _alloc_buffers(num_blocks, rows, width)
    host = BlockPool(num_blocks, bs, width)
    lens = {}
    for s in range(rows):
        n = rng.randrange(1, width + 1)
        host.allocate(s, s, n)
        lens[s] = n
    s_d = torch.arange(rows, dtype=torch.int32, device=DEV)
    c_d = torch.tensor([lens[s] for s in range(rows)], dtype=torch.int32, device=DEV)
    granted = torch.zeros(rows, dtype=torch.int32, device=DEV)
    _lib.call("cdb_block_alloc", _lib.ptr(ring), _lib.ptr(state), _lib.ptr(row_len), _lib.ptr(table), table.stride(0),
              width, _lib.ptr(s_d), _lib.ptr(c_d), rows, _lib.ptr(granted), _sp())
    items = rng.sample(range(rows), 11)
    pos = [rng.randrange(0, lens[s] * bs) for s in items]
    bucket = 16
    out = torch.full((bucket, width), 99, dtype=torch.int32, device=DEV)
    cu_q = torch.full((bucket + 1,), 99, dtype=torch.int32, device=DEV)
    cu_k = torch.full((bucket + 1,), 99, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    it_d = torch.tensor(items, dtype=torch.int32, device=DEV)
    pos_d = torch.tensor(pos, dtype=torch.int32, device=DEV)
    _lib.call("cdb_build_tables", _lib.ptr(table), table.stride(0), _lib.ptr(row_len), width, bs, _lib.ptr(it_d),
              _lib.ptr(pos_d), len(items), bucket, _lib.ptr(out), out.stride(0), _lib.ptr(cu_q), _lib.ptr(cu_k),
              _lib.ptr(status), _sp())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    n = len(items)
    want_rows = [host.tables[s] + [-1] * (width - len(host.tables[s])) for s in items] + [[-1] * width] * (bucket - n)
    assert out.tolist() == want_rows
    ks = [0]
    for p in pos:
        ks.append(ks[-1] + p + 1)
    assert cu_k.tolist() == ks + [ks[-1]] * (bucket - n)
    assert cu_q.tolist() == list(range(n + 1)) + [n] * (bucket - n)
    # a position past the row's blocks is reported, not read past
    bad = torch.tensor([lens[items[0]] * bs], dtype=torch.int32, device=DEV)
    _lib.call("cdb_build_tables", _lib.ptr(table), table.stride(0), _lib.ptr(row_len), width, bs, _lib.ptr(it_d),
              _lib.ptr(bad), 1, 1, _lib.ptr(out), out.stride(0), _lib.ptr(cu_q), _lib.ptr(cu_k), _lib.ptr(status),
              _sp())
    torch.cuda.synchronize()
    assert int(status.item()) == 6  # CDB_ERR_INDEX


@pytest.mark.parametrize("policy,slots", [("single", 1), ("first_then_shared", 2), ("depth_indexed", 4)])
def test_schedule_tick_matches_engine_queues(policy, slots):
    """cdb_schedule_tick against the engine's own queue operations (_enqueue, _enqueue_front,
    _pop_recurrent, the coda-first decision), the ones the reference traces pin: 150 ticks of
    routed batches with random exits, prefill and coda successors, and host prefill admissions.
    Every tick's kind and batch, both queues and the refill count must be equal."""

    from collections import deque

    from continuous_depth_batching_b200 import ContinuousDepthBatchingEngine
    from continuous_depth_batching_b200.engine import _Item

    rng = random.Random(slots)
    max_seqs, min_coda, cap, n_items = 12, 3, 256, 4000
    eng = ContinuousDepthBatchingEngine.__new__(ContinuousDepthBatchingEngine)
    eng.cdb_config = SimpleNamespace(kv_policy=policy)
    eng.slots, eng.max_num_seqs = slots, max_seqs
    eng.ready, eng.in_flight, eng.refills, eng.max_queue = deque(), set(), 0, 0
    coda_q: deque = deque()
    items: dict[int, _Item] = {}
    state = torch.zeros(8, dtype=torch.int32, device=DEV)
    ready = torch.zeros(cap, dtype=torch.int32, device=DEV)
    coda = torch.zeros(cap, dtype=torch.int32, device=DEV)
    step = torch.zeros(n_items, dtype=torch.int32, device=DEV)
    out = torch.zeros(2 + max_seqs, dtype=torch.int32, device=DEV)
    _lib.call("cdb_schedule_queues_init", _lib.ptr(state), cap, _sp())
    next_id = 0

    def new_items(k):
        nonlocal next_id
        made = []
        for _ in range(k):
            it = _Item(SimpleNamespace(idx=next_id), 0, None, next_id, -1)
            items[next_id] = it
            made.append(it)
            next_id += 1
        return made

    last_batch: list[_Item] = []
    for tick in range(150):
        exits = [int(rng.random() < 0.35 or it.step == 3) for it in last_batch]
        back = new_items(rng.randrange(0, 4) if tick % 7 == 0 else 0)
        front = new_items(rng.randrange(0, 3))
        admit = int(rng.random() < 0.1)
        # host: the engine's own queue operations in the engine's order
        surv = []
        for it, ex in zip(last_batch, exits, strict=True):
            if ex:
                coda_q.append(it)
            else:
                it.step += 1
                surv.append(it)
        eng._enqueue_front(surv)
        for it in back:
            eng._enqueue(it)
        eng._enqueue_front(front)
        if len(coda_q) >= min_coda:
            kind, batch = 1, [coda_q.popleft() for _ in range(min(max_seqs, len(coda_q)))]
        elif admit:
            kind, batch = 2, []
        elif eng.ready:
            kind, batch = 3, eng._pop_recurrent()
        elif coda_q:
            kind, batch = 1, [coda_q.popleft() for _ in range(min(max_seqs, len(coda_q)))]
        else:
            kind, batch = 0, []
        # device
        d = lambda v, dt=torch.int32: torch.tensor(v if v else [0], dtype=dt, device=DEV)  # noqa: E731
        routed = d([it.hidden for it in last_batch])
        ex_d = d(exits, torch.int8)
        back_d, front_d = d([it.hidden for it in back]), d([it.hidden for it in front])
        _lib.call(
            "cdb_schedule_tick", _lib.ptr(state), _lib.ptr(ready), _lib.ptr(coda), _lib.ptr(step), _lib.ptr(routed),
            _lib.ptr(ex_d), len(last_batch), _lib.ptr(back_d), len(back), _lib.ptr(front_d), len(front), min_coda,
            max_seqs, admit, slots, _lib.ptr(out), _sp(),
        )
        torch.cuda.synchronize()
        o = out.tolist()
        assert o[0] == kind, tick
        assert o[2 : 2 + o[1]] == [it.hidden for it in batch], tick
        st = state.tolist()
        assert ready[: st[1]].tolist() == [it.hidden for it in eng.ready], tick
        assert coda[: st[3]].tolist() == [it.hidden for it in coda_q], tick
        assert st[5] == eng.refills, tick
        assert step[: next_id].tolist() == [items[i].step for i in range(next_id)], tick
        last_batch = batch if kind == 3 else []
