"""LoopedKvLayout (CPU): the cache-layer numbering every attention launch and exit copy uses
(``kv_cache_policy.py:135-258``): prelude, then core slot-major, then coda."""

from __future__ import annotations

import pytest

from continuous_depth_batching_b200.kv_cache import LoopedKvLayout


def _huginn(policy, slots=None, steps=8):
    return LoopedKvLayout(num_prelude_layers=2, num_core_layers=4, num_coda_layers=2, total_recurrent_steps=steps,
                          policy=policy, requested_slots=slots)


@pytest.mark.parametrize(
    "policy,slots,cache_layers",
    [("single", None, 8), ("depth_indexed", None, 36), ("last_exited", None, 36), ("first_then_shared", None, 12),
     ("first_then_shared", 3, 16)],
)
def test_cache_layer_count(policy, slots, cache_layers):
    assert _huginn(policy, slots).num_cache_layers == cache_layers


@pytest.mark.parametrize("policy", ["single", "depth_indexed", "first_then_shared"])
def test_stage_indices_disjoint_and_dense(policy):
    lay = _huginn(policy)
    idx = [lay.prelude_layer_index(i) for i in range(2)]
    idx += [lay.core_slot_layer_index(s, i) for s in range(lay.slots_per_layer) for i in range(4)]
    idx += [lay.coda_layer_index(i) for i in range(2)]
    assert sorted(idx) == list(range(lay.num_cache_layers))
    assert idx[:2] == [0, 1] and idx[-2:] == [lay.num_cache_layers - 2, lay.num_cache_layers - 1]


@pytest.mark.parametrize(
    "policy,expected",
    [("single", [0] * 8), ("depth_indexed", list(range(8))), ("first_then_shared", [0] + [1] * 7)],
)
def test_core_slot_per_step(policy, expected):
    lay = _huginn(policy)
    assert [lay.slot_for_step(s) for s in range(8)] == expected
    assert [lay.core_layer_index(3, s) for s in range(8)] == [2 + slot * 4 + 3 for slot in expected]


@pytest.mark.parametrize("policy", ["single", "depth_indexed", "last_exited"])
def test_ouro_indexing_is_slot_times_layers_plus_layer(policy):
    lay = LoopedKvLayout(num_prelude_layers=0, num_core_layers=24, num_coda_layers=0, total_recurrent_steps=4,
                         policy=policy)
    for s in range(4):
        for layer in (0, 11, 23):
            assert lay.core_layer_index(layer, s) == lay.slot_for_step(s) * 24 + layer


def test_exit_copy_groups_target_every_deeper_slot():
    lay = LoopedKvLayout(num_prelude_layers=0, num_core_layers=3, num_coda_layers=0, total_recurrent_steps=4,
                         policy="last_exited")
    assert lay.exit_copy_layer_groups(1) == [(3, [6, 9]), (4, [7, 10]), (5, [8, 11])]
    assert lay.exit_copy_layer_groups(3) == []  # no deeper slot after the last step
    assert _huginn("last_exited").exit_copy_layer_groups(0)[0] == (2, [2 + 4 * s for s in range(1, 8)])


@pytest.mark.parametrize("policy", ["single", "first_then_shared"])
def test_exit_copy_groups_empty_for_slot_sharing_layouts(policy):
    lay = _huginn(policy)
    assert lay.exit_copy_layer_groups(lay.total_recurrent_steps - 2) == []


def test_out_of_range_rejected():
    lay = _huginn("depth_indexed")
    with pytest.raises(ValueError, match="prelude layer"):
        lay.prelude_layer_index(2)
    with pytest.raises(ValueError, match="core layer"):
        lay.core_layer_index(4, 0)
    with pytest.raises(ValueError, match="coda layer"):
        lay.coda_layer_index(-1)
    with pytest.raises(ValueError, match="recurrent_step"):
        lay.slot_for_step(8)
    with pytest.raises(ValueError, match="exceeds total_recurrent_steps"):
        _huginn("first_then_shared", slots=9)
