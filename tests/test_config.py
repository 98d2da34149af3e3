"""ContinuousDepthBatchingConfig against the reference's own validation (CPU).

``tests/golden/make_config_cases.py`` ran the reference's config over 46 settings and recorded,
for each, the exception (type and message) or the resolved KV slot count, and whether the
reference's ExitPolicy accepts the threshold for Ouro's cumulative hazard and Huginn's direct
threshold. This package must give the same outcome for every case. The one deliberate difference
is also checked: the paged-attention kernels are built for 16-token blocks.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from continuous_depth_batching_b200 import ContinuousDepthBatchingConfig
from continuous_depth_batching_b200.config import validate_exit_threshold
from continuous_depth_batching_b200.kv_cache import copies_exit_kv, kv_slot_for_step, resolve_kv_slots_per_layer

CASES = json.loads((Path(__file__).resolve().parent / "golden" / "config_cases.json").read_text())["cases"]


def _outcome(fn) -> str:
    try:
        fn()
    except Exception as e:  # noqa: BLE001 - the outcome is compared
        return f"{type(e).__name__}: {e}"
    return "ok"


@pytest.mark.parametrize("case", CASES, ids=[json.dumps(c["kwargs"]) for c in CASES])
def test_config_validation_matches_reference(case):
    kw = case["kwargs"]
    if "error" in case:
        with pytest.raises(Exception) as info:
            ContinuousDepthBatchingConfig(**kw).get_resolved()
        assert type(info.value).__name__ == case["error"]["type"]
        assert str(info.value) == case["error"]["message"]
        return
    resolved = ContinuousDepthBatchingConfig(**kw).get_resolved()
    assert resolved.kv_slots_per_layer == case["kv_slots_per_layer"]
    thr = resolved.exit_threshold
    assert _outcome(lambda: validate_exit_threshold(thr, "hazard")) == case["exit_policy"]["ouro"]
    assert _outcome(lambda: validate_exit_threshold(thr, "direct")) == case["exit_policy"]["huginn"]


def test_block_size_other_than_16_is_refused():
    with pytest.raises(NotImplementedError, match="block_size=16"):
        ContinuousDepthBatchingConfig(block_size=32, max_recurrent_steps=4).get_resolved()


@pytest.mark.parametrize(
    "policy,slots,expected",
    [
        ("single", 1, [0, 0, 0, 0]),
        ("depth_indexed", 4, [0, 1, 2, 3]),
        ("last_exited", 4, [0, 1, 2, 3]),
        ("first_then_shared", 2, [0, 1, 1, 1]),
        ("first_then_shared", 3, [0, 1, 2, 2]),
    ],
)
def test_kv_slot_per_step(policy, slots, expected):
    """Recurrent step -> KV slot (kv_cache_policy.py, LoopedKvLayout core slots)."""

    assert resolve_kv_slots_per_layer(policy, total_recurrent_steps=4, requested_slots=slots) == slots
    assert [kv_slot_for_step(s, policy=policy, slots_per_layer=slots) for s in range(4)] == expected
    assert copies_exit_kv(policy) == (policy == "last_exited")
