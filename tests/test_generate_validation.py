"""generate_batch input checks (CPU): the token-level inputs and the replay schedule are refused
with the reference's messages (``continuous_api.py:1766-1836``) before anything is scheduled."""

from __future__ import annotations

import pytest

from continuous_depth_batching_b200 import ContinuousDepthBatchingConfig, ContinuousDepthBatchingEngine

E = ContinuousDepthBatchingEngine


def test_scalar_and_list_lengths_accepted():
    E._validate_generate_inputs([[1, 2], [3]], 4)
    E._validate_generate_inputs([[1, 2], [3]], [4, 2])


@pytest.mark.parametrize(
    "prompts,new,match",
    [
        ([[1], [2], [3]], [4, 4], "has 2 entries but there are 3 prompts"),
        ([[1], [2]], [4, 0], r"must be >= 1 for every request, but got <1 at indices \[1\]"),
        ([[1]], 0, "must be positive, but got 0"),
        ([[1], []], 4, r"empty prompts at indices \[1\]"),
        ([], 4, "at least one prompt"),
    ],
)
def test_bad_inputs_refused(prompts, new, match):
    with pytest.raises(ValueError, match=match):
        E._validate_generate_inputs(prompts, new)


def _engine(**cfg):
    eng = E.__new__(E)
    eng.cdb_config = ContinuousDepthBatchingConfig(max_recurrent_steps=4, **cfg).get_resolved()
    return eng


@pytest.mark.parametrize(
    "cfg,depths,match",
    [
        ({}, [[0, 1]], "requires cdb_config.synthetic_exit_replay=True"),
        ({"synthetic_exit_replay": True}, [[0, 1], [0]], "has 2 entries but there are 1 requests"),
        ({"synthetic_exit_replay": True}, [[0]], r"exit_depths\[0\] has 1 entries but the request stages 2"),
        ({"synthetic_exit_replay": True}, [[0, 4]], r"value 4 is out of range \[0, 4\); values are 0-based"),
        (
            {"synthetic_exit_replay": True, "kv_policy": "depth_indexed", "use_async_batching": False},
            [[2, 3]],
            "must write all static KV slots before exit: kv_slots_per_layer=4, exit step 3",
        ),
        (
            {"synthetic_exit_replay": True, "kv_policy": "first_then_shared", "use_async_batching": False},
            [[0, 1]],
            "kv_slots_per_layer=2, exit step 1",
        ),
    ],
)
def test_bad_replay_schedules_refused(cfg, depths, match):
    with pytest.raises(ValueError, match=match):
        _engine(**cfg)._validate_exit_depths([[5]], [3], depths)


def test_replay_schedules_accepted():
    # delayed timing writes one more slot before a replayed exit; copy-on-exit accepts any depth
    _engine(synthetic_exit_replay=True, kv_policy="first_then_shared")._validate_exit_depths([[5]], [3], [[0, 1]])
    _engine(synthetic_exit_replay=True, kv_policy="last_exited", kv_pressure_mode="reserve")._validate_exit_depths(
        [[5]], [3], [[0, 0]]
    )
    _engine(synthetic_exit_replay=True)._validate_exit_depths([[5]], [3], None)


def test_model_len_caps_and_refusals():
    from continuous_depth_batching_b200.engine import cap_max_new_tokens_to_model_len as cap

    mnt = [4, 4, 4]
    assert cap([[1], [2], [3]], mnt, None) is mnt
    assert cap([[0] * 2, [0] * 8, [0] * 3], [5, 5, 5], 10) == [5, 2, 5]
    assert cap([[0] * 9], [16], 10) == [1]  # one below the limit: exactly one token
    with pytest.raises(ValueError, match=r"1 prompt\(s\) have length >= max_model_len \(10\).*request 1 \(len 10\)"):
        cap([[0] * 5, [0] * 10], [4, 4], 10)
    with pytest.raises(ValueError, match="max_model_len"):
        cap([[0] * 11], [4], 10)


def test_replay_schedule_checked_against_capped_lengths():
    eng = _engine(synthetic_exit_replay=True, max_model_len=12)
    # the 10-token prompt leaves 2 tokens, so its schedule holds max_new - 1 = 1 depth
    assert eng._validate([[1] * 10], 5, [[0]], None) == [2]
    with pytest.raises(ValueError, match="stages 1 decode tokens"):
        eng._validate([[1] * 10], 5, [[0, 0, 0, 0]], None)
