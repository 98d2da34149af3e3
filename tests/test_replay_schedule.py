"""Replayed exit schedules (CPU): each request hands out its recorded depths in order, one per
staged decode token, with its own cursor; an exhausted schedule is an error
(``RequestState.next_synthetic_exit_depth``, reference ``requests.py``)."""

from __future__ import annotations

import pytest

from continuous_depth_batching_b200.engine import _Req


def _req(idx, depths):
    return _Req(idx, [1, 2, 3], 4, depths, set(), [], False)


def test_depths_returned_in_order():
    r = _req(0, [2, 0, 3])
    assert [r.next_depth() for _ in range(3)] == [2, 0, 3]


def test_no_schedule_gives_none():
    assert _req(0, []).next_depth() is None


def test_exhausted_schedule_raises():
    r = _req(0, [1])
    r.next_depth()
    with pytest.raises(RuntimeError, match="exhausted"):
        r.next_depth()


def test_cursors_are_per_request():
    a, b = _req(0, [1, 2]), _req(1, [3, 0])
    assert (a.next_depth(), b.next_depth(), b.next_depth(), a.next_depth()) == (1, 3, 0, 2)
