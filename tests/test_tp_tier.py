"""Host logic of the tensor-parallel CPU tier (kvoff.tp_tier), no GPU."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from kvoff import tp_tier


class SlowEvent:
    """A mailbox event that a reader clears after a few polls."""

    def __init__(self, polls: int):
        self.polls = polls

    def is_set(self) -> bool:
        self.polls -= 1
        return self.polls > 0


def test_wait_taken_returns_once_every_rank_cleared_its_event():
    runner = SimpleNamespace(event=[SlowEvent(3), SlowEvent(50)])
    tp_tier.wait_taken(runner)
    assert all(not e.is_set() for e in runner.event)


def test_wait_taken_times_out_when_a_rank_never_reads():
    stuck = SimpleNamespace(is_set=lambda: True)
    with pytest.raises(RuntimeError, match="did not take"):
        tp_tier.wait_taken(SimpleNamespace(event=[stuck]), timeout=0.05)


def test_wait_taken_ignores_runners_without_mailbox_events():
    tp_tier.wait_taken(SimpleNamespace())
    tp_tier.wait_taken(SimpleNamespace(event=SimpleNamespace(is_set=lambda: True)))


def test_dispatch_rules():
    assert tp_tier.dispatch(SimpleNamespace(rank=0), "save", [1], [0]) is None
    follower = SimpleNamespace(rank=1)
    with pytest.raises(RuntimeError, match="before init"):
        tp_tier.dispatch(follower, "save", [1], [0])


def test_send_calls_every_rank_then_waits():
    calls = []
    runner = SimpleNamespace(call=lambda *a: calls.append(a), event=[SlowEvent(2)])
    tp_tier.send(runner, "grow", 4)
    assert calls == [("kvoff_tier", "grow", 4)]
