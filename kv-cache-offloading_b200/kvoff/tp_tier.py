"""Per-rank CPU tier under tensor parallelism.

With tensor parallelism each rank's KV pool holds its own KV heads of every
block ([2, L, NB, BS, H / tp, D], nanovllm/engine/model_runner.py:110), so each
rank saves and restores its own heads, over its own PCIe link into its own
pinned slab, and no collective is needed. The CPUBlockCache on rank 0 (the
leader) keeps the bookkeeping and mirrors every device operation to the other
ranks through the engine's runner RPC, where a follower cache replays it on
that rank's shard with the same slot numbers and the same stream ordering.

Engine side: the runner forwards one method, on every rank,

    def kvoff_tier(self, op, *args):
        from kvoff.tp_tier import dispatch
        return dispatch(self, op, *args)

The reference runner's RPC (ModelRunner.call / write_shm) has a one-message
mailbox, so after each message the leader waits until every other rank has
taken it (their mailbox events are cleared) before sending the next one.
"""

from __future__ import annotations

import time

_FOLLOWERS: dict[int, object] = {}
SEND_TIMEOUT_S = 120.0


def dispatch(runner, op: str, *args):
    """Apply a leader's operation on this rank (rank 0 does its own work)."""
    if getattr(runner, "rank", 0) == 0:
        return None
    key = id(runner)
    if op == "init":
        from kvoff.cpu_prefix_cache import CPUBlockCache

        _FOLLOWERS[key] = CPUBlockCache._follower(runner, *args)
        return None
    cache = _FOLLOWERS.get(key)
    if cache is None:
        raise RuntimeError(f"kvoff tier operation {op!r} before init on rank {runner.rank}")
    if op == "close":
        cache.close()
        del _FOLLOWERS[key]
        return None
    handler = getattr(cache, f"_tp_{op}", None)
    if handler is None:
        raise ValueError(f"unknown kvoff tier operation {op!r}")
    return handler(*args)


def send(runner, op: str, *args) -> None:
    """Leader side: run `op` on every rank, then wait until all ranks took it."""
    runner.call("kvoff_tier", op, *args)
    wait_taken(runner)


def wait_taken(runner, timeout: float = SEND_TIMEOUT_S) -> None:
    """Block until the other ranks have consumed the last RPC message.

    The reference runner signals one multiprocessing Event per other rank and
    each rank clears its event once it has read the message. Runners without
    such events (single process, or a synchronous RPC) return at once.
    """
    events = getattr(runner, "event", None)
    if not isinstance(events, (list, tuple)):
        return
    deadline = time.monotonic() + timeout
    while any(event.is_set() for event in events):
        if time.monotonic() > deadline:
            raise RuntimeError("tensor-parallel ranks did not take the CPU tier message")
        time.sleep(0)
