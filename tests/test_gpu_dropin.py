"""The drop-in CPUBlockCache on a CUDA pool (native copy path), reference-style.

Restates the reference's CUDA scenarios (bench/test_cpu_prefix_cache.py,
bench/test_cpu_cache_optimizations.py, bench/test_automatic_cpu_cache.py):
byte-exact BF16 round trips of arbitrary bit patterns for every copy method,
FP8 slots bit-exact against the oracle for both FP8 methods, and the stream
ordering races provoked by delaying copies with a bounded torch.cuda._sleep on
the cache's own streams (slabs poisoned with 0xAB so an early read shows).
Failures are injected on the host through kvoff_debug_fail_next.
"""

from __future__ import annotations

import gc

import numpy as np
import pytest
import torch

import kvoff
from fake_engine import FakeEngine, bits_u16, block_bytes
from oracle import oracle

pytestmark = pytest.mark.gpu

SLEEP_CYCLES = 20_000_000  # about 10 ms at B200 clocks


def arbitrary_pool(shape, device) -> torch.Tensor:
    n = int(np.prod(shape))
    raw = torch.arange(2 * n, dtype=torch.int64).remainder(251).to(torch.uint8)
    return raw.view(torch.bfloat16).reshape(shape).to(device)


def finite_pool(shape, device, seed=0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g)
    x[..., 3] *= 20  # an outlier channel
    return x.to(torch.bfloat16).to(device)


def per_block(pool) -> int:
    return pool[:, :, 0].numel() * pool.element_size()


def slow_copies(cache, names=("save_block", "_copy_entry")):
    """Enqueue a bounded spin on the cache's copy streams before each call."""
    streams = {"save_block": cache._copy_stream, "_copy_entry": cache._restore_stream}
    for name in names:
        original, stream = getattr(cache, name), streams[name]

        def delayed(*args, _original=original, _stream=stream, **kwargs):
            with torch.cuda.stream(_stream):
                torch.cuda._sleep(SLEEP_CYCLES)
            return _original(*args, **kwargs)

        setattr(cache, name, delayed)


SHAPES = [(2, 2, 4, 256, 1, 4), (2, 3, 6, 256, 8, 128)]


@pytest.mark.parametrize("method", ["staged", "engine", "tma", "sm"])
@pytest.mark.parametrize("shape", SHAPES)
def test_bf16_round_trip_byte_exact(cuda, monkeypatch, method, shape):
    monkeypatch.setenv("KVOFF_BF16_SAVE", method)
    monkeypatch.setenv("KVOFF_BF16_RESTORE", method)
    engine = FakeEngine(arbitrary_pool(shape, cuda))
    m = engine.manager
    key = m.publish(1)
    expected = block_bytes(engine.pool, 1)
    cache = engine.create_cpu_prefix_cache(2 * per_block(engine.pool), split_streams=True)
    assert cache.save_block(key)
    m.forget(key)
    cache.before_block_reuse(1)  # the engine's protocol: the save must read block 1 first
    engine.pool.fill_(-7)
    target = cache.restore_block(key)
    cache.synchronize()
    assert torch.equal(block_bytes(engine.pool, target), expected)
    payload, _ = cache._slot_view(cache._entries[key].slot)
    assert torch.equal(payload.view(torch.uint8).reshape(-1), expected.reshape(-1))


@pytest.mark.parametrize("mode", ["staged", "mapped"])
@pytest.mark.parametrize("shape", SHAPES)
def test_fp8_slots_bit_exact_and_within_bound(cuda, monkeypatch, mode, shape):
    monkeypatch.setenv("KVOFF_FP8_SAVE", mode)
    monkeypatch.setenv("KVOFF_FP8_RESTORE", mode)
    engine = FakeEngine(finite_pool(shape, cuda))
    m = engine.manager
    keys = [m.publish(b) for b in (2, 0)]
    pool = engine.pool
    source = bits_u16(pool)
    cache = engine.create_cpu_prefix_cache(4 * per_block(pool), fp8=True, split_streams=True)
    numel = pool[:, :, 0].numel()
    assert cache.block_bytes == numel + numel // pool.shape[-1] * pool.element_size()
    for key in keys:
        assert cache.save_block(key)
    cache.synchronize()
    want_p, want_s = oracle.fp8_save_blocks(source, [2, 0])
    for i, key in enumerate(keys):
        entry = cache._entries[key]
        assert np.array_equal(entry.kv.view(torch.uint8).numpy(), want_p[i])
        assert np.array_equal(bits_u16(entry.scale), want_s[i])
    for key in keys:
        m.forget(key)
    m.free_block_ids.rotate(-3)  # restore into blocks 3 and 4
    targets = [cache.restore_block(k) for k in keys]
    cache.synchronize()
    oracle.fp8_restore_blocks(source, targets, want_p, want_s)
    assert np.array_equal(bits_u16(pool), source)
    src = pool[:, :, 0].float()
    back = pool[:, :, targets[1]].float()
    assert torch.all((back - src).abs() <= src.abs().amax(-1, keepdim=True) / 16)
    assert cache.stats["restored_blocks"] == 2


def split_stream_cache(pool, fp8=False):
    engine = FakeEngine(pool)
    key = engine.manager.publish(1)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), split_streams=True,
                                           preallocate=True, fp8=fp8)
    assert cache._restore_stream is not cache._copy_stream
    for slab in cache._slabs:
        slab.view(torch.uint8).fill_(0xAB)  # an early read cannot see matching bytes
    return engine, key, cache


@pytest.mark.parametrize("slow", [False, True])
@pytest.mark.parametrize("fp8", [False, True])
def test_restore_waits_for_its_save(cuda, slow, fp8):
    engine, key, cache = split_stream_cache(finite_pool(SHAPES[1], cuda), fp8)
    if slow:
        slow_copies(cache, ["save_block"])  # a restore that ignored the save would overtake it
    source = bits_u16(engine.pool)
    expected = block_bytes(engine.pool, 1)
    assert cache.save_block(key)
    engine.manager.forget(key)
    target = cache.restore_block(key)
    cache.synchronize()
    if fp8:
        p, s = oracle.fp8_save_blocks(source, [1])
        oracle.fp8_restore_blocks(source, [target], p, s)
        assert np.array_equal(bits_u16(engine.pool[:, :, target]), source[:, :, target])
    else:
        assert torch.equal(block_bytes(engine.pool, target), expected)


@pytest.mark.parametrize("slow", [False, True])
def test_slot_reuse_waits_for_pending_restore(cuda, slow):
    engine, key, cache = split_stream_cache(arbitrary_pool(SHAPES[1], cuda))
    m = engine.manager
    expected = block_bytes(engine.pool, 1)
    assert cache.save_block(key)
    cache.synchronize()
    m.forget(key)
    if slow:
        slow_copies(cache, ["_copy_entry"])  # a fast save would overwrite the slot first
    entry = cache._entries[key]
    target = m.restore_cached_block(key, entry.token_ids,
                                    lambda b: cache._copy_entry(entry, b, wait=False))
    assert cache.discard(key)
    other = next(i for i in range(len(m.blocks)) if i != target)
    engine.pool[:, :, other].fill_(7)
    other_key = m.publish(other)
    assert cache.save_block(other_key)  # reuses the slot the restore is still reading
    cache.synchronize()
    cache.before_block_use(target)
    assert torch.equal(block_bytes(engine.pool, target), expected)
    payload, _ = cache._slot_view(0)
    assert torch.equal(payload.view(torch.uint8).reshape(-1),
                       block_bytes(engine.pool, other).reshape(-1))


def test_block_reuse_waits_for_pending_save(cuda):
    """A recycled block is rewritten only after its save finished (before_block_reuse)."""
    engine = FakeEngine(arbitrary_pool(SHAPES[1], cuda))
    m = engine.manager
    key = m.publish(0)  # block 0 is first in the free list: the next allocation recycles it
    expected = block_bytes(engine.pool, 0)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), automatic=True,
                                           split_streams=True)
    slow_copies(cache, ["save_block"])
    block = m.allocate_block()  # preserve-before-recycle saves it, then orders reuse
    assert block == 0 and key in cache
    engine.pool[:, :, block].fill_(3)  # the compute stream's next write of the block
    cache.synchronize()
    payload, _ = cache._slot_view(cache._entries[key].slot)
    assert torch.equal(payload.view(torch.uint8).reshape(-1), expected.reshape(-1))


def _reuse_while_draining(engine, cache, key, block):
    """Save `block` while the copy stream sleeps, then reuse it (before_block_reuse
    and the next writer). Returns (ms to the writer's end, ms to the drain's end),
    both from the start of the sleep, on device clocks. The sequence runs once
    untimed first: a first launch in a process can synchronize implicitly while
    its kernel module loads, which would hide what the ordering alone does.

    The garbage collector is off while the sequence is enqueued: a collection
    there could free an earlier test's pinned slab, and unpinning waits for the
    device (the sleep included), which would delay the writer's enqueue on the
    host rather than its ordering on the device."""
    original = engine.pool[:, :, block].clone()
    gc.collect()
    gc.disable()
    try:
        for timed in (False, True):
            slept = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(cache._copy_stream):
                slept.record()
                if timed:
                    torch.cuda._sleep(5 * SLEEP_CYCLES)
            assert cache.save_block(key)
            drained = torch.cuda.Event(enable_timing=True)
            drained.record(cache._copy_stream)  # after the drain to host
            cache.before_block_reuse(block)
            engine.pool[:, :, block].fill_(5)  # the block's next writer
            written = torch.cuda.Event(enable_timing=True)
            written.record(torch.cuda.current_stream(engine.pool.device))
            cache.synchronize()
            torch.cuda.synchronize()
            if not timed:
                assert cache.discard(key)
                engine.pool[:, :, block].copy_(original)
    finally:
        gc.enable()
    return slept.elapsed_time(written), slept.elapsed_time(drained)


def test_fp8_block_reuse_waits_for_the_read_not_the_drain(cuda, monkeypatch):
    """Staged FP8 (pipelined: KVOFF_COPY_YIELD=0): before_block_reuse waits for
    the quantize kernel alone.

    The copy stream sleeps before the save, so the drain to host is still
    queued when the block is overwritten; the writer must finish long before
    the drain, and the slot must still hold the block as it was when saved.
    """
    monkeypatch.setenv("KVOFF_COPY_YIELD", "0")
    engine = FakeEngine(finite_pool(SHAPES[1], cuda, seed=2))
    m = engine.manager
    key = m.publish(3)
    source = bits_u16(engine.pool)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), fp8=True,
                                           split_streams=True, preallocate=True)
    assert cache._modes["fp8_save"] == "staged"
    write_ms, drain_ms = _reuse_while_draining(engine, cache, key, 3)
    assert write_ms < drain_ms / 2, (write_ms, drain_ms)
    want_p, want_s = oracle.fp8_save_blocks(source, [3])
    entry = cache._entries[key]
    assert np.array_equal(entry.kv.view(torch.uint8).numpy(), want_p[0])
    assert np.array_equal(bits_u16(entry.scale), want_s[0])


def test_bf16_staged_block_reuse_waits_for_the_gather_not_the_drain(cuda, monkeypatch):
    """Staged BF16 (pipelined: KVOFF_COPY_YIELD=0): before_block_reuse waits for the
    gather kernel alone, as for staged FP8; the slot still receives the block
    as it was when saved."""
    monkeypatch.setenv("KVOFF_COPY_YIELD", "0")
    engine = FakeEngine(arbitrary_pool(SHAPES[1], cuda))
    m = engine.manager
    key = m.publish(3)
    expected = block_bytes(engine.pool, 3)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), split_streams=True,
                                           preallocate=True)
    assert cache._modes["bf16_save"] == "staged"
    write_ms, drain_ms = _reuse_while_draining(engine, cache, key, 3)
    assert write_ms < drain_ms / 2, (write_ms, drain_ms)
    payload, _ = cache._slot_view(cache._entries[key].slot)
    assert torch.equal(payload.view(torch.uint8).reshape(-1), expected.reshape(-1))


@pytest.mark.parametrize("split", [True, False])
def test_fp8_back_to_back_restores_match_oracle(cuda, split):
    """Per-block staged restores share two staging halves without a join per
    call; a batched restore on the same stream then grows the staging. Without
    split streams, saves and restores also share one kernel stream and ring."""
    shape = (2, 3, 16, 256, 8, 128)
    engine = FakeEngine(finite_pool(shape, cuda, seed=6))
    m = engine.manager
    sources = [9, 2, 5, 7, 11, 0]
    keys = [m.publish(b) for b in sources]
    pool = engine.pool
    source = bits_u16(pool)
    cache = engine.create_cpu_prefix_cache(8 * per_block(pool), fp8=True, split_streams=split)
    assert all(cache.save_block(k) for k in keys)
    entries = [cache._entries[k] for k in keys]
    want_p, want_s = oracle.fp8_save_blocks(source, sources)
    expected = source.copy()
    for rounds, targets in enumerate(([1, 3, 4, 6, 8, 10], [12, 13, 14, 15, 1, 3])):
        if rounds == 0:
            with torch.cuda.stream(cache._restore_stream):
                torch.cuda._sleep(SLEEP_CYCLES)  # the copies queue up behind a slow start
            for e, b in zip(entries, targets):
                cache._copy_entry(e, b, wait=False)
        else:
            cache._copy_entries(entries, targets, wait=False)
            # Saves interleaved with pending restores: a block being restored is
            # saved again only after its restore has written it.
            again = m.publish(targets[0])
            assert cache.save_block(again)
        for b in targets:
            cache.before_block_use(b)
        oracle.fp8_restore_blocks(expected, targets, want_p, want_s)
        assert np.array_equal(bits_u16(pool), expected)
    cache.synchronize()
    # The block saved right after its restore holds the restored values, whose
    # FP8 slot is the original slot again (restore -> save is idempotent).
    entry = cache._entries[again]
    assert np.array_equal(entry.kv.view(torch.uint8).numpy(), want_p[0])
    assert np.array_equal(bits_u16(entry.scale), want_s[0])


@pytest.mark.parametrize("method", ["staged", "engine"])
def test_injected_failures_roll_back_and_retry_is_byte_exact(cuda, monkeypatch, method):
    monkeypatch.setenv("KVOFF_BF16_SAVE", method)
    monkeypatch.setenv("KVOFF_BF16_RESTORE", method)
    op = {"staged": "copy_blocks_staged", "engine": "copy_blocks"}[method]
    engine = FakeEngine(arbitrary_pool(SHAPES[1], cuda))
    m = engine.manager
    key = m.publish(1)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool))
    expected = block_bytes(engine.pool, 1)
    kvoff.debug_fail_next(op, 1)
    with pytest.raises(RuntimeError, match="injected"):
        cache.save_block(key)
    assert len(cache) == cache.bytes_used == 0 and key in m.hash_to_block_id
    assert cache.save_block(key)
    m.forget(key)
    kvoff.debug_fail_next(op, 1)
    with pytest.raises(kvoff.KvoffError, match="injected"):
        cache.restore_block(key)
    assert key in cache and key not in m.hash_to_block_id
    assert sorted(m.free_block_ids) == list(range(len(m.blocks))) and not m.used_block_ids
    target = cache.restore_block(key)
    cache.synchronize()
    assert torch.equal(block_bytes(engine.pool, target), expected)


def test_fp8_injected_failure_on_staged_save(cuda):
    engine = FakeEngine(finite_pool(SHAPES[1], cuda))
    key = engine.manager.publish(2)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), fp8=True)
    kvoff.debug_fail_next("fp8_save_blocks_staged", 1)
    with pytest.raises(RuntimeError, match="injected"):
        cache.save_block(key)
    assert len(cache) == 0 and cache._free_slots
    assert cache.save_block(key)


@pytest.mark.parametrize("fp8", [False, True])
def test_measure_restore_s_per_block(cuda, fp8):
    engine = FakeEngine(finite_pool(SHAPES[1], cuda))
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), fp8=fp8, split_streams=True)
    seconds = cache.measure_restore_s_per_block(repeats=4)
    assert 0 < seconds < 1.0
    batched = cache.measure_restore_s_per_block(repeats=2, batch=8)
    assert 0 < batched < 1.0
    with pytest.raises(ValueError):
        cache.measure_restore_s_per_block(batch=0)


def test_prefetch_restore_orders_first_use(cuda):
    engine = FakeEngine(arbitrary_pool(SHAPES[1], cuda))
    m = engine.manager
    key = m.publish(1)
    expected = block_bytes(engine.pool, 1)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), automatic=True,
                                           prefetch=True, split_streams=True)
    assert cache.save_block(key)
    cache.synchronize()
    m.forget(key)
    slow_copies(cache, ["_copy_entry"])
    entry = cache._entries[key]
    target = m.restore_cached_block(key, entry.token_ids,
                                    lambda b: cache._copy_entry(entry, b, wait=False))
    m.acquire_block(target)  # first reader: waits for the pending restore
    got = engine.pool[:, :, target].contiguous().view(torch.uint8).cpu()
    assert torch.equal(got, expected)


@pytest.mark.parametrize("modes", [("staged", "staged"), ("staged", "engine"), ("mapped", "sm"),
                                   ("staged", "tma")])
@pytest.mark.parametrize("fp8", [False, True])
def test_batched_calls_match_per_block_calls(cuda, monkeypatch, modes, fp8):
    fp8_mode, bf16_mode = modes
    for key in ("KVOFF_FP8_SAVE", "KVOFF_FP8_RESTORE"):
        monkeypatch.setenv(key, fp8_mode)
    for key in ("KVOFF_BF16_SAVE", "KVOFF_BF16_RESTORE"):
        monkeypatch.setenv(key, bf16_mode)
    shape = (2, 3, 10, 256, 8, 128)
    results = []
    for batched in (False, True):
        engine = FakeEngine(finite_pool(shape, cuda, seed=4))
        m = engine.manager
        keys = [m.publish(b) for b in (9, 2, 5, 7)]
        cache = engine.create_cpu_prefix_cache(6 * per_block(engine.pool), fp8=fp8,
                                               split_streams=True)
        if batched:
            assert cache.save_blocks(keys) == [True] * 4
        else:
            assert all(cache.save_block(k) for k in keys)
        entries = [cache._entries[k] for k in keys]
        targets = [0, 1, 3, 4]
        if batched:
            cache._copy_entries(entries, targets, wait=False)
        else:
            for e, b in zip(entries, targets):
                cache._copy_entry(e, b, wait=False)
        for b in targets:
            cache.before_block_use(b)
        cache.synchronize()
        results.append((bits_u16(engine.pool),
                        [e.kv.view(torch.uint8).clone() for e in entries]))
    assert np.array_equal(results[0][0], results[1][0])
    assert all(torch.equal(a, b) for a, b in zip(results[0][1], results[1][1]))


def test_batched_restore_waits_for_its_saves(cuda):
    engine = FakeEngine(arbitrary_pool((2, 3, 8, 256, 8, 128), cuda))
    m = engine.manager
    keys = [m.publish(b) for b in (1, 2, 3)]
    expected = [block_bytes(engine.pool, b) for b in (1, 2, 3)]
    cache = engine.create_cpu_prefix_cache(3 * per_block(engine.pool), split_streams=True,
                                           preallocate=True)
    for slab in cache._slabs:
        slab.view(torch.uint8).fill_(0xAB)
    with torch.cuda.stream(cache._copy_stream):
        torch.cuda._sleep(SLEEP_CYCLES)
    assert cache.save_blocks(keys) == [True] * 3
    cache._copy_entries([cache._entries[k] for k in keys], [5, 6, 7])
    cache.synchronize()
    for b, want in zip((5, 6, 7), expected):
        assert torch.equal(block_bytes(engine.pool, b), want)
