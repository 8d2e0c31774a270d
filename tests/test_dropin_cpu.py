"""Host logic of the drop-in CPUBlockCache on CPU pools (no GPU).

Mirrors the scenarios of the reference tests for the CPU tier
(bench/test_cpu_prefix_cache.py, bench/test_cpu_cache_optimizations.py):
byte-exact round trips of arbitrary bit patterns, the FP8 size formula and
error bound, budget / dedup / discard / close semantics, slab growth and slot
reuse without allocation, publish-after-copy and rollback on copy failure.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from fake_engine import FakeEngine, bits_u16, block_bytes
from kvoff import cpu_prefix_cache as cpc
from oracle import oracle

SHAPE = (2, 2, 4, 256, 1, 4)  # the reference tests' tiny pool: L=2, H=1, D=4


def arbitrary_pool(shape=SHAPE) -> torch.Tensor:
    n = int(np.prod(shape))
    raw = torch.arange(2 * n, dtype=torch.int64).remainder(256).to(torch.uint8)
    return raw.view(torch.bfloat16).reshape(shape).clone()


def finite_pool(shape=SHAPE) -> torch.Tensor:
    return torch.arange(int(np.prod(shape))).remainder(251).to(torch.bfloat16).reshape(shape)


def per_block(pool: torch.Tensor) -> int:
    return pool[:, :, 0].numel() * pool.element_size()


def test_round_trip_is_byte_exact_for_arbitrary_bits():
    engine = FakeEngine(arbitrary_pool())
    key = engine.manager.publish(1)
    expected = block_bytes(engine.pool, 1)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool))
    assert cache.save_block(key)
    assert key in cache and len(cache) == 1
    assert cache.bytes_used == cache.block_bytes == cache.max_bytes
    engine.manager.forget(key)
    engine.pool.fill_(-7)
    target = cache.restore_block(key)
    assert torch.equal(block_bytes(engine.pool, target), expected)
    assert engine.manager.hash_to_block_id[key] == target
    assert cache.stats == {"saved_blocks": 1, "restored_blocks": 1, "budget_skips": 0}


def test_fp8_slots_match_the_oracle_and_bound():
    engine = FakeEngine(finite_pool())
    pool = engine.pool
    keys = [engine.manager.publish(b) for b in (2, 0)]
    cache = engine.create_cpu_prefix_cache(4 * per_block(pool), fp8=True)
    numel = pool[:, :, 0].numel()
    assert cache.block_bytes == numel + numel // pool.shape[-1] * pool.element_size()
    source = bits_u16(pool)
    for key in keys:
        assert cache.save_block(key)
    want_p, want_s = oracle.fp8_save_blocks(source, [2, 0])
    for i, key in enumerate(keys):
        entry = cache._entries[key]
        assert np.array_equal(entry.kv.view(torch.uint8).numpy(), want_p[i])
        assert np.array_equal(bits_u16(entry.scale), want_s[i])
    for key in keys:
        engine.manager.forget(key)
    engine.manager.free_block_ids.rotate(-1)  # restore into 1 and 2
    targets = [cache.restore_block(k) for k in keys]
    oracle.fp8_restore_blocks(source, targets, want_p, want_s)
    assert np.array_equal(bits_u16(pool), source)
    src = pool[:, :, 0].float()
    back = pool[:, :, targets[1]].float()
    assert torch.all((back - src).abs() <= src.abs().amax(-1, keepdim=True) / 16)


def test_budget_dedup_discard_and_clear():
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    key, other = m.publish(1), m.publish(2)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool))
    assert cache.save_block(key)
    assert not cache.save_block(key)
    m.forget(key)
    assert not cache.save_block(key)  # the CPU copy survives the GPU miss
    with pytest.raises(MemoryError, match="budget"):
        cache.save_block(other)
    assert cache.bytes_used == cache.block_bytes and other not in cache
    assert cache.discard(key) and not cache.discard(key)
    assert cache.bytes_used == 0
    assert cache.save_block(other)
    cache.clear()
    assert cache.bytes_used == len(cache) == 0
    assert other in m.hash_to_block_id


def test_budget_rejects_before_allocating(monkeypatch):
    engine = FakeEngine(arbitrary_pool())
    key = engine.manager.publish(1)
    cache = engine.create_cpu_prefix_cache(1)

    def no_alloc(*args, **kwargs):
        raise AssertionError("budget check must precede host allocation")

    monkeypatch.setattr(torch, "empty", no_alloc)
    with pytest.raises(MemoryError, match="budget"):
        cache.save_block(key)
    assert cache.bytes_used == 0


def test_discarded_slots_are_reused_without_allocation(monkeypatch):
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    key, other = m.publish(1), m.publish(2)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool))
    assert cache.reserved_bytes == 0
    assert cache.save_block(key)
    assert cache.reserved_bytes == cache.block_bytes
    assert cache.discard(key)

    def no_alloc(*args, **kwargs):
        raise AssertionError("a free slot must be reused")

    monkeypatch.setattr(torch, "empty", no_alloc)
    assert cache.save_block(other)
    assert cache.reserved_bytes == cache.bytes_used == cache.block_bytes


def test_preallocated_multi_slab_slots(monkeypatch):
    monkeypatch.setattr(cpc, "_SLAB_CHUNK_BYTES", 1)
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    cache = engine.create_cpu_prefix_cache(3 * per_block(engine.pool), preallocate=True)
    assert len(cache._slabs) == 3 and cache.reserved_bytes == 3 * cache.block_bytes
    keys = [m.publish(b) for b in (1, 3)]
    expected = {k: block_bytes(engine.pool, m.hash_to_block_id[k]) for k in keys}
    for k in keys:
        cache.save_block(k)
    assert cache._entries[keys[0]].slot != cache._entries[keys[1]].slot
    for k, data in expected.items():
        m.forget(k)
        assert torch.equal(block_bytes(engine.pool, cache.restore_block(k)), data)


def test_failed_copy_rolls_back(monkeypatch):
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    key = m.publish(1)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool))
    mapping = dict(m.hash_to_block_id)

    def fail(*args, **kwargs):
        raise RuntimeError("host allocation/copy failed")

    with monkeypatch.context() as patch:
        patch.setattr(torch.Tensor, "copy_", fail)
        with pytest.raises(RuntimeError, match="copy failed"):
            cache.save_block(key)
    assert len(cache) == cache.bytes_used == 0 and m.hash_to_block_id == mapping
    assert cache.save_block(key)
    expected = block_bytes(engine.pool, 1)
    m.forget(key)
    with monkeypatch.context() as patch:
        patch.setattr(torch.Tensor, "copy_", fail)
        with pytest.raises(RuntimeError, match="copy failed"):
            cache.restore_block(key)
    assert key in cache and key not in m.hash_to_block_id
    assert sorted(m.free_block_ids) == list(range(4)) and not m.used_block_ids
    assert torch.equal(block_bytes(engine.pool, cache.restore_block(key)), expected)


def test_validation_and_close():
    engine = FakeEngine(arbitrary_pool())
    for bad in (0, -1, 1.5, True):
        with pytest.raises(ValueError, match="positive integer"):
            engine.create_cpu_prefix_cache(bad)
    engine.model_runner.world_size = 2
    with pytest.raises(NotImplementedError, match="TP=1"):
        engine.create_cpu_prefix_cache(1 << 20)
    engine.model_runner.world_size = 1
    engine.model_runner.block_size = 128
    with pytest.raises(ValueError, match="layout"):
        engine.create_cpu_prefix_cache(1 << 20)
    engine.model_runner.block_size = 256
    with pytest.raises(ValueError, match="automatic"):
        engine.create_cpu_prefix_cache(1 << 20, save_on_release=True)
    with pytest.raises(ValueError, match="nonnegative"):
        engine.create_cpu_prefix_cache(1 << 20, automatic=True, hybrid=(1.0, -1.0, 0.0))
    cache = engine.create_cpu_prefix_cache(1 << 20, automatic=True)
    with pytest.raises(RuntimeError, match="already has"):
        engine.create_cpu_prefix_cache(1 << 20, automatic=True)
    cache.hybrid = (1.0, 2, 3)
    assert cache.hybrid == (1.0, 2.0, 3.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.measure_restore_s_per_block()
    key = engine.manager.publish(1)
    cache.save_block(key)
    cache.close()
    cache.close()
    assert cache.closed and cache.bytes_used == 0 and cache._manager is None
    assert engine.manager._cpu_prefix_cache is None
    with pytest.raises(RuntimeError, match="closed"):
        cache.save_block(key)
    with pytest.raises(RuntimeError, match="closed"):
        cache.restore_block(key)
    manual = engine.create_cpu_prefix_cache(1 << 20)
    with pytest.raises(ValueError, match="automatic"):
        manual.hybrid = (1.0, 0.0, 0.0)


def test_rejects_unknown_partial_and_conflicting_blocks():
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    key = m.publish(1)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool))
    with pytest.raises(KeyError):
        cache.save_block(-1)
    with pytest.raises(KeyError):
        cache.restore_block(key)
    block = m.blocks[1]
    block.token_ids = block.token_ids[:-1]
    with pytest.raises(ValueError, match="full prefix block"):
        cache.save_block(key)
    block.token_ids = [7] * 256
    cache.save_block(key)
    block.token_ids = [8] * 256
    with pytest.raises(ValueError, match="conflicting token"):
        cache.save_block(key)


def test_automatic_preserve_before_recycle_and_budget_skips():
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    keys = [m.publish(b) for b in (0, 1)]
    expected = block_bytes(engine.pool, 0)
    cache = engine.create_cpu_prefix_cache(per_block(engine.pool), automatic=True)
    assert cache.automatic
    first = m.allocate_block()  # recycles block 0: its published block is saved first
    assert first == 0 and keys[0] in cache
    second = m.allocate_block()  # block 1: budget is full, a counted skip
    assert second == 1 and keys[1] not in cache
    assert cache.stats["budget_skips"] == 1
    engine.pool[:, :, 0].fill_(3)
    m.release_block(first)
    m.release_block(second)
    target = cache.restore_block(keys[0])
    assert torch.equal(block_bytes(engine.pool, target), expected)


def test_save_on_release_only_while_admission_is_blocked():
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    cache = engine.create_cpu_prefix_cache(4 * per_block(engine.pool), automatic=True,
                                           save_on_release=True)
    block = m.allocate_block()
    key = m.publish(block)
    m.release_block(block)
    assert key not in cache
    block = m.allocate_block()
    key = m.publish(block)
    m.admission_blocked = True
    m.release_block(block)
    assert key in cache


def test_reference_quality_harness_slice_still_loads():
    """The reference's FP8 quality tool execs the source between two markers."""
    source = Path(cpc.__file__).read_text()
    start = source.index("# Largest finite float8_e4m3fn magnitude.")
    end = source.index("@dataclass(frozen=True)")
    namespace = {"torch": torch}
    exec(compile(source[start:end], cpc.__file__, "exec"), namespace)
    golden = np.load(Path(__file__).resolve().parent / "golden" / "fp8_rows.npz")
    x = torch.from_numpy(golden["x_128"].view(np.int16)).view(torch.bfloat16)
    payload = torch.empty(x.shape, dtype=torch.float8_e4m3fn)
    scale = torch.empty((*x.shape[:-1], 1), dtype=torch.bfloat16)
    namespace["fp8_quantize"](x, payload, scale)
    assert np.array_equal(payload.view(torch.uint8).numpy(), golden["payload_128"])
    assert np.array_equal(bits_u16(scale), golden["scale_128"])
    out = torch.empty_like(x)
    namespace["fp8_dequantize"](payload, scale, out)
    assert np.array_equal(bits_u16(out), golden["deq_128"])


@pytest.mark.parametrize("fp8", [False, True])
def test_batched_save_and_restore_match_per_block_calls(fp8):
    shape = (2, 2, 8, 256, 1, 4)
    pools = [finite_pool(shape) for _ in range(2)]
    outs = []
    for batched, pool in zip((False, True), pools):
        engine = FakeEngine(pool)
        m = engine.manager
        keys = [m.publish(b) for b in (5, 1, 6)]
        cache = engine.create_cpu_prefix_cache(8 * per_block(pool), fp8=fp8)
        if batched:
            assert cache.save_blocks(keys + [keys[0]]) == [True, True, True, False]
            assert cache.save_blocks(keys) == [False, False, False]
        else:
            assert all(cache.save_block(k) for k in keys)
        entries = [cache._entries[k] for k in keys]
        if batched:
            cache._copy_entries(entries, [0, 2, 3])
        else:
            for e, b in zip(entries, [0, 2, 3]):
                cache._copy_entry(e, b)
        outs.append((bits_u16(pool), [e.kv.view(torch.uint8).clone() for e in entries]))
        assert cache.stats["saved_blocks"] == 3 and cache.stats["restored_blocks"] == 3
    assert np.array_equal(outs[0][0], outs[1][0])
    assert all(torch.equal(a, b) for a, b in zip(outs[0][1], outs[1][1]))


def test_batched_save_is_all_or_nothing():
    engine = FakeEngine(arbitrary_pool())
    m = engine.manager
    keys = [m.publish(b) for b in (0, 1, 2)]
    cache = engine.create_cpu_prefix_cache(2 * per_block(engine.pool))
    with pytest.raises(MemoryError, match="budget"):
        cache.save_blocks(keys)
    assert len(cache) == 0 and cache.reserved_bytes == 0
    with pytest.raises(KeyError):
        cache.save_blocks([keys[0], 12345])
    assert len(cache) == 0
    assert cache.save_blocks(keys[:2]) == [True, True]
    assert cache.bytes_used == 2 * cache.block_bytes


def test_copy_method_defaults_and_overrides(monkeypatch):
    """CUDA pools default to the staged calls for both payload kinds; the
    KVOFF_* variables choose another method, and unknown names are rejected
    before any cache is built."""
    for key in ("KVOFF_FP8_SAVE", "KVOFF_FP8_RESTORE", "KVOFF_BF16_SAVE", "KVOFF_BF16_RESTORE"):
        monkeypatch.delenv(key, raising=False)
    assert cpc._transfer_modes() == {"fp8_save": "staged", "fp8_restore": "staged",
                                     "bf16_save": "staged", "bf16_restore": "staged"}
    monkeypatch.setenv("KVOFF_BF16_RESTORE", "engine")
    monkeypatch.setenv("KVOFF_FP8_SAVE", "mapped")
    modes = cpc._transfer_modes()
    assert modes["bf16_restore"] == "engine" and modes["fp8_save"] == "mapped"
    monkeypatch.setenv("KVOFF_BF16_SAVE", "dma")
    with pytest.raises(ValueError, match="KVOFF_BF16_SAVE"):
        cpc._transfer_modes()
