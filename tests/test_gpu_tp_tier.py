"""Tensor-parallel CPU tier on one GPU: each simulated rank owns a KV-head shard.

The leader cache on rank 0 drives the followers through a stand-in for the
engine's runner RPC (call() runs the method on every rank, as ModelRunner.call
does). Saves and restores through the leader must leave every rank's pool shard
and slots equal to the head-slice of the unsharded result: FP8 keeps one scale
per (token, KV head), so sharding by head changes nothing.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import workloads
from fake_engine import FakeBlockManager, bits_u16
from kvoff import tp_tier
from kvoff.cpu_prefix_cache import CPUBlockCache
from oracle import oracle

pytestmark = pytest.mark.gpu


class RankRunner:
    def __init__(self, rank: int, world: int, pool: torch.Tensor, ranks: list):
        self.rank, self.world_size, self.kv_cache = rank, world, pool
        self.block_size = pool.shape[3]
        self._ranks = ranks

    def call(self, method, *args):
        for other in self._ranks[1:]:  # the others run the message, then rank 0
            getattr(other, method)(*args)
        return getattr(self, method)(*args)

    def kvoff_tier(self, op, *args):
        return tp_tier.dispatch(self, op, *args)


def make_ranks(full_bits: np.ndarray, world: int, device):
    heads = full_bits.shape[4] // world
    ranks = []
    for r in range(world):
        shard = np.ascontiguousarray(full_bits[:, :, :, :, r * heads:(r + 1) * heads])
        pool = torch.from_numpy(shard.view(np.int16)).view(torch.bfloat16).to(device)
        ranks.append(RankRunner(r, world, pool, ranks))
    return ranks


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("fp8", [False, True])
def test_sharded_save_restore_equals_unsharded(cuda, world, fp8):
    layers, nb, bs, heads, dim = 2, 6, 64, 8, 128
    full = workloads.pool_with_blocks(range(nb), layers, nb, bs, heads, dim, seed=5)
    ranks = make_ranks(full, world, cuda)
    leader = ranks[0]
    manager = FakeBlockManager(nb, bs)
    keys = [manager.publish(b) for b in (4, 1, 5)]
    cache = CPUBlockCache(leader, manager, 8 * leader.kv_cache[:, :, 0].numel() * 2 * world,
                          fp8=fp8, split_streams=True)
    assert cache.save_block(keys[0])
    assert cache.save_blocks(keys[1:]) == [True, True]
    for k in keys:
        manager.forget(k)
    manager.free_block_ids.rotate(-2)  # the per-block restore lands in block 2
    assert cache.restore_block(keys[0]) == 2
    cache._copy_entries([cache._entries[k] for k in keys[1:]], [0, 3], wait=False)
    targets = [2, 0, 3]
    for b in (0, 3):
        cache.before_block_use(b)
    cache.synchronize()
    expected = full.copy()
    if fp8:
        p, s = oracle.fp8_save_blocks(full, [4, 1, 5])
        oracle.fp8_restore_blocks(expected, targets, p, s)
    else:
        slots = oracle.copy_blocks(full, [4, 1, 5])
        oracle.copy_blocks(expected, targets, slots, restore=True)
    per = heads // world
    for r, rank in enumerate(ranks):
        torch.cuda.synchronize()
        assert np.array_equal(bits_u16(rank.kv_cache), expected[:, :, :, :, r * per:(r + 1) * per])
    assert cache.block_bytes == world * cache._slot_bytes
    cache.close()
    assert not tp_tier._FOLLOWERS
