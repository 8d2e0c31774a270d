"""A minimal block manager and engine for driving the drop-in CPU tier in tests.

It restates only the protocol CPUBlockCache relies on from the reference's
BlockManager (nanovllm/engine/block_manager.py): published blocks
(hash_to_block_id), LRU victim choice with the _preserve_before_recycle /
before_block_reuse hooks (:97-116), release with _preserve_on_release
(:118-127), before_block_use on acquisition (:129-137) and
restore_cached_block's reserve -> copy -> publish-or-free protocol (:145-183).
"""

from __future__ import annotations

from collections import deque
from types import SimpleNamespace

import torch

from kvoff.cpu_prefix_cache import CPUBlockCache


class Block:
    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []


class FakeBlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        self.block_size = block_size
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()
        self._cpu_prefix_cache = None
        self.admission_blocked = False
        self._next_hash = 1

    def publish(self, block_id: int, tokens: list[int] | None = None) -> int:
        """Mark block_id as holding a full prefix block; return its hash."""
        h = self._next_hash
        self._next_hash += 1
        block = self.blocks[block_id]
        block.hash, block.token_ids = h, list(tokens or [h % 1000] * self.block_size)
        self.hash_to_block_id[h] = block_id
        return h

    def forget(self, prefix_hash: int) -> int:
        """Unpublish a block without touching its bytes."""
        block_id = self.hash_to_block_id.pop(prefix_hash)
        self.blocks[block_id].hash, self.blocks[block_id].token_ids = -1, []
        return block_id

    def _published(self, block: Block) -> bool:
        return block.hash != -1 and self.hash_to_block_id.get(block.hash) == block.block_id

    def allocate_block(self, order_writes: bool = True) -> int:
        block_id = self.free_block_ids[0]
        block = self.blocks[block_id]
        if self._published(block):
            if self._cpu_prefix_cache is not None:
                self._cpu_prefix_cache._preserve_before_recycle(block.hash)
            del self.hash_to_block_id[block.hash]
        if order_writes and self._cpu_prefix_cache is not None:
            self._cpu_prefix_cache.before_block_reuse(block_id)
        self.free_block_ids.popleft()
        block.ref_count, block.hash, block.token_ids = 1, -1, []
        self.used_block_ids.add(block_id)
        return block_id

    def release_block(self, block_id: int) -> None:
        block = self.blocks[block_id]
        block.ref_count = 0
        self.used_block_ids.discard(block_id)
        self.free_block_ids.append(block_id)
        if self._cpu_prefix_cache is not None and self._published(block):
            self._cpu_prefix_cache._preserve_on_release(block.hash)

    def acquire_block(self, block_id: int) -> None:
        if self.blocks[block_id].ref_count == 0:
            self.free_block_ids.remove(block_id)
            self.used_block_ids.add(block_id)
        if self._cpu_prefix_cache is not None:
            self._cpu_prefix_cache.before_block_use(block_id)
        self.blocks[block_id].ref_count += 1

    def restore_cached_block(self, prefix_hash, token_ids, copy_to_block) -> int:
        tokens = list(token_ids)
        existing = self.hash_to_block_id.get(prefix_hash)
        if existing is not None:
            if self.blocks[existing].token_ids != tokens:
                raise ValueError("prefix hash has conflicting token metadata")
            return existing
        if not self.free_block_ids:
            raise MemoryError("not enough free KV blocks to restore a prefix")
        block_id = self.allocate_block(order_writes=False)
        block = self.blocks[block_id]
        try:
            copy_to_block(block_id)
            block.hash, block.token_ids = prefix_hash, tokens
            self.hash_to_block_id[prefix_hash] = block_id
        except BaseException:
            if self.hash_to_block_id.get(prefix_hash) == block_id:
                del self.hash_to_block_id[prefix_hash]
            block.hash, block.token_ids = -1, []
            raise
        finally:
            self.release_block(block_id)
        return block_id


class FakeEngine:
    """runner + block manager + create_cpu_prefix_cache, like LLMEngine's."""

    def __init__(self, pool: torch.Tensor):
        num_blocks, block_size = pool.shape[2], pool.shape[3]
        self.model_runner = SimpleNamespace(world_size=1, block_size=block_size, kv_cache=pool)
        self.manager = FakeBlockManager(num_blocks, block_size)
        self.cache = None

    def create_cpu_prefix_cache(self, max_bytes: int, **kwargs) -> CPUBlockCache:
        self.cache = CPUBlockCache(self.model_runner, self.manager, max_bytes, **kwargs)
        return self.cache

    @property
    def pool(self) -> torch.Tensor:
        return self.model_runner.kv_cache


def block_bytes(pool: torch.Tensor, block_id: int) -> torch.Tensor:
    """Raw bytes of pool[:, :, block_id] on the host."""
    return pool[:, :, block_id].contiguous().cpu().view(torch.uint8).clone()


def bits_u16(t: torch.Tensor):
    """bf16 tensor -> numpy uint16 bit patterns."""
    return t.contiguous().cpu().view(torch.int16).numpy().view("uint16")
