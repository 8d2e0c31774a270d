"""The drop-in KV handoff on a CUDA pool: byte-exact export / import.

export_kv must return exactly the reference's dense snapshot (the pool's
index_select over the sequence's blocks, flattened over tokens and cut at the
written-token count, nanovllm/engine/kv_handoff.py:46-55), and import_kv must
place every token back into the newly allocated blocks (:112-118). The engine
modules the drop-in imports (Sequence, SamplingParams, PhaseTimer) are replaced
by small test doubles with the attributes it uses.
"""

from __future__ import annotations

import enum
import importlib
import sys
from contextlib import contextmanager
from dataclasses import dataclass
from types import ModuleType, SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu


class SequenceStatus(enum.Enum):
    WAITING = 1
    RUNNING = 2
    FINISHED = 3


@dataclass
class SamplingParams:
    temperature: float = 1.0
    max_tokens: int = 64
    ignore_eos: bool = False


class Sequence:
    counter = 0

    def __init__(self, token_ids, sampling_params=SamplingParams()):
        Sequence.counter += 1
        self.seq_id = Sequence.counter
        self.status = SequenceStatus.WAITING
        self.token_ids = list(token_ids)
        self.num_prompt_tokens = len(token_ids)
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.block_table = []
        self.is_prefill = True
        self.temperature = sampling_params.temperature
        self.max_tokens = sampling_params.max_tokens
        self.ignore_eos = sampling_params.ignore_eos

    def __len__(self):
        return len(self.token_ids)

    def append_token(self, token):
        self.token_ids.append(token)


class PhaseTimer:
    def __init__(self, name, **fields):
        self.phases = []

    @contextmanager
    def phase(self, name):
        self.phases.append(name)
        yield

    def finish(self, **fields):
        return None

    def abort(self, error):
        return None


@pytest.fixture
def handoff(monkeypatch):
    modules = {
        "nanovllm": ModuleType("nanovllm"),
        "nanovllm.engine": ModuleType("nanovllm.engine"),
        "nanovllm.engine.handoff_timing": SimpleNamespace(PhaseTimer=PhaseTimer),
        "nanovllm.engine.sequence": SimpleNamespace(Sequence=Sequence,
                                                     SequenceStatus=SequenceStatus),
        "nanovllm.sampling_params": SimpleNamespace(SamplingParams=SamplingParams),
    }
    for name, module in modules.items():
        monkeypatch.setitem(sys.modules, name, module)
    monkeypatch.delitem(sys.modules, "kvoff.kv_handoff", raising=False)
    return importlib.import_module("kvoff.kv_handoff")


class ResumeManager:
    """allocate_for_resume / hash_blocks / deallocate of the block manager."""

    def __init__(self, free, block_size):
        self.free, self.block_size = list(free), block_size

    def allocate_for_resume(self, seq, num_cached_tokens):
        n = -(-num_cached_tokens // self.block_size)
        seq.block_table = [self.free.pop(0) for _ in range(n)]
        seq.num_cached_tokens = num_cached_tokens

    def hash_blocks(self, seq):
        pass

    def deallocate(self, seq):
        self.free.extend(seq.block_table)
        seq.block_table = []


@pytest.mark.parametrize("shape,count", [((2, 3, 8, 16, 2, 8), 37), ((2, 2, 6, 256, 8, 128), 513),
                                          ((2, 2, 4, 256, 1, 4), 256)])
def test_export_import_round_trip_is_byte_exact(cuda, handoff, shape, count):
    n = 1
    for s in shape:
        n *= s
    raw = torch.arange(2 * n, dtype=torch.int64).remainder(253).to(torch.uint8)
    pool = raw.view(torch.bfloat16).reshape(shape).to(cuda)
    block_size = shape[3]
    runner = SimpleNamespace(world_size=1, block_size=block_size, kv_cache=pool)
    blocks = -(-count // block_size)
    seq = Sequence(list(range(count - 3)), SamplingParams(max_tokens=64))
    for token in (7, 8, 9, 10):
        seq.append_token(token)
    seq.status = SequenceStatus.RUNNING
    seq.num_cached_tokens = count
    seq.block_table = list(range(shape[2] - 1, shape[2] - 1 - blocks, -1))
    snapshot = handoff.export_kv(runner, seq)
    ids = torch.tensor(seq.block_table, dtype=torch.int64)
    want = pool.cpu().index_select(2, ids).flatten(2, 3)[:, :, :count].contiguous()
    assert snapshot.kv.shape == want.shape and not snapshot.kv.is_cuda
    assert torch.equal(snapshot.kv.view(torch.uint8), want.view(torch.uint8))
    assert snapshot.payload_bytes == want.numel() * want.element_size()

    target = torch.zeros_like(pool)
    runner2 = SimpleNamespace(world_size=1, block_size=block_size, kv_cache=target)
    manager = ResumeManager(range(shape[2]), block_size)
    restored = handoff.import_kv(runner2, manager, snapshot)
    assert restored.status == SequenceStatus.RUNNING and not restored.is_prefill
    assert restored.num_cached_tokens == count and len(restored.block_table) == blocks
    assert handoff.verify_imported_kv(runner2, restored, snapshot)
    got = target.cpu().index_select(2, torch.tensor(restored.block_table)).flatten(2, 3)
    assert torch.equal(got[:, :, :count].contiguous().view(torch.uint8), want.view(torch.uint8))
    # Tokens past the written count stay untouched in the last block.
    assert not got[:, :, count:].view(torch.uint8).any()
    # A pageable (unpinned) snapshot imports the same way.
    snapshot.kv = snapshot.kv.clone()
    target.zero_()
    manager = ResumeManager(range(shape[2]), block_size)
    restored = handoff.import_kv(runner2, manager, snapshot)
    assert handoff.verify_imported_kv(runner2, restored, snapshot)


def test_import_validation_matches_the_reference(cuda, handoff):
    pool = torch.zeros((2, 2, 4, 16, 1, 8), dtype=torch.bfloat16, device=cuda)
    runner = SimpleNamespace(world_size=1, block_size=16, kv_cache=pool)
    manager = ResumeManager(range(4), 16)
    bad = handoff.KVSnapshot(list(range(10)), 5, 9, 16, 1.0, 64, False,
                             torch.zeros((2, 2, 8, 1, 8), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="layout"):
        handoff.import_kv(runner, manager, bad)
    runner.world_size = 2
    with pytest.raises(NotImplementedError, match="tensor_parallel_size=1"):
        handoff.import_kv(runner, manager, bad)


@pytest.mark.parametrize("chunk_blocks", [1, 2, 64])
def test_verify_imported_kv_reads_back_in_chunks_and_finds_any_changed_byte(
        cuda, handoff, monkeypatch, chunk_blocks):
    """verify_imported_kv compares every written token, in one chunk or in
    chunks of whole blocks, on the device; one changed byte anywhere fails it."""
    shape, count = (2, 2, 6, 16, 2, 8), 70  # 5 blocks, the last one partial
    token_bytes = 2 * shape[1] * shape[4] * shape[5] * 2
    monkeypatch.setattr(handoff, "_VERIFY_CHUNK_BYTES", chunk_blocks * shape[3] * token_bytes)
    g = torch.Generator().manual_seed(3)
    pool = torch.randn(shape, generator=g).to(torch.bfloat16).to(cuda)
    runner = SimpleNamespace(world_size=1, block_size=shape[3], kv_cache=pool)
    seq = Sequence(list(range(count - 1)), SamplingParams(max_tokens=64))
    seq.append_token(5)
    seq.append_token(6)
    seq.status = SequenceStatus.RUNNING
    seq.num_cached_tokens = count
    seq.block_table = [5, 0, 3, 1, 4]
    snapshot = handoff.export_kv(runner, seq)
    assert handoff.verify_imported_kv(runner, seq, snapshot)
    # One changed byte anywhere among the written tokens is found: first block,
    # a middle block, the last written token of the partial block.
    for block, token in ((5, 0), (3, 7), (4, count - 4 * shape[3] - 1)):
        saved = pool[1, 1, block, token].clone()
        pool[1, 1, block, token, 1, 2] += 1
        assert not handoff.verify_imported_kv(runner, seq, snapshot)
        pool[1, 1, block, token] = saved
    assert handoff.verify_imported_kv(runner, seq, snapshot)
    # Tokens past the written count are not part of the snapshot.
    pool[0, 0, 4, count - 4 * shape[3]:] = 9
    assert handoff.verify_imported_kv(runner, seq, snapshot)
    # A block table without room for every written token does not verify.
    seq.block_table = seq.block_table[:-1]
    assert not handoff.verify_imported_kv(runner, seq, snapshot)
    # A snapshot of another length does not verify (and is not read past its end).
    shorter = handoff.KVSnapshot(snapshot.token_ids, snapshot.num_prompt_tokens, count,
                                 snapshot.block_size, 1.0, 64, False, snapshot.kv[:, :, :-1])
    seq.block_table = [5, 0, 3, 1, 4]
    assert not handoff.verify_imported_kv(runner, seq, shorter)
    # A pageable snapshot verifies the same way.
    pageable = handoff.KVSnapshot(snapshot.token_ids, snapshot.num_prompt_tokens, count,
                                  snapshot.block_size, 1.0, 64, False, snapshot.kv.clone())
    assert handoff.verify_imported_kv(runner, seq, pageable)
