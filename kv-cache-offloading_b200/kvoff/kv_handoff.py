"""Drop-in KV handoff (export / import of one sequence's KV) with native copies.

Replaces nanovllm/engine/kv_handoff.py of the reference engine, keeping its
API: KVSnapshot, export_kv, verify_imported_kv, import_kv, their validation
and error messages and the PhaseTimer phases. For a CUDA pool, export gathers
the sequence's written tokens straight from its paged blocks into one pinned
dense [2, L, tokens, H, D] host tensor with a single strided DMA per block
(kvoff_copy_tokens), instead of index_select + contiguous + a pageable
.cpu() copy; import scatters the snapshot back the same way instead of a
device copy plus one copy_ per block. The bytes are moved unchanged, so the
result is byte-identical. A CPU pool keeps the reference's torch copies.
"""

from dataclasses import dataclass

import torch

from nanovllm.engine.handoff_timing import PhaseTimer
from nanovllm.engine.sequence import Sequence, SequenceStatus
from nanovllm.sampling_params import SamplingParams


@dataclass
class KVSnapshot:
    token_ids: list[int]
    num_prompt_tokens: int
    num_cached_tokens: int
    block_size: int
    temperature: float
    max_tokens: int
    ignore_eos: bool
    kv: torch.Tensor  # [K/V, layer, written token, KV head, head dim], CPU

    @property
    def payload_bytes(self):
        return self.kv.numel() * self.kv.element_size()


def _require_single_worker(runner):
    if runner.world_size != 1:
        raise NotImplementedError("KV handoff currently requires tensor_parallel_size=1")


@torch.inference_mode()
def export_kv(runner, seq: Sequence) -> KVSnapshot:
    """Snapshot of a running sequence's written KV, taken between steps."""
    _require_single_worker(runner)
    if seq.status != SequenceStatus.RUNNING or seq.num_scheduled_tokens:
        raise ValueError("export requires a running sequence between steps")
    count = seq.num_cached_tokens
    if count <= 0 or count != len(seq) - 1:
        raise ValueError("export requires exactly one pending, uncached token")
    cache = runner.kv_cache
    num_blocks = -(-count // runner.block_size)
    timer = PhaseTimer("export_kv", seq_id=seq.seq_id, num_tokens=count, num_blocks=num_blocks)
    with timer.phase("gather_blocks"):
        block_ids = list(seq.block_table[:num_blocks])
        if len(block_ids) != num_blocks:
            raise ValueError("sequence is missing KV blocks")
        if not cache.is_cuda:
            index = torch.tensor(block_ids, dtype=torch.int64)
            packed = cache.index_select(2, index).flatten(2, 3)
    with timer.phase("pack"):
        if cache.is_cuda:  # the DMA writes the dense layout directly into pinned memory
            payload = torch.empty((2, cache.shape[1], count, *cache.shape[-2:]),
                                  dtype=cache.dtype, pin_memory=True)
        else:
            dense = packed[:, :, :count].contiguous()
    with timer.phase("copy_to_host"):
        if cache.is_cuda:
            from kvoff import ops

            ops.copy_tokens(cache, block_ids, count, payload.data_ptr())
            torch.cuda.current_stream(cache.device).synchronize()
        else:
            payload = dense.cpu()
    timer.finish(payload_bytes=payload.numel() * payload.element_size())
    return KVSnapshot(seq.token_ids.copy(), seq.num_prompt_tokens, count, runner.block_size,
                      seq.temperature, seq.max_tokens, seq.ignore_eos, payload)


# Device memory a verification of a CUDA pool holds at once: two buffers (the
# pool's tokens and the snapshot's) of at most this many bytes each (whole
# blocks; at least one block).
_VERIFY_CHUNK_BYTES = 128 << 20


@torch.inference_mode()
def verify_imported_kv(runner, seq: Sequence, snapshot: KVSnapshot) -> bool:
    """True when the sequence's blocks hold exactly the snapshot's KV bytes.

    CUDA pool: the comparison runs on the GPU, in chunks of whole blocks. For
    each chunk the sequence's tokens are gathered device to device into one
    dense buffer (kvoff_copy_tokens, as export_kv does into host memory), the
    snapshot's matching tokens are copied host to device into another (one
    contiguous copy per (K/V, layer) row of the snapshot), and a device-side
    byte comparison folds into one flag that the host reads once at the end.
    So the snapshot crosses PCIe once and the host does no byte work; device
    memory stays bounded (two buffers of about _VERIFY_CHUNK_BYTES) however
    long the sequence is. A CPU pool is gathered and compared in one pass.
    Missing blocks, or a snapshot of another shape or dtype, compare unequal.
    """
    cache = runner.kv_cache
    count = snapshot.num_cached_tokens
    block_size = runner.block_size
    num_blocks = -(-count // block_size)
    block_ids = list(seq.block_table[:num_blocks])
    kv = snapshot.kv
    if len(block_ids) < num_blocks or kv.dtype != cache.dtype:
        return False
    if count <= 0:
        return True
    if tuple(kv.shape) != (2, cache.shape[1], count, *cache.shape[-2:]):
        return False
    if not cache.is_cuda:
        index = torch.tensor(block_ids, dtype=torch.int64)
        actual = cache.index_select(2, index).flatten(2, 3)[:, :, :count]
        return torch.equal(actual.view(torch.uint8), kv.view(torch.uint8))
    from kvoff import ops

    kv = kv if kv.is_contiguous() else kv.contiguous()
    layers, (heads, dim) = cache.shape[1], cache.shape[-2:]
    row_bytes = heads * dim * cache.element_size()  # one token of one (K/V, layer) row
    chunk_blocks = max(1, _VERIFY_CHUNK_BYTES // (2 * layers * block_size * row_bytes))
    chunk_tokens = chunk_blocks * block_size
    width = min(count, chunk_tokens)
    actual = torch.empty((2 * layers * width * heads * dim,), dtype=cache.dtype,
                         device=cache.device)
    expected = torch.empty_like(actual)
    differs = torch.zeros((), dtype=torch.bool, device=cache.device)
    rows = kv.view(2 * layers, count, heads, dim)
    for first in range(0, count, chunk_tokens):
        n = min(chunk_tokens, count - first)
        here = actual[:2 * layers * n * heads * dim]
        want = expected[:2 * layers * n * heads * dim].view(2 * layers, n, heads, dim)
        ops.copy_tokens(cache, block_ids[first // block_size:], n, here.data_ptr())
        for r in range(2 * layers):
            ops.memcpy(want[r].data_ptr(), rows[r, first].data_ptr(), n * row_bytes,
                       device=cache.device)
        differs |= torch.ne(here.view(torch.uint8), want.view(-1).view(torch.uint8)).any()
    return not bool(differs.item())


@torch.inference_mode()
def import_kv(runner, block_manager, snapshot: KVSnapshot) -> Sequence:
    """Allocate fresh blocks, copy the snapshot in and return a decode-ready sequence.

    Both workers must use the same model weights and KV dtype. The caller owns
    admission into its scheduler and releasing the source after acknowledgement.
    """
    _require_single_worker(runner)
    timer = PhaseTimer("import_kv", num_cached_tokens=snapshot.num_cached_tokens,
                       num_tokens=len(snapshot.token_ids))
    seq = None
    try:
        with timer.phase("validate"):
            cache = runner.kv_cache
            expected = (2, cache.shape[1], snapshot.num_cached_tokens, *cache.shape[-2:])
            layout_ok = (snapshot.block_size == runner.block_size == block_manager.block_size
                         and tuple(snapshot.kv.shape) == expected
                         and snapshot.kv.dtype == cache.dtype
                         and snapshot.kv.device.type == "cpu")
            if not layout_ok:
                raise ValueError("snapshot layout, dtype or block size does not match this worker")
            generated = len(snapshot.token_ids) - snapshot.num_prompt_tokens
            if (not 0 < snapshot.num_prompt_tokens < len(snapshot.token_ids)
                    or snapshot.num_cached_tokens != len(snapshot.token_ids) - 1
                    or generated >= snapshot.max_tokens):
                raise ValueError(
                    "snapshot must contain an unfinished completion and one uncached token")
        with timer.phase("rebuild_sequence"):
            seq = Sequence(snapshot.token_ids[:snapshot.num_prompt_tokens], SamplingParams(
                temperature=snapshot.temperature, max_tokens=snapshot.max_tokens,
                ignore_eos=snapshot.ignore_eos))
            for token in snapshot.token_ids[snapshot.num_prompt_tokens:]:
                seq.append_token(token)
        with timer.phase("allocate_blocks"):
            block_manager.allocate_for_resume(seq, snapshot.num_cached_tokens)
        with timer.phase("copy_to_device"):
            if cache.is_cuda:  # one DMA per block, straight into the assigned blocks
                from kvoff import ops

                kv = snapshot.kv if snapshot.kv.is_contiguous() else snapshot.kv.contiguous()
                ops.copy_tokens(cache, list(seq.block_table), snapshot.num_cached_tokens,
                                kv.data_ptr(), restore=True)
            else:
                payload = snapshot.kv.to(device=cache.device)
        with timer.phase("scatter_blocks"):
            if cache.is_cuda:
                if not kv.is_pinned():  # a pageable source must outlive its copy
                    torch.cuda.current_stream(cache.device).synchronize()
            else:
                for logical, physical in enumerate(seq.block_table):
                    start = logical * runner.block_size
                    end = min(start + runner.block_size, snapshot.num_cached_tokens)
                    cache[:, :, physical, :end - start].copy_(payload[:, :, start:end])
        with timer.phase("publish_cache"):
            # Prefix metadata becomes valid only once the payload has been copied.
            seq.num_cached_tokens = 0
            seq.num_scheduled_tokens = snapshot.num_cached_tokens
            block_manager.hash_blocks(seq)
            seq.num_scheduled_tokens = 0
            seq.num_cached_tokens = snapshot.num_cached_tokens
            seq.status = SequenceStatus.RUNNING
            seq.is_prefill = False
        timer.finish(payload_bytes=lambda: snapshot.payload_bytes,
                     num_blocks=lambda: len(seq.block_table))
        return seq
    except Exception as error:
        timer.abort(error)
        if seq is not None:
            block_manager.deallocate(seq)
        raise
