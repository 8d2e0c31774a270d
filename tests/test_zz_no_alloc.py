"""The allocation-free staged FP8 save against the regular staged save.

kvoff_fp8_save_blocks_staged_noalloc exists for callers that cannot allocate
device memory at save time (an engine that reserved nearly all HBM for its KV
pool, or a host runtime with no device allocator): it stages through a fixed
16 MiB scratch array inside libkvoff instead of a caller buffer. Its slots must
be bit-identical to kvoff_fp8_save_blocks_staged's, on consecutive calls (the
scratch keeps the previous call's data) and for blocks larger than the scratch
(processed in chunk pieces). Collected last so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from kvoff import _lib

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20


def _geometry(pool: torch.Tensor):
    _, layers, nb, bs, h, d = pool.shape
    return (2 * layers, nb * bs * h * d, bs * h * d, nb, bs * h, d)


def _slots(n: int, rows: int, d: int):
    payload = torch.empty((n, rows * d), dtype=torch.uint8).pin_memory()
    scale = torch.empty((n, rows * 2), dtype=torch.uint8).pin_memory()
    payload.fill_(0x5A)
    scale.fill_(0xA5)
    return payload, scale


def _save(name: str, pool, ids, payload, scale, staging=None) -> None:
    chunks, cs, bst, nb, rpc, d = _geometry(pool)
    stream = torch.cuda.current_stream(pool.device).cuda_stream
    args = [pool.data_ptr(), chunks, cs, bst, nb, rpc, d, _lib.int64_array(ids), len(ids),
            _lib.pointer_array([p.data_ptr() for p in payload]),
            _lib.pointer_array([s.data_ptr() for s in scale])]
    if staging is not None:
        args += [staging[0].data_ptr(), staging[1].data_ptr(), 1]
    _lib.call(name, *args, ctypes.c_void_p(stream))


@pytest.mark.parametrize("shape", [
    (2, 36, 4, 256, 8, 128),  # Qwen3-8B block (19.2 MB of FP8): two scratch pieces
    (2, 2, 5, 256, 1, 4),     # the reference tests' tiny pool: one piece, generic kernel
])
def test_noalloc_save_matches_staged_save_on_consecutive_calls(shape):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device unavailable")
    device = torch.device("cuda", 0)
    torch.manual_seed(7)
    pool = torch.randn(shape, device=device).to(torch.bfloat16)
    pool[:, :, :, ::17] *= 30  # outlier tokens
    chunks, _, _, _, rpc, d = _geometry(pool)
    rows = chunks * rpc
    staging = (torch.empty(rows * d, dtype=torch.uint8, device=device),
               torch.empty(rows * 2, dtype=torch.uint8, device=device))
    for ids in ([shape[2] - 1, 0], [1, 2]):  # two calls in a row
        want = _slots(len(ids), rows, d)
        got = _slots(len(ids), rows, d)
        _save("kvoff_fp8_save_blocks_staged", pool, ids, *want, staging=staging)
        _save("kvoff_fp8_save_blocks_staged_noalloc", pool, ids, *got)
        torch.cuda.synchronize()
        assert torch.equal(got[0], want[0])
        assert torch.equal(got[1], want[1])


def test_noalloc_save_rejects_chunks_larger_than_the_scratch():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device unavailable")
    rows_per_chunk = SCRATCH_BYTES // 128  # one chunk of 128-wide rows > 16 MiB with scales
    ids = _lib.int64_array([0])
    slot = _lib.pointer_array([1 << 20])
    rc = _lib.lib().kvoff_fp8_save_blocks_staged_noalloc(
        ctypes.c_void_p(1 << 20), 2, rows_per_chunk * 128, rows_per_chunk * 128, 1,
        rows_per_chunk, 128, ids, 1, slot, slot, None)
    assert rc == _lib.KVOFF_EINVAL
    assert "maximum" in _lib.last_error()


def test_noalloc_save_rejects_a_pool_off_the_current_device():
    """The scratch used is the current device's, so a pool in host memory (or
    on another device) is refused before anything is enqueued."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA device unavailable")
    torch.cuda.set_device(0)
    pool = torch.zeros((2, 2, 2, 256, 1, 4), dtype=torch.bfloat16)  # host memory
    chunks, cs, bst, nb, rpc, d = _geometry(pool)
    slot = torch.empty(chunks * rpc * d, dtype=torch.uint8, pin_memory=True)
    rc = _lib.lib().kvoff_fp8_save_blocks_staged_noalloc(
        ctypes.c_void_p(pool.data_ptr()), chunks, cs, bst, nb, rpc, d, _lib.int64_array([0]), 1,
        _lib.pointer_array([slot.data_ptr()]), _lib.pointer_array([slot.data_ptr()]), None)
    assert rc == _lib.KVOFF_EINVAL
    assert "current device" in _lib.last_error()
