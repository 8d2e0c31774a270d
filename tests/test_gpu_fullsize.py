"""BASELINE config-2 sizes: a 12 GB pool whose far blocks sit past 2^32 bytes.

The kernels address the pool with 64-bit offsets; these checks place the
compared blocks at the end of a full Qwen3-8B-shaped pool [2, 36, 320, 256, 8,
128] (the last block's last chunk starts 11.9 GB in) and compare against the
oracle, which runs on just those blocks. Also checks size-independent
properties: a save / restore / save round trip reproduces the same FP8 slot
(dequantized values re-quantize to themselves once the scale is fixed by the
first pass) and restored blocks stay within the reference's amax / 16 bound.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

LAYERS, NUM_BLOCKS, BS, HEADS, DIM = 36, 320, 256, 8, 128


@pytest.fixture(scope="module")
def big_pool():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device unavailable")
    device = torch.device("cuda", 0)
    pool = torch.zeros((2, LAYERS, NUM_BLOCKS, BS, HEADS, DIM), dtype=torch.bfloat16, device=device)
    blocks = [319, 318, 160, 0]
    mask = workloads.outlier_mask(LAYERS, HEADS, DIM, seed=9)
    host = {}
    for b in blocks:
        bits = workloads.block_values(b, LAYERS, BS, HEADS, DIM, seed=9, mask=mask)
        host[b] = bits
        pool[:, :, b].copy_(torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16))
    yield pool, host
    del pool
    torch.cuda.empty_cache()


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def test_pool_offsets_exceed_32_bits(big_pool):
    pool, _ = big_pool
    last_chunk = (2 * LAYERS - 1) * pool.stride(1) + (NUM_BLOCKS - 1) * pool.stride(2)
    assert last_chunk * pool.element_size() > 2 ** 32


def test_fp8_far_blocks_bit_exact_and_stable(big_pool):
    from kvoff import ops

    pool, host = big_pool
    g = ops.geometry(pool)
    ids = [319, 318, 160, 0]
    payload = torch.empty((4, g.fp8_payload_bytes), dtype=torch.uint8, device=pool.device)
    scale = torch.empty((4, g.fp8_scale_bytes), dtype=torch.uint8, device=pool.device)
    ops.save_fp8(pool, ids, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    small = np.stack([host[b] for b in ids], axis=2)  # [2, L, 4, BS, H, D]
    want_p, want_s = oracle.fp8_save_blocks(small, [0, 1, 2, 3])
    assert np.array_equal(payload.cpu().numpy().reshape(want_p.shape), want_p)
    assert np.array_equal(scale.cpu().numpy().view(np.uint16).reshape(want_s.shape), want_s)
    # Restore into other far blocks, compare with the oracle and the reference bound.
    targets = [317, 316, 1, 2]
    ops.restore_fp8(pool, targets, [p.data_ptr() for p in payload], [s.data_ptr() for s in scale])
    restored = np.zeros_like(small)
    oracle.fp8_restore_blocks(restored, [0, 1, 2, 3], want_p, want_s)
    for i, t in enumerate(targets):
        got = u16(pool[:, :, t])
        assert np.array_equal(got, restored[:, :, i])
        src = torch.from_numpy(small[:, :, i].view(np.int16)).view(torch.bfloat16).float()
        back = torch.from_numpy(got.view(np.int16)).view(torch.bfloat16).float()
        assert torch.all((back - src).abs() <= src.abs().amax(-1, keepdim=True) / 16)
    # Saving the restored blocks gives back the same slots.
    again = torch.empty_like(payload), torch.empty_like(scale)
    ops.save_fp8(pool, targets, [p.data_ptr() for p in again[0]], [s.data_ptr() for s in again[1]])
    assert torch.equal(again[0], payload) and torch.equal(again[1], scale)


@pytest.mark.parametrize("method", ["engine", "tma", "sm"])
def test_bf16_far_blocks_byte_exact(big_pool, method):
    from kvoff import ops

    pool, host = big_pool
    code = {"engine": ops.COPY_ENGINE, "tma": ops.COPY_TMA, "sm": ops.COPY_SM}[method]
    g = ops.geometry(pool)
    slots = torch.empty((2, g.block_bytes), dtype=torch.uint8, device=pool.device)
    ops.copy_blocks(pool, [319, 160], [s.data_ptr() for s in slots], method=code)
    assert np.array_equal(slots[0].cpu().numpy().view(np.uint16), host[319].reshape(-1))
    ops.copy_blocks(pool, [315, 314], [s.data_ptr() for s in slots], restore=True, method=code)
    assert np.array_equal(u16(pool[:, :, 315]), host[319])
    assert np.array_equal(u16(pool[:, :, 314]), host[160])


def test_store_kvcache_into_far_slots(big_pool):
    from kvoff import ops

    pool, _ = big_pool
    n = 64
    torch.manual_seed(3)
    key = torch.randn(n, HEADS, DIM, dtype=torch.bfloat16, device=pool.device)
    value = torch.randn(n, HEADS, DIM, dtype=torch.bfloat16, device=pool.device)
    last = NUM_BLOCKS * BS
    slots = torch.arange(last - n, last, dtype=torch.int32, device=pool.device).flip(0)
    layer = LAYERS - 1
    ops.store_kvcache(key, value, pool[0, layer], pool[1, layer], slots)
    k_rows = pool[0, layer].view(-1, HEADS * DIM)[slots.long()]
    v_rows = pool[1, layer].view(-1, HEADS * DIM)[slots.long()]
    assert torch.equal(k_rows.view(torch.int16), key.reshape(n, -1).view(torch.int16))
    assert torch.equal(v_rows.view(torch.int16), value.reshape(n, -1).view(torch.int16))
