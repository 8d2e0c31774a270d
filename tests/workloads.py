"""Seeded synthetic KV workloads shared by the tests and the golden generator.

Values are N(0, 1) with a fixed 1% of (K/V, layer, KV head, channel) channels
scaled x20 as outliers, the distribution the reference's quality and copy
benchmarks use for KV. Each block is generated from its own seed pair, so a
test can build just the blocks it needs, identically on every machine
(numpy's PCG64 stream is platform independent).
"""

from __future__ import annotations

import numpy as np

# Qwen3-0.6B-shaped paged cache of BASELINE config 1: [2, 28, 64, 256, 8, 128].
CONFIG1 = dict(layers=28, num_blocks=64, block_size=256, heads=8, head_dim=128, seed=0,
               saved=16)
# Qwen3-8B-shaped cache of BASELINE config 2: [2, 36, 320, 256, 8, 128].
CONFIG2 = dict(layers=36, num_blocks=320, block_size=256, heads=8, head_dim=128)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs).

    In-place uint32 arithmetic: a finite pattern plus the rounding increment
    stays below 2**32, and no wide temporaries are allocated.
    """
    u = np.array(x, dtype=np.float32, copy=True).view(np.uint32)
    odd = (u >> 16) & 1
    u += np.uint32(0x7FFF)
    u += odd
    u >>= 16
    return u.astype(np.uint16)


def outlier_mask(layers: int, heads: int, head_dim: int, seed: int,
                 fraction: float = 0.01) -> np.ndarray:
    """Boolean [2, L, H, D]: channels scaled x20."""
    rng = np.random.default_rng([seed, 7919])
    return rng.random((2, layers, heads, head_dim)) < fraction


def block_values(block: int, layers: int, block_size: int, heads: int, head_dim: int,
                 seed: int, mask: np.ndarray | None = None) -> np.ndarray:
    """bf16 bits [2, L, BS, H, D] of one block."""
    if mask is None:
        mask = outlier_mask(layers, heads, head_dim, seed)
    rng = np.random.default_rng([seed, 1_000_003 + block])
    x = rng.standard_normal((2, layers, block_size, heads, head_dim), dtype=np.float32)
    x *= np.where(mask[:, :, None, :, :], np.float32(20.0), np.float32(1.0))
    return f32_to_bf16_bits(x)


def pool_with_blocks(blocks, layers: int, num_blocks: int, block_size: int, heads: int,
                     head_dim: int, seed: int, fill: int = 0) -> np.ndarray:
    """bf16 bits [2, L, NB, BS, H, D]; listed blocks get values, the rest `fill`."""
    pool = np.full((2, layers, num_blocks, block_size, heads, head_dim), fill, dtype=np.uint16)
    mask = outlier_mask(layers, heads, head_dim, seed)
    for b in blocks:
        pool[:, :, b] = block_values(b, layers, block_size, heads, head_dim, seed, mask)
    return pool


def config1_ids(seed: int = 0, num_blocks: int = 64, saved: int = 16) -> tuple[list, list]:
    """16 source block ids and 16 distinct restore targets for config 1."""
    rng = np.random.default_rng(seed)
    ids = rng.choice(num_blocks, 2 * saved, replace=False)
    return [int(i) for i in ids[:saved]], [int(i) for i in ids[saved:]]


def special_rows(head_dim: int, seed: int) -> np.ndarray:
    """bf16 bits [R, D]: rows that exercise every branch of the FP8 codec."""
    rng = np.random.default_rng([seed, head_dim])
    d = head_dim
    rows = []

    def row(values):
        rows.append(f32_to_bf16_bits(np.asarray(values, dtype=np.float32)))

    row(np.zeros(d))
    neg0 = np.zeros(d, dtype=np.uint16)
    neg0[::2] = 0x8000
    rows.append(neg0)
    row(rng.standard_normal(d))
    row(rng.standard_normal(d) * 1e-3)
    row(rng.standard_normal(d) * 3e4)
    row(np.linspace(-448, 448, d))
    row(np.linspace(-1, 1, d) * 2.0 ** -120)  # tiny amax: scale clamps to 1e-30
    sub = rng.integers(1, 0x80, d).astype(np.uint16)  # bf16 subnormals
    sub[::3] |= 0x8000
    rows.append(sub)
    big = np.full(d, 0x7F7F, dtype=np.uint16)  # bf16 max magnitude
    big[1::2] |= 0x8000
    rows.append(big)
    # e4m3 rounding ties: with amax 448 the scale is 1.0 exactly, so x / s = x.
    ties = np.array([448.0] + [1.0625, 1.1875, -1.0625, 0.5 + 1 / 32, 2.0 ** -10,
                               3 * 2.0 ** -10, -(2.0 ** -10), 2.0 ** -11, 464 / 1.0625] * d)[:d]
    row(ties)
    for code in (0x7F80, 0xFF80, 0x7FC0, 0xFFC1):  # +Inf, -Inf, +NaN, -NaN in a finite row
        bits = f32_to_bf16_bits(rng.standard_normal(d))
        bits[d // 3] = code
        rows.append(bits)
    both = f32_to_bf16_bits(rng.standard_normal(d))
    both[0], both[-1] = 0x7F80, 0x7FC0  # Inf and NaN in one row
    rows.append(both)
    # Arbitrary bit patterns (NaNs and Infs included) and many random finite rows.
    rows.extend(rng.integers(0, 1 << 16, (8, d)).astype(np.uint16))
    finite = rng.standard_normal((48, d)).astype(np.float32)
    finite *= np.float32(2.0) ** rng.integers(-30, 30, (48, 1)).astype(np.float32)
    rows.extend(f32_to_bf16_bits(finite))
    return np.stack(rows)


# store_kvcache cases: (tokens, KV heads, head_dim, blocks, block_size, qkv row padding).
# name: (tokens, KV heads, head dim, cache blocks, block size, q width before K in each qkv row)
STORE_CASES = {"vec": (300, 8, 128, 6, 64, 3 * 1024), "tiny": (37, 1, 4, 3, 16, 5),
               "prefill": (4096, 8, 128, 20, 256, 32 * 128)}


def store_kvcache_inputs(name: str):
    """(qkv bits [N, pad + 2*H*D], slot_mapping int32 [N], k_cache bits, v_cache bits).

    K is qkv[:, pad:pad + H*D] and V is qkv[:, pad + H*D:], so rows are strided
    like the q/k/v split of a fused projection; ~15% of slots are -1.
    """
    n, h, d, nb, bs, pad = STORE_CASES[name]
    rng = np.random.default_rng([3, n, d])
    qkv = rng.integers(0, 1 << 16, (n, pad + 2 * h * d)).astype(np.uint16)
    slots = rng.permutation(nb * bs)[:n].astype(np.int32)
    slots[rng.random(n) < 0.15] = -1
    k_cache = rng.integers(0, 1 << 16, (nb, bs, h, d)).astype(np.uint16)
    v_cache = rng.integers(0, 1 << 16, (nb, bs, h, d)).astype(np.uint16)
    return qkv, slots, k_cache, v_cache
