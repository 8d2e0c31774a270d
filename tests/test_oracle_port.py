"""The fast CPU port (timed baseline) computes exactly what the checker computes."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import workloads
from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("d", [4, 8, 16, 64, 128, 256])
def test_fast_port_matches_checker_on_special_rows(d):
    rows = np.load(GOLDEN / "fp8_rows.npz")[f"x_{d}"]
    pool = np.ascontiguousarray(np.resize(rows, (2, 1, 3, 32, 1, d)))
    slow = oracle.fp8_save_blocks(pool, [2, 0])
    fast = oracle.fp8_save_blocks(pool, [2, 0], fast=True)
    assert np.array_equal(slow[0], fast[0]) and np.array_equal(slow[1], fast[1])
    rng = np.random.default_rng(d)
    p = rng.integers(0, 256, slow[0].shape).astype(np.uint8)
    s = rng.integers(0, 1 << 16, slow[1].shape).astype(np.uint16)
    a, b = pool.copy(), pool.copy()
    oracle.fp8_restore_blocks(a, [1, 2], p, s)
    oracle.fp8_restore_blocks(b, [1, 2], p, s, fast=True)
    assert np.array_equal(a, b)


def test_fast_port_matches_checker_on_a_config1_block():
    c = workloads.CONFIG1
    pool = workloads.pool_with_blocks([0, 1], c["layers"], 2, c["block_size"], c["heads"],
                                      c["head_dim"], c["seed"])
    slow = oracle.fp8_save_blocks(pool, [0])
    fast = oracle.fp8_save_blocks(pool, [0], fast=True)
    assert np.array_equal(slow[0], fast[0]) and np.array_equal(slow[1], fast[1])
    a, b = pool.copy(), pool.copy()
    oracle.fp8_restore_blocks(a, [1], *slow)
    oracle.fp8_restore_blocks(b, [1], *slow, fast=True)
    assert np.array_equal(a, b)
