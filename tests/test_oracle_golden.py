"""Pin the CPU oracle against fixtures produced by the reference itself.

The fixtures under tests/golden/ come from running the reference's own
fp8_quantize / fp8_dequantize and its CPUBlockCache (tests/golden/make_golden.py).
Quantization is compared bit for bit, NaN encodings included. Dequantized
values are bit-exact except NaN results, whose encoding the reference leaves
to torch's code path (0x7FC0 from its scalar path, 0xFFFF from its vector
path): there only NaN-ness is compared.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import workloads
from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def is_nan_bf16(bits: np.ndarray) -> np.ndarray:
    return (bits & 0x7FFF) > 0x7F80


def assert_bf16_equal(got: np.ndarray, want: np.ndarray) -> None:
    nan_got, nan_want = is_nan_bf16(got), is_nan_bf16(want)
    assert np.array_equal(nan_got, nan_want)
    assert np.array_equal(got[~nan_got], want[~nan_want])


@pytest.fixture(scope="module")
def rows():
    return np.load(GOLDEN / "fp8_rows.npz")


@pytest.mark.parametrize("d", [4, 8, 16, 64, 128, 256])
def test_quantize_matches_reference_bits(rows, d):
    payload, scale = oracle.fp8_quantize_rows(rows[f"x_{d}"])
    assert np.array_equal(scale, rows[f"scale_{d}"])
    assert np.array_equal(payload, rows[f"payload_{d}"])


@pytest.mark.parametrize("d", [4, 8, 16, 64, 128, 256])
def test_dequantize_matches_reference_bits(rows, d):
    out = oracle.fp8_dequantize_rows(rows[f"payload_{d}"], rows[f"scale_{d}"])
    assert_bf16_equal(out, rows[f"deq_{d}"])
    out = oracle.fp8_dequantize_rows(rows[f"rp_{d}"], rows[f"rs_{d}"])
    assert_bf16_equal(out, rows[f"rdeq_{d}"])


def test_scalar_conversions_match_torch():
    rng = np.random.default_rng(1)
    f = rng.integers(0, 1 << 32, 100_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    f = f[~np.isnan(f)]
    want = torch.from_numpy(f.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([oracle.bf16_from_f32(float(v)) for v in f], dtype=np.uint16)
    assert np.array_equal(got, want)
    # e4m3 over every fp32 value the quantizer can produce near the rounding
    # boundaries (|q| <= 448 after the clamp), plus all e4m3 decodings.
    g = f[np.abs(f) <= 448]
    edges = np.arange(0x43D00000, 0x43E00001, 97, dtype=np.uint32).view(np.float32)
    tiny = np.arange(0x3A000000, 0x3C900000, 1013, dtype=np.uint32).view(np.float32)
    g = np.concatenate([g, edges, -edges, tiny, -tiny])
    want = torch.from_numpy(g.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([oracle.e4m3_from_f32(float(v)) for v in g], dtype=np.uint8)
    assert np.array_equal(got, want)
    every = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(every.copy()).view(torch.float8_e4m3fn).float().numpy()
    got = np.array([oracle.e4m3_value(int(v)) for v in every], dtype=np.float32)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])


def test_tiny_pool_round_trips_match_reference_cache():
    g = np.load(GOLDEN / "dropin_tiny.npz")
    pool = g["bf16_pool"].copy()
    slots = oracle.copy_blocks(pool, [1, 3])
    assert np.array_equal(slots, g["bf16_slots"])
    oracle.copy_blocks(pool, [0, 2], slots, restore=True)
    assert np.array_equal(pool[:, :, [0, 2]].transpose(2, 0, 1, 3, 4, 5), g["bf16_restored"])

    pool = g["fp8_pool"].copy()
    payload, scale = oracle.fp8_save_blocks(pool, [2, 0])
    assert np.array_equal(payload, g["fp8_payload"])
    assert np.array_equal(scale, g["fp8_scale"])
    oracle.fp8_restore_blocks(pool, [1, 3], payload, scale)
    assert np.array_equal(pool[:, :, [1, 3]].transpose(2, 0, 1, 3, 4, 5), g["fp8_restored"])


def test_config1_digests_match_reference_cache():
    """All 16 config-1 blocks against the reference cache's per-block digests.

    The digests are per block (each saved slot, each restored target), so the
    blocks are checked one at a time in a reused one-block pool instead of the
    full 1.9 GB config-1 pool.
    """
    golden = json.loads((GOLDEN / "config1.json").read_text())
    c = golden["config"]
    sources, targets = golden["sources"], golden["targets"]
    assert [sources, targets] == list(workloads.config1_ids(c["seed"], c["num_blocks"],
                                                            c["saved"]))
    mask = workloads.outlier_mask(c["layers"], c["heads"], c["head_dim"], c["seed"])
    block = np.empty((2, c["layers"], 1, c["block_size"], c["heads"], c["head_dim"]), np.uint16)
    for i, source in enumerate(sources):
        block[:, :, 0] = workloads.block_values(source, c["layers"], c["block_size"], c["heads"],
                                                c["head_dim"], c["seed"], mask)
        assert sha(oracle.copy_blocks(block, [0])[0]) == golden["bf16"]["payload_sha256"][i]
        payload, scale = oracle.fp8_save_blocks(block, [0])
        assert sha(payload[0]) == golden["fp8"]["payload_sha256"][i]
        assert sha(scale[0]) == golden["fp8"]["scale_sha256"][i]
        oracle.fp8_restore_blocks(block, [0], payload, scale)  # slot i -> targets[i]
        assert sha(block[:, :, 0]) == golden["fp8"]["restored_sha256"][i]
    assert golden["fp8"]["within_amax_over_16"]


@pytest.mark.parametrize("name", sorted(workloads.STORE_CASES))
def test_store_kvcache_restatement_matches_fixture(name):
    golden = json.loads((GOLDEN / "store_kvcache.json").read_text())[name]
    n, h, d, nb, bs, pad = workloads.STORE_CASES[name]
    qkv, slots, k_cache, v_cache = workloads.store_kvcache_inputs(name)
    key = qkv[:, pad:pad + h * d].reshape(n, h, d)
    value = qkv[:, pad + h * d:].reshape(n, h, d)
    oracle.store_kvcache(key, value, k_cache, v_cache, slots)
    assert sha(k_cache) == golden["k_cache_sha256"]
    assert sha(v_cache) == golden["v_cache_sha256"]


def test_planted_mistake_in_oracle_is_detected(rows):
    """A corrupted oracle output must fail the golden comparison (test sanity)."""
    payload, scale = oracle.fp8_quantize_rows(rows["x_128"])
    payload[3, 7] ^= 1
    assert not np.array_equal(payload, rows["payload_128"])
