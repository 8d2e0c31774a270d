"""The drop-ins inside the reference engine: an offloaded prefix restores exactly.

Each case runs tests/engine_driver.py in fresh processes: the reference engine
(a copy of its tree, stock or with kvoff's drop-ins) with a small random Qwen3
checkpoint, three greedy requests, and a turn (A2) whose prefix either stayed
on the GPU ("resident") or went through the CPU tier ("offload": saved when
another request recycled its blocks, restored at admission). Checks:

* BF16 tier: a restored prefix is byte-identical KV, so A2's tokens equal the
  resident run's, for the stock engine and for kvoff at TP=1, and for kvoff's
  per-rank tier at TP=2 (each rank saves and restores its own KV heads; the
  stock engine rejects a CPU tier under TP).
* FP8 tier: kvoff's quantizer is bit-exact with the reference's, so kvoff's
  A2 tokens, prefix hits and block counts equal the stock engine's.

Skipped without a reference checkout (see test_reference_suite.py); the TP=2
case needs two GPUs.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

from test_reference_suite import REFERENCE

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(REFERENCE is None, reason="reference checkout not present")]

DRIVER = Path(__file__).resolve().with_name("engine_driver.py")
_RUNS: dict[tuple, dict] = {}


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def run(tmp_path_factory, impl: str, tp: int, scenario: str, fp8: bool) -> dict:
    key = (impl, tp, scenario, fp8)
    if key not in _RUNS:
        out = tmp_path_factory.mktemp("engine") / "result.json"
        result = subprocess.run(
            [sys.executable, str(DRIVER), "--reference", str(REFERENCE), "--impl", impl,
             "--tp", str(tp), "--scenario", scenario, "--fp8", str(int(fp8)), "--out", str(out)],
            capture_output=True, text=True, timeout=900)
        assert result.returncode == 0, result.stdout[-2000:] + result.stderr[-4000:]
        _RUNS[key] = json.loads(out.read_text())
    return _RUNS[key]


@pytest.mark.parametrize("impl", ["reference", "kvoff"])
def test_bf16_restored_prefix_gives_the_resident_outputs(tmp_path_factory, impl):
    if _gpus() < 1:
        pytest.skip("CUDA device unavailable")
    resident = run(tmp_path_factory, "reference", 1, "resident", False)
    offload = run(tmp_path_factory, impl, 1, "offload", False)
    assert offload["stats"]["restored_blocks"] >= 1
    assert offload["cached_tokens"]["A2"] == resident["cached_tokens"]["A2"] > 0
    assert offload["outputs"] == resident["outputs"]


def test_fp8_tier_matches_the_stock_engine(tmp_path_factory):
    if _gpus() < 1:
        pytest.skip("CUDA device unavailable")
    stock = run(tmp_path_factory, "reference", 1, "offload", True)
    kvoff = run(tmp_path_factory, "kvoff", 1, "offload", True)
    assert kvoff["stats"]["restored_blocks"] >= 1
    assert kvoff["stats"] == stock["stats"]
    assert kvoff["cached_tokens"] == stock["cached_tokens"]
    assert kvoff["outputs"] == stock["outputs"]


@pytest.mark.parametrize("fp8", [False, True])
def test_per_rank_tier_under_tensor_parallelism(tmp_path_factory, fp8):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    resident = run(tmp_path_factory, "kvoff", 2, "resident", False)
    offload = run(tmp_path_factory, "kvoff", 2, "offload", fp8)
    assert offload["stats"]["restored_blocks"] >= 1
    assert offload["cached_tokens"]["A2"] == resident["cached_tokens"]["A2"] > 0
    assert offload["outputs"]["A1"] == resident["outputs"]["A1"]
    assert offload["outputs"]["B1"] == resident["outputs"]["B1"]
    if not fp8:
        assert offload["outputs"]["A2"] == resident["outputs"]["A2"]
