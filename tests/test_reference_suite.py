"""Run the reference project's own test suite against the drop-in modules.

A temporary copy of the reference tree gets kvoff's cpu_prefix_cache.py and
kv_handoff.py in place of nanovllm/engine/cpu_prefix_cache.py and
nanovllm/engine/kv_handoff.py, then the reference's pytest suite runs
unmodified. On a CPU-only host its CUDA cases skip; the gpu-marked test runs
exactly those cases (CUDA pools, split streams, slowed copy streams, CUDA KV
import) on the GPU, where every copy goes through libkvoff. Skipped when no
reference checkout is available: KVOFF_REFERENCE, else a "reference" directory
beside this repository, else baseline/_ref inside it.
"""

from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KVOFF = ROOT / "kv-cache-offloading_b200" / "kvoff"
DROPINS = {"cpu_prefix_cache.py": KVOFF / "cpu_prefix_cache.py",
           "kv_handoff.py": KVOFF / "kv_handoff.py"}


def _reference() -> Path | None:
    if "KVOFF_REFERENCE" in os.environ:
        candidates = [Path(os.environ["KVOFF_REFERENCE"])]
    else:
        candidates = [ROOT.parent / "reference", ROOT / "baseline" / "_ref"]
    return next((path for path in candidates if (path / "bench").is_dir()), None)


REFERENCE = _reference()
needs_reference = pytest.mark.skipif(REFERENCE is None, reason="reference checkout not present")


def _run_suite(tmp_path: Path, *pytest_args: str) -> tuple[subprocess.CompletedProcess, str]:
    tree = tmp_path / "ref"
    shutil.copytree(REFERENCE / "bench", tree / "bench")
    shutil.copytree(REFERENCE / "nanovllm_upstream", tree / "nanovllm_upstream",
                    ignore=shutil.ignore_patterns("assets", "*.png"))
    engine = tree / "nanovllm_upstream" / "nanovllm" / "engine"
    for name, source in DROPINS.items():
        shutil.copyfile(source, engine / name)
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(
        [str(tree), str(ROOT / "kv-cache-offloading_b200")]), PYTHONDONTWRITEBYTECODE="1")
    result = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                             "bench", *pytest_args], cwd=tree, env=env, capture_output=True,
                            text=True, timeout=900)
    return result, result.stdout[-3000:] + result.stderr[-2000:]


def _count(word: str, stdout: str) -> int:
    found = re.search(rf"(\d+) {word}", stdout)
    return int(found.group(1)) if found else 0


@needs_reference
def test_reference_suite_passes_with_the_dropin(tmp_path):
    result, tail = _run_suite(tmp_path)
    assert result.returncode == 0, tail
    assert _count("passed", result.stdout) >= 170, tail
    assert " failed" not in result.stdout, tail


@pytest.mark.gpu
@needs_reference
def test_reference_cuda_cases_pass_with_the_dropin_on_the_gpu(tmp_path):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device unavailable")
    result, tail = _run_suite(tmp_path, "-k", "cuda")
    assert result.returncode == 0, tail
    # The reference's 15 CUDA cases: none may skip, so every one ran on the GPU.
    assert _count("passed", result.stdout) >= 15, tail
    assert _count("skipped", result.stdout) == 0, tail
    assert " failed" not in result.stdout, tail
