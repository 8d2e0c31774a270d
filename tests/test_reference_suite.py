"""Run the reference project's own test suite against the drop-in modules.

A temporary copy of the reference tree gets kvoff's cpu_prefix_cache.py and
kv_handoff.py in place of nanovllm/engine/cpu_prefix_cache.py and
nanovllm/engine/kv_handoff.py, then the reference's pytest suite runs
unmodified (its CUDA cases skip without a GPU). Skipped when the reference
checkout is not available (set KVOFF_REFERENCE to point at it).
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
# The reference checkout: KVOFF_REFERENCE, else a "reference" directory beside this repository.
REFERENCE = Path(os.environ.get("KVOFF_REFERENCE", ROOT.parent / "reference"))
KVOFF = ROOT / "kv-cache-offloading_b200" / "kvoff"
DROPINS = {"cpu_prefix_cache.py": KVOFF / "cpu_prefix_cache.py",
           "kv_handoff.py": KVOFF / "kv_handoff.py"}


@pytest.mark.skipif(not (REFERENCE / "bench").is_dir(), reason="reference checkout not present")
def test_reference_suite_passes_with_the_dropin(tmp_path):
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
                             "bench"], cwd=tree, env=env, capture_output=True, text=True,
                            timeout=600)
    tail = result.stdout[-3000:] + result.stderr[-2000:]
    assert result.returncode == 0, tail
    passed = int(re.search(r"(\d+) passed", result.stdout).group(1))
    assert passed >= 170, tail
    assert " failed" not in result.stdout, tail
