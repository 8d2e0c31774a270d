"""bench_replay.py wires the drop-ins into the reference engine it runs.

The agent-replay measurement (trajectories/min) runs the reference's own
harness and engine; its kvoff arm must actually use kvoff's CPU tier, KV
handoff, store_kvcache and the runner's tensor-parallel tier method, and its
reference arm must not. Checked on CPU in a
child process (the engine's modules are imported there, not here), without
running a model. Skipped when no reference checkout is available.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

from test_reference_suite import REFERENCE

ROOT = Path(__file__).resolve().parents[1]

PROBE = """
import json, sys
from pathlib import Path
sys.path.insert(0, {root!r})
import bench_replay
scratch = Path({scratch!r})
tree = bench_replay._engine_tree(Path({reference!r}), {impl!r}, scratch)
bench_replay._install(tree, {impl!r})
import transformers
import nanovllm.engine.llm_engine as llm_engine
import nanovllm.engine.model_runner as model_runner
import nanovllm.layers.attention as attention
print(json.dumps({{
    "store": attention.store_kvcache.__module__,
    "cache_has_batched_calls": hasattr(llm_engine.CPUBlockCache, "save_blocks"),
    "handoff": sys.modules["nanovllm.engine.kv_handoff"].__file__,
    "cache": sys.modules["nanovllm.engine.cpu_prefix_cache"].__file__,
    "loader": model_runner.load_model.__name__,
    "runner_tier": callable(getattr(model_runner.ModelRunner, "kvoff_tier", None)),
    "eos": transformers.AutoTokenizer.from_pretrained("unused").eos_token_id,
    "tree": str(tree),
}}))
"""


@pytest.mark.skipif(REFERENCE is None, reason="reference checkout not present")
@pytest.mark.parametrize("impl", ["kvoff", "reference"])
def test_replay_arms_bind_the_expected_modules(impl, tmp_path):
    code = PROBE.format(root=str(ROOT), reference=str(REFERENCE), impl=impl,
                        scratch=str(tmp_path))
    result = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                            timeout=600, cwd=ROOT)
    assert result.returncode == 0, result.stderr[-3000:]
    got = json.loads(result.stdout.strip().splitlines()[-1])
    assert got["loader"] == "_random_init"
    assert got["eos"] == 151645
    kvoff_dir = ROOT / "kv-cache-offloading_b200" / "kvoff"
    for name in ("handoff", "cache"):
        assert got[name].startswith(got["tree"])  # the engine tree's own module file
    same_handoff = Path(got["handoff"]).read_bytes() == (kvoff_dir / "kv_handoff.py").read_bytes()
    same_cache = Path(got["cache"]).read_bytes() == (kvoff_dir / "cpu_prefix_cache.py").read_bytes()
    assert same_handoff == same_cache == (impl == "kvoff")
    if impl == "kvoff":
        assert got["store"] == "kvoff.attention"
        assert got["cache_has_batched_calls"] and got["runner_tier"]
    else:
        assert got["store"] == "nanovllm.layers.attention"
        assert not (got["cache_has_batched_calls"] or got["runner_tier"])
