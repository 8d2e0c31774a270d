"""End-to-end agent replay (trajectories/min) in the reference engine, stock or with kvoff.

This runs the reference project's own multi-turn agent harness
(`bench/agent_replay.py`, `run_replay` :110-246) and its engine (the nano-vllm
fork) on one GPU, from a checkout of the reference given by `--reference`
(default `baseline/_ref`, a copy of the reference's `bench/` and
`nanovllm_upstream/` trees; it is not part of this repository). Two arms:

* `--impl kvoff`: the engine with kvoff's drop-ins put in place as the
  integration guide describes: `nanovllm/engine/cpu_prefix_cache.py` and
  `nanovllm/engine/kv_handoff.py` replaced by kvoff's modules,
  `nanovllm/layers/attention.py` importing `kvoff.attention.store_kvcache` over
  its Triton one, and the runner's `kvoff_tier` method (used only under tensor
  parallelism) added to `ModelRunner`.
* `--impl reference`: the stock engine (torch-op FP8 quantizer on the copy
  streams, the Triton `store_kvcache_kernel`).

Workloads (the agent-replay configurations of the hot path's benchmark plan):

* `config3`: Qwen3-8B architecture, 4 agents x 32,768-token prompts x 3 turns,
  2,048 tool-result tokens and 256 output tokens per turn, 5 s tool waits.
* `config5`: 4 agents x 12 turns, prompts growing from 4,096 to 35,842 tokens
  (2,758 tool-result tokens and 128 output tokens per turn), 5 s tool waits.
* `tiny`: a seconds-long shape with a pool small enough that every turn goes
  through the CPU tier, for checking that an arm runs at all.

Both agent-replay workloads use the reference's published settings: an
81,920-token (320-block) GPU pool, a 24 GiB FP8 CPU tier with save-on-release,
prefetch, split streams and hybrid admission, CUDA graphs, fixed output
lengths (`--ignore-eos`), and token ids drawn uniformly over the vocabulary by
the harness itself. Weights are random (N(0, 0.02), RMSNorm gains 1) because
no checkpoint is available; the harness feeds token ids, so the tokenizer is a
stand-in that only supplies the end-of-sequence id and decodes ids as text.

Prints one JSON line: trajectories/min and the harness's summary (TTFT, turn
latency, prefix reuse, CPU-tier block counts).

    python bench_replay.py --impl kvoff --workload config3 [--seed 7]
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
KVOFF_DIR = ROOT / "kv-cache-offloading_b200"
DROPINS = ("cpu_prefix_cache.py", "kv_handoff.py")
# The one method tensor parallelism needs on the engine's runner (every rank).
RUNNER_METHOD = """

def _kvoff_tier(self, op, *args):
    from kvoff.tp_tier import dispatch
    return dispatch(self, op, *args)


ModelRunner.kvoff_tier = _kvoff_tier
"""
STORE_DROPIN = """

from kvoff.attention import store_kvcache  # noqa: E402,F811  (kvoff's slot store)
"""

# Qwen3-8B architecture (the public model configuration's hyperparameters).
QWEN3_8B = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "attention_bias": False,
    "attention_dropout": 0.0, "bos_token_id": 151643, "eos_token_id": 151645, "head_dim": 128,
    "hidden_act": "silu", "hidden_size": 4096, "initializer_range": 0.02,
    "intermediate_size": 12288, "max_position_embeddings": 40960, "max_window_layers": 36,
    "num_attention_heads": 32, "num_hidden_layers": 36, "num_key_value_heads": 8,
    "rms_norm_eps": 1e-06, "rope_scaling": None, "rope_theta": 1000000, "sliding_window": None,
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "use_cache": True,
    "use_sliding_window": False, "vocab_size": 151936,
}

# The CPU-tier flags of the reference's published agent-replay runs.
CPU_TIER = ["--policy", "cpu_backed", "--cpu-cache-save-on-release", "--cpu-cache-prefetch",
            "--cpu-cache-split-streams", "--cpu-cache-fp8", "--cpu-cache-hybrid",
            "--cuda-graphs", "--ignore-eos", "--gpu-memory-utilization", "0.9"]



def tier_flags(tier: str) -> list[str]:
    """Harness flags for an FP8 or BF16 CPU tier, or for the GPU-only policy."""
    if tier == "none":
        return ["--policy", "gpu_only", "--cuda-graphs", "--ignore-eos",
                "--gpu-memory-utilization", "0.9"]
    return [flag for flag in CPU_TIER if tier == "fp8" or flag != "--cpu-cache-fp8"]


WORKLOADS = {
    "config3": ["--num-agents", "4", "--turns-per-agent", "3", "--initial-prompt", "32768",
                "--tool-result-tokens", "2048", "--output-tokens", "256", "--tool-wait-s", "5",
                "--num-kvcache-blocks", "320", "--cpu-cache-gib", "24",
                "--max-model-len", "40960", "--timeout-s", "900"],
    "config5": ["--num-agents", "4", "--turns-per-agent", "12", "--initial-prompt", "4096",
                "--tool-result-tokens", "2758", "--output-tokens", "128", "--tool-wait-s", "5",
                "--num-kvcache-blocks", "320", "--cpu-cache-gib", "24",
                "--max-model-len", "40960", "--timeout-s", "1200"],
    # 2 agents x 2 turns in a 12-block pool: the second turns restore from the CPU tier.
    "tiny": ["--num-agents", "2", "--turns-per-agent", "2", "--initial-prompt", "2048",
             "--tool-result-tokens", "512", "--output-tokens", "16", "--tool-wait-s", "0.5",
             "--num-kvcache-blocks", "12", "--cpu-cache-gib", "2", "--max-model-len", "4096",
             "--max-num-seqs", "8", "--timeout-s", "300"],
}


class _IdTokenizer:
    """Tokenizer stand-in: the replay passes token ids, so only eos and decode are used."""

    def __init__(self, eos_token_id: int):
        self.eos_token_id = eos_token_id

    def encode(self, text):
        raise ValueError("this replay passes token ids; there is no vocabulary to encode text")

    def decode(self, token_ids):
        return " ".join(map(str, token_ids))


def _random_init(model, path):
    """Stand-in for nanovllm.utils.loader.load_model: random weights, seeded."""
    import torch

    gen = torch.Generator(device="cuda").manual_seed(0)
    with torch.no_grad():
        for name, param in model.named_parameters():
            if name.endswith("norm.weight"):  # RMSNorm gains: input/post/q/k/final norms
                param.fill_(1.0)
            else:
                param.normal_(0.0, 0.02, generator=gen)


def _engine_tree(reference: Path, impl: str, scratch: Path) -> Path:
    """Copy the reference's bench/ and nanovllm/ trees and, for kvoff, put the drop-ins in place."""
    tree = scratch / "ref"
    shutil.copytree(reference / "bench", tree / "bench")
    shutil.copytree(reference / "nanovllm_upstream" / "nanovllm",
                    tree / "nanovllm_upstream" / "nanovllm")
    if impl == "kvoff":
        engine = tree / "nanovllm_upstream" / "nanovllm" / "engine"
        for name in DROPINS:
            shutil.copyfile(KVOFF_DIR / "kvoff" / name, engine / name)
        with open(engine / "model_runner.py", "a") as runner:
            runner.write(RUNNER_METHOD)
        # Rebinds the module's store_kvcache, which Attention.forward calls, in every
        # process that imports it (tensor-parallel ranks included).
        with open(engine.parent / "layers" / "attention.py", "a") as attention:
            attention.write(STORE_DROPIN)
    return tree


def _install(tree: Path, impl: str, random_weights: bool = True,
             eos_token_id: int = QWEN3_8B["eos_token_id"]) -> None:
    """Import the engine from the tree and bind the model-free stand-ins (and kvoff's store).

    random_weights=False keeps the engine's own loader, for a model directory
    that holds a checkpoint (tensor-parallel ranks load it in their own
    processes, where a stand-in bound here would not reach).
    """
    sys.path[:0] = [str(tree), str(tree / "nanovllm_upstream"), str(KVOFF_DIR)]
    import transformers

    import nanovllm.engine.model_runner as model_runner
    import nanovllm.layers.attention as attention

    if random_weights:
        model_runner.load_model = _random_init
    transformers.AutoTokenizer.from_pretrained = staticmethod(
        lambda *args, **kwargs: _IdTokenizer(eos_token_id))
    if impl == "kvoff":
        import nanovllm.engine.cpu_prefix_cache as cache

        if not (hasattr(cache.CPUBlockCache, "save_blocks")
                and attention.store_kvcache.__module__ == "kvoff.attention"
                and callable(getattr(model_runner.ModelRunner, "kvoff_tier", None))):
            raise RuntimeError("the engine tree did not pick up kvoff's drop-ins")


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--impl", choices=("kvoff", "reference"), default="kvoff")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="config3")
    parser.add_argument("--seed", type=int, default=7)
    parser.add_argument("--reference", type=Path, default=ROOT / "baseline" / "_ref",
                        help="checkout holding the reference's bench/ and nanovllm_upstream/")
    parser.add_argument("--out", type=Path, default=None,
                        help="directory for the harness's result.json and trace.json")
    parser.add_argument("--tier", choices=("fp8", "bf16", "none"), default="fp8",
                        help="CPU tier payload; none runs the harness's GPU-only policy "
                             "(no CPU tier, so --impl makes no difference to the copy path)")
    args = parser.parse_args()
    flags = tier_flags(args.tier) + WORKLOADS[args.workload]

    reference = args.reference.resolve()
    if not (reference / "bench" / "agent_replay.py").is_file():
        print(json.dumps({"metric": "trajectories/min", "impl": args.impl,
                          "workload": args.workload,
                          "unavailable": f"no reference checkout at {reference}"}))
        return 0
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("the agent replay needs a CUDA device")

    scratch = Path(tempfile.mkdtemp(prefix="kvoff_replay_"))
    try:
        tree = _engine_tree(reference, args.impl, scratch)
        model = scratch / "qwen3-8b-random"
        model.mkdir()
        (model / "config.json").write_text(json.dumps(QWEN3_8B))
        out = (args.out or scratch / "run").resolve()
        _install(tree, args.impl)
        from bench import agent_replay

        sys.argv = ["agent_replay", "--model", str(model), "--out", str(out),
                    "--seed", str(args.seed), *flags]
        started = time.perf_counter()
        agent_replay.main()
        wall = time.perf_counter() - started
        summary = json.loads((out / "result.json").read_text())["summary"]
    finally:
        shutil.rmtree(scratch, ignore_errors=True)

    print(json.dumps({
        "metric": "completed agent trajectories per minute", "unit": "traj/min",
        "value": summary["completed_trajectories_per_min"], "higher_is_better": True,
        "impl": args.impl, "workload": args.workload, "tier": args.tier, "seed": args.seed,
        "data": "synthetic (harness-seeded uniform token ids, random-init weights)",
        "gpu": torch.cuda.get_device_name(0), "process_wall_s": wall,
        "flags": flags, "summary": summary,
    }))
    return 0


if __name__ == "__main__":
    sys.exit(main())
