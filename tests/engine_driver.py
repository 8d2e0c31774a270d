"""Child-process driver: one offload-and-restore conversation in the reference engine.

Used by tests/test_gpu_engine.py. It builds a copy of the reference engine (stock,
or with kvoff's drop-ins as bench_replay.py puts them in place), writes a small
random Qwen3-architecture checkpoint (the engine's own loader reads it, in every
tensor-parallel rank), and runs three requests one after another through the
engine's public API with greedy sampling:

  A1: prompt PA                  -> 8 tokens
  B1: an unrelated prompt PB     -> 8 tokens (fills the pool, recycling A's blocks)
  A2: PA + A1's output + TA      -> 8 tokens (its prefix is a prefix-cache hit)

In the "resident" scenario the pool is large enough that A's blocks stay on
the GPU; in "offload" the pool is small and a CPU tier (automatic,
save-on-release, split streams; BF16 or FP8) saves A's blocks when B1 recycles
them and restores them when A2 is admitted. Writes a JSON file with the
outputs, the prefix-cache hit of each admission and the tier's block counts.

    python engine_driver.py --reference DIR --impl kvoff --tp 2 --scenario offload \
        --fp8 0 --out result.json
"""

from __future__ import annotations

import argparse
import atexit
import json
import random
import shutil
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

# Small Qwen3 architecture: 128-wide heads and 8 KV heads as in the Qwen3 family,
# so tensor parallelism up to 8 splits whole heads.
TINY_QWEN3 = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "attention_bias": False,
    "bos_token_id": 1, "eos_token_id": 2, "head_dim": 128, "hidden_act": "silu",
    "hidden_size": 512, "intermediate_size": 1024, "max_position_embeddings": 4096,
    "num_attention_heads": 16, "num_hidden_layers": 4, "num_key_value_heads": 8,
    "rms_norm_eps": 1e-06, "rope_scaling": None, "rope_theta": 1000000,
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "vocab_size": 4096,
}
POOL_BLOCKS = {"resident": 16, "offload": 6}


def write_checkpoint(model: Path) -> None:
    """config.json plus one seeded random safetensors file in the checkpoint's naming."""
    import torch
    from safetensors.torch import save_file

    c = TINY_QWEN3
    h, inter, d = c["hidden_size"], c["intermediate_size"], c["head_dim"]
    q, kv = c["num_attention_heads"] * d, c["num_key_value_heads"] * d
    shapes = {"model.embed_tokens.weight": (c["vocab_size"], h), "model.norm.weight": (h,),
              "lm_head.weight": (c["vocab_size"], h)}
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        shapes.update({
            p + "self_attn.q_proj.weight": (q, h), p + "self_attn.k_proj.weight": (kv, h),
            p + "self_attn.v_proj.weight": (kv, h), p + "self_attn.o_proj.weight": (h, q),
            p + "self_attn.q_norm.weight": (d,), p + "self_attn.k_norm.weight": (d,),
            p + "mlp.gate_proj.weight": (inter, h), p + "mlp.up_proj.weight": (inter, h),
            p + "mlp.down_proj.weight": (h, inter),
            p + "input_layernorm.weight": (h,), p + "post_attention_layernorm.weight": (h,),
        })
    gen = torch.Generator().manual_seed(1234)
    tensors = {}
    for name, shape in sorted(shapes.items()):
        if name.endswith("norm.weight"):
            tensors[name] = torch.ones(shape, dtype=torch.bfloat16)
        else:
            tensors[name] = (torch.randn(shape, generator=gen) * 0.05).to(torch.bfloat16)
    model.mkdir(parents=True)
    (model / "config.json").write_text(json.dumps(c))
    save_file(tensors, str(model / "model.safetensors"))


def converse(llm, sampling_params_cls, manager) -> tuple[dict, dict]:
    rng = random.Random(7)
    vocab = TINY_QWEN3["vocab_size"]
    pa = [rng.randrange(3, vocab) for _ in range(1000)]
    pb = [rng.randrange(3, vocab) for _ in range(1200)]
    ta = [rng.randrange(3, vocab) for _ in range(300)]

    hits: dict[int, int] = {}
    allocate = manager.allocate

    def tracked(seq, num_cached_blocks):
        result = allocate(seq, num_cached_blocks)
        span = getattr(seq, "restore_span", None)
        hits[seq.seq_id] = span[1] - span[0] if span else seq.num_cached_tokens
        return result

    manager.allocate = tracked

    def run(prompt):
        seq_id = llm.add_request(prompt, sampling_params_cls(temperature=0, max_tokens=8,
                                                             ignore_eos=True))
        outputs = {}
        while not llm.is_finished():
            for sid, ids in llm.step_with_events().outputs:
                outputs[sid] = list(ids)
        return seq_id, outputs[seq_id]

    out, cached = {}, {}
    for name, prompt in (("A1", lambda: pa), ("B1", lambda: pb),
                         ("A2", lambda: pa + out["A1"] + ta)):
        seq_id, out[name] = run(prompt())
        cached[name] = hits.get(seq_id)
    return out, cached


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", type=Path, required=True)
    parser.add_argument("--impl", choices=("kvoff", "reference"), required=True)
    parser.add_argument("--tp", type=int, default=1)
    parser.add_argument("--scenario", choices=sorted(POOL_BLOCKS), required=True)
    parser.add_argument("--fp8", type=int, default=0)
    parser.add_argument("--out", type=Path, required=True)
    args = parser.parse_args()

    sys.path.insert(0, str(ROOT))
    import bench_replay

    scratch = Path(tempfile.mkdtemp(prefix="kvoff_engine_"))
    try:
        tree = bench_replay._engine_tree(args.reference.resolve(), args.impl, scratch)
        model = scratch / "tiny-qwen3"
        write_checkpoint(model)
        bench_replay._install(tree, args.impl, random_weights=False,
                              eos_token_id=TINY_QWEN3["eos_token_id"])
        from nanovllm import LLM, SamplingParams

        llm = LLM(str(model), tensor_parallel_size=args.tp, enforce_eager=True, max_num_seqs=4,
                  max_num_batched_tokens=4096, max_model_len=4096,
                  num_kvcache_blocks=POOL_BLOCKS[args.scenario], gpu_memory_utilization=0.5)
        try:
            cache = None
            if args.scenario == "offload":
                cache = llm.create_cpu_prefix_cache(256 << 20, automatic=True,
                                                    save_on_release=True, split_streams=True,
                                                    fp8=bool(args.fp8))
            outputs, cached = converse(llm, SamplingParams, llm.scheduler.block_manager)
            stats = dict(cache.stats) if cache is not None else {}
        finally:
            atexit.unregister(llm.exit)  # the engine registers it; exit exactly once
            llm.exit()
    finally:
        shutil.rmtree(scratch, ignore_errors=True)
    args.out.write_text(json.dumps({"impl": args.impl, "tp": args.tp, "scenario": args.scenario,
                                    "fp8": bool(args.fp8), "outputs": outputs,
                                    "cached_tokens": cached, "stats": stats}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
