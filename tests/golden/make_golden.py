"""Generate the golden fixtures from the reference implementation itself.

Runs the reference's own code on CPU (it is pure Python on torch) and writes
small fixtures that pin the CPU oracle and, through it, the CUDA library:

* fp8_rows.npz     - reference fp8_quantize / fp8_dequantize
                     (nanovllm/engine/cpu_prefix_cache.py:20-28) on rows that
                     cover every codec branch, for D in {4, 8, 16, 64, 128, 256},
                     plus dequantization of arbitrary payload / scale bits.
* dropin_tiny.npz  - the reference CPUBlockCache (cpu_prefix_cache.py:44-448)
                     with the reference BlockManager on the tiny pool of the
                     reference tests ([2, 2, NB, 256, 1, 4]; D = 4): BF16 byte
                     moves of arbitrary bit patterns and FP8 slots.
* config1.json     - BASELINE config 1 (Qwen3-0.6B-shaped pool [2, 28, 64,
                     256, 8, 128], N(0,1) + 1% x20 outlier channels, seed 0):
                     SHA-256 digests of the 16 saved FP8 slots (payload and
                     scales) and of the 16 restored blocks, plus the BF16
                     round trip, produced by the reference CPUBlockCache.
* store_kvcache.json - the reference's own store_kvcache
                     (nanovllm/layers/attention.py:10-40): its Triton kernel
                     runs on CPU tensors under Triton's interpreter
                     (TRITON_INTERPRET=1), on seeded inputs; digests of the
                     caches after the scatter. The torch-indexing restatement
                     must produce the same bytes.

The reference checkout is located by KVOFF_REFERENCE (default: a "reference"
directory beside this repository). Run from the repository root:

    python tests/golden/make_golden.py [--only store_kvcache ...]
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
from collections import deque
from pathlib import Path
from types import ModuleType, SimpleNamespace

# The reference's store_kvcache is a Triton kernel; the interpreter runs it on
# CPU tensors. The variable is read when the kernel's module is imported.
os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import workloads  # noqa: E402

# The reference checkout: KVOFF_REFERENCE, else a "reference" directory beside this repository.
REFERENCE = Path(os.environ.get("KVOFF_REFERENCE", HERE.parents[2] / "reference"))
ENGINE_ROOT = REFERENCE / "nanovllm_upstream" / "nanovllm"


def load_reference_engine():
    """Import the reference's cache + block manager without its CUDA model code."""
    sys.dont_write_bytecode = True
    for name, path in (("nanovllm", ENGINE_ROOT), ("nanovllm.engine", ENGINE_ROOT / "engine")):
        package = ModuleType(name)
        package.__path__ = [str(path)]
        sys.modules[name] = package
    modules = {}
    for name, rel in (("nanovllm.sampling_params", "sampling_params.py"),
                      ("nanovllm.engine.sequence", "engine/sequence.py"),
                      ("nanovllm.engine.block_manager", "engine/block_manager.py"),
                      ("nanovllm.engine.cpu_prefix_cache", "engine/cpu_prefix_cache.py")):
        spec = importlib.util.spec_from_file_location(name, ENGINE_ROOT / rel)
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
        modules[name.rsplit(".", 1)[1]] = module
    return modules["block_manager"], modules["cpu_prefix_cache"]


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw bit patterns of a bf16 / fp8 tensor as a numpy array."""
    view = {torch.bfloat16: torch.int16, torch.float8_e4m3fn: torch.uint8}[t.dtype]
    out = t.contiguous().view(view).numpy()
    return out.view(np.uint16) if view == torch.int16 else out


def bf16(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def fp8_rows(cache_mod) -> dict:
    quantize, dequantize = cache_mod.fp8_quantize, cache_mod.fp8_dequantize
    out = {}
    rng = np.random.default_rng(11)
    for d in (4, 8, 16, 64, 128, 256):
        x = workloads.special_rows(d, seed=5)
        src = bf16(x)
        payload = torch.empty(src.shape, dtype=torch.float8_e4m3fn)
        scale = torch.empty((*src.shape[:-1], 1), dtype=torch.bfloat16)
        quantize(src, payload, scale)
        restored = torch.empty_like(src)
        dequantize(payload, scale, restored)
        out[f"x_{d}"] = x
        out[f"payload_{d}"] = bits(payload)
        out[f"scale_{d}"] = bits(scale)
        out[f"deq_{d}"] = bits(restored)
        # Dequantization of arbitrary payload and scale bit patterns.
        p = rng.integers(0, 256, (32, d)).astype(np.uint8)
        s = rng.integers(0, 1 << 16, (32, 1)).astype(np.uint16)
        target = torch.empty((32, d), dtype=torch.bfloat16)
        dequantize(torch.from_numpy(p).view(torch.float8_e4m3fn), bf16(s), target)
        out[f"rp_{d}"], out[f"rs_{d}"], out[f"rdeq_{d}"] = p, s, bits(target)
    return out


def publish(manager, block_id: int, tokens: list[int]) -> int:
    h = manager.compute_hash(tokens)
    manager.blocks[block_id].update(h, tokens)
    manager.hash_to_block_id[h] = block_id
    return h


def round_trip(bm_mod, cache_mod, pool: torch.Tensor, sources, targets, fp8: bool):
    """Save `sources` through the reference cache, restore them into `targets`."""
    num_blocks, block_size = pool.shape[2], pool.shape[3]
    manager = bm_mod.BlockManager(num_blocks, block_size)
    hashes = [publish(manager, b, [1000 + i] * block_size) for i, b in enumerate(sources)]
    runner = SimpleNamespace(world_size=1, block_size=block_size, kv_cache=pool)
    per_block = pool[:, :, 0].numel() * pool.element_size()
    cache = cache_mod.CPUBlockCache(runner, manager, len(sources) * per_block, fp8=fp8)
    for h in hashes:
        assert cache.save_block(h)
    slots = [cache._entries[h] for h in hashes]
    payload = np.stack([bits(e.kv) for e in slots])
    scale = np.stack([bits(e.scale) for e in slots]) if fp8 else None
    for h in hashes:  # forget the GPU copies; restores go to `targets` in order
        manager.blocks[manager.hash_to_block_id.pop(h)].hash = -1
    rest = [b for b in range(num_blocks) if b not in targets]
    manager.free_block_ids = deque([*targets, *rest])
    restored_ids = [cache.restore_block(h) for h in hashes]
    assert restored_ids == list(targets), restored_ids
    restored = np.stack([bits(pool[:, :, b]) for b in targets])
    return payload, scale, restored


def dropin_tiny(bm_mod, cache_mod) -> dict:
    out = {}
    shape = (2, 2, 4, 256, 1, 4)
    n = int(np.prod(shape))
    # Arbitrary byte patterns (NaN encodings included), as the reference's
    # byte-exactness tests fill the pool (bench/test_cpu_prefix_cache.py:15-18).
    raw = (np.arange(2 * n, dtype=np.int64) % 256).astype(np.uint8)
    pool = torch.from_numpy(raw.view(np.int16).reshape(shape).copy()).view(torch.bfloat16)
    out["bf16_pool"] = bits(pool).copy()
    payload, _, restored = round_trip(bm_mod, cache_mod, pool, [1, 3], [0, 2], fp8=False)
    out["bf16_slots"], out["bf16_restored"] = payload, restored
    # Finite values as the reference's cached_engine fixture builds them
    # (bench/test_engine_handoff.py:16-19): arange % 251 in bf16.
    pool = torch.arange(n).remainder(251).to(torch.bfloat16).reshape(shape)
    out["fp8_pool"] = bits(pool).copy()
    payload, scale, restored = round_trip(bm_mod, cache_mod, pool, [2, 0], [1, 3], fp8=True)
    out["fp8_payload"], out["fp8_scale"], out["fp8_restored"] = payload, scale, restored
    return out


def config1(bm_mod, cache_mod) -> dict:
    c = workloads.CONFIG1
    sources, targets = workloads.config1_ids(c["seed"], c["num_blocks"], c["saved"])
    pool_bits = workloads.pool_with_blocks(range(c["num_blocks"]), c["layers"], c["num_blocks"],
                                           c["block_size"], c["heads"], c["head_dim"], c["seed"])
    result = {"config": c, "sources": sources, "targets": targets}
    for fp8 in (True, False):
        pool = bf16(pool_bits.copy())
        payload, scale, restored = round_trip(bm_mod, cache_mod, pool, sources, targets, fp8)
        key = "fp8" if fp8 else "bf16"
        result[key] = {
            "payload_sha256": [digest(p) for p in payload],
            "restored_sha256": [digest(r) for r in restored],
        }
        if fp8:
            result[key]["scale_sha256"] = [digest(s) for s in scale]
            src = torch.from_numpy(pool_bits[:, :, sources].view(np.int16)).view(
                torch.bfloat16).float()
            back = bf16(np.stack(restored, axis=2)).float()
            amax = src.abs().amax(-1, keepdim=True)
            result[key]["max_err_over_amax"] = float(((back - src).abs() / amax).max())
            result[key]["within_amax_over_16"] = bool(((back - src).abs() <= amax / 16).all())
    return result


def reference_store_kvcache():
    """store_kvcache of the reference (nanovllm/layers/attention.py:10-40)."""
    if "nanovllm" not in sys.modules:
        package = ModuleType("nanovllm")
        package.__path__ = [str(ENGINE_ROOT)]
        sys.modules["nanovllm"] = package
    spec = importlib.util.spec_from_file_location("nanovllm.layers.attention",
                                                  ENGINE_ROOT / "layers" / "attention.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module.store_kvcache


def store_kvcache_fixture() -> dict:
    store = reference_store_kvcache()
    out = {}
    for name, (n, h, d, nb, bs, pad) in workloads.STORE_CASES.items():
        qkv, slots, k_in, v_in = workloads.store_kvcache_inputs(name)
        rows = torch.from_numpy(qkv.view(np.int16)).view(torch.bfloat16)
        k = rows[:, pad:pad + h * d].view(n, h, d)
        v = rows[:, pad + h * d:].view(n, h, d)
        k_cache, v_cache = bf16(k_in.copy()), bf16(v_in.copy())
        store(k, v, k_cache, v_cache, torch.from_numpy(slots))  # the reference kernel
        # The restatement the oracle follows must give the same bytes.
        k_check, v_check = bf16(k_in.copy()), bf16(v_in.copy())
        m = torch.from_numpy(slots) != -1
        idx = torch.from_numpy(slots.astype(np.int64))[m]
        k_check.view(-1, h * d)[idx] = k.reshape(n, -1)[m]
        v_check.view(-1, h * d)[idx] = v.reshape(n, -1)[m]
        assert np.array_equal(bits(k_cache), bits(k_check)), name
        assert np.array_equal(bits(v_cache), bits(v_check)), name
        out[name] = {"k_cache_sha256": digest(bits(k_cache)),
                     "v_cache_sha256": digest(bits(v_cache)),
                     "source": "reference Triton store_kvcache_kernel under TRITON_INTERPRET=1"}
    return out


FIXTURES = ("fp8_rows", "dropin_tiny", "store_kvcache", "config1")


def main():
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--only", nargs="+", choices=FIXTURES, default=list(FIXTURES))
    only = set(parser.parse_args().only)
    if not ENGINE_ROOT.exists():
        raise SystemExit(f"reference checkout not found at {REFERENCE}")
    torch.manual_seed(0)
    bm_mod, cache_mod = load_reference_engine()
    if "fp8_rows" in only:
        np.savez_compressed(HERE / "fp8_rows.npz", **fp8_rows(cache_mod))
    if "dropin_tiny" in only:
        np.savez_compressed(HERE / "dropin_tiny.npz", **dropin_tiny(bm_mod, cache_mod))
    if "store_kvcache" in only:
        (HERE / "store_kvcache.json").write_text(
            json.dumps(store_kvcache_fixture(), indent=1) + "\n")
    if "config1" in only:
        (HERE / "config1.json").write_text(json.dumps(config1(bm_mod, cache_mod), indent=1) + "\n")
    meta = {"torch": torch.__version__, "numpy": np.__version__,
            "threads": torch.get_num_threads()}
    (HERE / "generated_with.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
