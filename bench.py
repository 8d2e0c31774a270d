#!/usr/bin/env python
"""KV-cache offload copy path benchmark (one line of JSON).

Default workload, BASELINE config 2, per GPU: a Qwen3-8B-shaped paged KV pool
[2, 36, 320, 256, 8, 128] bf16 on the device (12.1 GB), filled with N(0,1)
values and 1% x20 outlier channels per (K/V, layer, KV head), and a pinned
NUMA-local host slab. One step saves 128 random blocks as FP8 while restoring
128 other saved blocks into 128 other GPU blocks, concurrently on a save stream
and a restore stream. `--workload config4` runs BASELINE config 4 instead: a
Qwen3-32B pool sharded by KV head ([2, 64, 2048, 256, 8 / tp, 128] per rank),
restoring 512 blocks (131,072 tokens) while saving 512 others.

* value  - the step with the slots in HBM (device-resident inputs): the fused
           gather+quantize and dequantize+scatter kernels alone.
* e2e    - the step through the C ABI with the slots in pinned host memory,
           PCIe transfers inside the timed region (save D2H, restore H2D).
Both are GB/s of KV processed, counted as bf16 bytes for saves plus restores;
tokens/s counts block_size tokens per block moved.

`--impl reference` times the reference algorithm on the host cores instead
(the C oracle port of the reference's CPU-pool save / restore path), with all
the host threads of the process's affinity set.
Multi-GPU (torchrun): every rank runs the workload on its own GPU and slab
(KV-head sharding needs no collective); time is the max over ranks. At N > 1
the line also carries `config4`: BASELINE config 4 on the same ranks (each
rank's KV-head shard, 512-block restore || 512-block save), after config 2.

At N=1 the line also reports the single-GPU characterizations: the staged /
mapped and BF16 mode sweep, the staging-depth and issue-order sweep of the e2e
step, the BF16 copy kernels, store_kvcache against the reference's own Triton
kernel, KV handoff, and the drop-in cache beside the reference's own
CPUBlockCache on the same GPU (both loaded from the reference's installed copy
under baseline/_ref when it is present).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "kv-cache-offloading_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

SWEEP_BATCHES = (1, 8, 32, 128)
FALLBACK_HBM_GBS = 6650.0
METRIC = "KV restore+save GB/s (FP8, bf16-equivalent bytes)"
# dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of a full
# 128-block config-2 launch of the save kernel (profiles/fp8_save_kernel_config2.md),
# per byte of bf16 block read; other batch sizes scale it by blocks per launch.
SAVE_KERNEL_DRAM_BYTES_PER_BF16_BYTE = (4_832_047_616 + 2_400_740_352) / (128 * 37_748_736)
TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one 128-block config-2 "
                  "launch (profiles/fp8_save_kernel_config2.md), scaled by blocks per launch")


@dataclass(frozen=True)
class Workload:
    name: str
    layers: int
    num_blocks: int
    heads: int
    batch: int
    block_size: int = 256
    head_dim: int = 128

    @property
    def rows(self) -> int:
        return 2 * self.layers * self.block_size * self.heads

    @property
    def bf16_block(self) -> int:
        return self.rows * self.head_dim * 2

    @property
    def fp8_payload(self) -> int:
        return self.rows * self.head_dim

    @property
    def fp8_scale(self) -> int:
        return self.rows * 2

    @property
    def fp8_block(self) -> int:
        return self.fp8_payload + self.fp8_scale

    @property
    def kernel_bytes(self) -> int:
        """HBM bytes one FP8 save (or restore) kernel moves per block."""
        return self.bf16_block + self.fp8_block

    def describe(self) -> str:
        return (f"{self.name}: paged KV [2,{self.layers},{self.num_blocks},{self.block_size},"
                f"{self.heads},{self.head_dim}] bf16 per GPU; FP8 save of {self.batch} random "
                f"blocks concurrent with FP8 restore of {self.batch} others, split streams")


def make_workload(args, world: int) -> Workload:
    if args.workload == "config4":
        tp = args.tp or world
        if 8 % tp:
            raise SystemExit("--tp must divide the 8 KV heads")
        return Workload("config4 (Qwen3-32B, KV heads sharded tp=%d)" % tp, layers=64,
                        num_blocks=args.pool_blocks or 2048, heads=8 // tp,
                        batch=args.batch or 512)
    return Workload("config2 (Qwen3-8B)", layers=36, num_blocks=args.pool_blocks or 320, heads=8,
                    batch=args.batch or 128)


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--workload", choices=("config2", "config4"), default="config2")
    p.add_argument("--tp", type=int, default=0, help="config4 KV-head shards (default: --gpus)")
    p.add_argument("--batch", type=int, default=0, help="blocks saved and restored per step")
    p.add_argument("--pool-blocks", type=int, default=0,
                   help="GPU pool size in blocks (smaller pools are for profiler captures)")
    p.add_argument("--slab-gib", type=float, default=24.0, help="pinned host slab per GPU")
    p.add_argument("--no-sweep", action="store_true", help="skip the batch-size / mode sweep")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-store", action="store_true", help="skip the store_kvcache measurement")
    p.add_argument("--no-handoff", action="store_true",
                   help="skip the KV handoff export / import measurement")
    p.add_argument("--no-dropin", action="store_true",
                   help="skip the per-block vs batched CPUBlockCache measurement")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length")
    p.add_argument("--staging-blocks", type=int, default=64,
                   help="FP8 staging depth (blocks) of the e2e step; at N=1 the arrangement "
                        "sweep may pick another")
    p.add_argument("--no-config4", action="store_true",
                   help="at N > 1, skip the extra config-4 (KV-head sharded) measurement")
    args = p.parse_args()
    if args.warmup < 3:
        p.error("--warmup must be >= 3")
    return args


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def emit(line: dict) -> None:
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# host-side helpers


def mem_available_bytes() -> int:
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def measured_peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


class ClockSampler:
    """nvidia-smi samples of one GPU while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.proc is None or self.file is None:
            return None
        self.file.seek(0)
        sm, max_sm, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.file.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != 7:
                continue
            try:
                sm.append(float(parts[0]))
                max_sm.append(float(parts[1]))
                power.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(max_sm),
                "power_w_max": max(power), "samples": len(sm), "reasons": sorted(reasons)}


# --------------------------------------------------------------------------
# reference arm: the reference's CPU-pool save/restore path, as the C oracle port

_CPU_STATE: dict = {}


def host_cpu() -> dict:
    """The host CPU the baseline ran on (model, usable and logical CPUs)."""
    model = ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"model": model, "affinity_cpus": len(os.sched_getaffinity(0)),
            "logical_cpus": os.cpu_count()}


def host_threads() -> int:
    """Host CPUs this process may run on (its affinity set).

    torchrun exports OMP_NUM_THREADS=1 to every rank; the host-core baseline
    sets its thread count from the affinity set instead, so that it uses the
    cores the job holds whatever the launcher exported.
    """
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def cpu_sample(w: Workload, seconds: float, threads: int | None = None) -> dict:
    """Save + restore FP8 blocks of the workload's shape on the host cores."""
    import numpy as np

    from oracle import oracle

    oracle.set_threads(threads or host_threads())
    cores = oracle.max_threads()
    if _CPU_STATE.get("workload") != w:  # 4 blocks: 2 saved + 2 restored per iteration
        rng = np.random.default_rng(0)
        x = rng.standard_normal((2, w.layers, 4, w.block_size, w.heads, w.head_dim),
                                dtype=np.float32)
        u = x.view(np.uint32).astype(np.uint64)
        pool = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        _CPU_STATE.update(workload=w, pool=pool,
                          slots=oracle.fp8_save_blocks(pool, [2, 3], fast=True))
    pool = _CPU_STATE["pool"]
    payload, scale = _CPU_STATE["slots"]

    def step():
        oracle.fp8_save_blocks(pool, [0, 1], fast=True)
        oracle.fp8_restore_blocks(pool, [2, 3], payload, scale, fast=True)

    step()
    iters, start = 0, time.perf_counter()
    while True:
        step()
        iters += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    return {"value": iters * 4 * w.bf16_block / elapsed / 1e9, "unit": "GB/s", "cores": cores,
            "kind": "port",
            "sample": f"{iters} x (FP8 save of 2 + restore of 2 blocks of the workload shape), "
                      f"{elapsed:.1f} s on {cores} OpenMP threads",
            "tokens_per_s": iters * 4 * w.block_size / elapsed,
            "ms_per_block": 1000 * elapsed / (iters * 4), "host": host_cpu()}


def torch_ops_sample(w: Workload, seconds: float) -> dict:
    """The reference's own CPU-pool path: its torch op chain on CPU tensors."""
    import numpy as np
    import torch

    from kvoff.cpu_prefix_cache import fp8_dequantize, fp8_quantize

    torch.set_num_threads(host_threads())
    bits = _CPU_STATE["pool"]
    pool = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    shape = (2, w.layers, w.block_size, w.heads, w.head_dim)
    payload = torch.empty(shape, dtype=torch.float8_e4m3fn)
    scale = torch.empty((*shape[:-1], 1), dtype=torch.bfloat16)
    iters, start = 0, time.perf_counter()
    while True:
        fp8_quantize(pool[:, :, 0], payload, scale)
        fp8_dequantize(payload, scale, pool[:, :, 2])
        iters += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    return {"GBps": iters * 2 * w.bf16_block / elapsed / 1e9, "threads": torch.get_num_threads(),
            "what": "reference fp8_quantize + fp8_dequantize torch ops on host tensors"}


def run_reference(args) -> None:
    rank, _, world = dist_env()
    if rank != 0:
        return  # rank 0 alone runs the host-core baseline
    w = make_workload(args, world)
    threads = host_threads()
    per_step = max(0.5, min(5.0, 120.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_sample(w, per_step / 4, threads)
    samples = [cpu_sample(w, per_step, threads) for _ in range(args.steps)]
    value = statistics.mean(s["value"] for s in samples)
    emit({"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
          "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": statistics.mean(s["ms_per_block"] for s in samples) * 4,
          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
          "data": "synthetic N(0,1), seed 0",
          "config": {"workload": w.describe(), "batch_blocks": w.batch,
                     "pool_blocks": w.num_blocks, "sample_blocks_per_step": 4,
                     "note": "host-core sample of the workload: each step saves 2 and "
                             "restores 2 blocks of the same shape (GB/s does not depend on "
                             "the batch on the host)",
                     "basis": "aggregate: the reference's CPU tier runs on the host's cores, "
                              "which serve every GPU of the job, so its whole-job throughput "
                              "is one sample on all the cores the job holds (the affinity "
                              "set, not the launcher's OMP_NUM_THREADS)",
                     "value_per_gpu": value / world},
          "cpu_baseline": {"value": value, "unit": "GB/s", "cores": samples[0]["cores"],
                           "kind": "port", "sample": samples[0]["sample"],
                           "host": samples[0]["host"]},
          "tokens_per_s": statistics.mean(s["tokens_per_s"] for s in samples),
          "torch_ops_cpu": torch_ops_sample(w, per_step),
          "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                  "d2h_bytes_per_step": 0}})


# --------------------------------------------------------------------------
# our arm


def fill_pool(pool, heads: int, seed: int) -> None:
    """N(0,1) with 1% of (K/V, layer, KV head, channel) channels scaled x20."""
    import torch

    gen = torch.Generator(device=pool.device)
    gen.manual_seed(seed)
    two, layers = pool.shape[:2]
    mask = torch.rand((two, layers, heads, pool.shape[-1]), generator=gen,
                      device=pool.device) < 0.01
    scale = torch.where(mask, 20.0, 1.0)
    for kv in range(two):
        for layer in range(layers):
            for first in range(0, pool.shape[2], 256):  # bounded fp32 temporaries
                part = pool[kv, layer, first:first + 256]
                chunk = torch.randn(part.shape, generator=gen, device=pool.device)
                part.copy_(chunk.mul_(scale[kv, layer]))


class Timer:
    """CUDA-event timing of K steps on `stream`, bracketed by sync (+ barrier)."""

    def __init__(self, torch, stream, world: int):
        self.torch, self.stream, self.world = torch, stream, world

    def run(self, step, steps: int, warmup: int) -> float:
        torch = self.torch
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if self.world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(self.stream)
        for _ in range(steps):
            step()
        end.record(self.stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(end)
        if self.world > 1:
            torch.distributed.barrier()
        return ms


def max_over_ranks(torch, value: float, device) -> float:
    if not torch.distributed.is_initialized():
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def store_kvcache_bench(torch, w: Workload, pool, args, hbm_peak: float) -> dict:
    """Prefill slot store (BASELINE config 5 shape): 4096 new tokens per step for
    each of the model's layers, from K/V views strided like a fused qkv
    projection (Qwen3-8B: q 4096 + k 1024 + v 1024 wide rows, a separate
    projection output per layer), into slots of the pool.

    Two slot patterns: "block_slots" is what a prefill gets from the block
    manager (16 random free blocks, 256 consecutive slots each); "random_slots"
    scatters every token to an independent random slot (a stress case: each
    2 KB row write opens its own DRAM page). Every 97th token is padding (-1).
    Algorithmic bytes per token and layer: K and V rows read and written
    (4 * H * D * 2) plus the 4-byte slot.

    Three timings per arm (kvoff and the reference's own Triton kernel):
    eager (one Python call per layer); graph (the 36 stores back to back in a
    CUDA graph, sources in HBM); forward (each layer's store between a kernel
    that writes that layer's qkv rows and a kernel that reads them, 36 layers
    in a CUDA graph, as the engine runs it; reported as the time the store
    adds over the same chain without it, with the rows fresh in L2).
    """
    from kvoff import ops

    device, caches = pool.device, pool  # the store overwrites slots of the pool
    tokens, q_width = 4096, 32 * w.head_dim
    kv_width = w.heads * w.head_dim
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    # One qkv projection output per layer (1.8 GB in all), so sources come from HBM.
    qkv = torch.randn((w.layers, tokens, q_width + 2 * kv_width), generator=gen,
                      device=device).to(torch.bfloat16)
    keys = [qkv[layer, :, q_width:q_width + kv_width].view(tokens, w.heads, w.head_dim)
            for layer in range(w.layers)]
    values = [qkv[layer, :, q_width + kv_width:].view(tokens, w.heads, w.head_dim)
              for layer in range(w.layers)]
    num_slots = w.num_blocks * w.block_size
    blocks = torch.randperm(w.num_blocks, generator=gen, device=device)[:tokens // w.block_size]
    patterns = {
        "block_slots": (blocks[:, None] * w.block_size
                        + torch.arange(w.block_size, device=device)).reshape(-1),
        "random_slots": torch.randperm(num_slots, generator=gen, device=device)[:tokens],
    }
    per_step = w.layers * tokens * (4 * kv_width * 2 + 4)
    out = {"tokens": tokens, "layers": w.layers, "algorithmic_bytes_per_step": per_step}
    ref_store = reference_store_kvcache()
    sink = torch.empty((w.layers, tokens, kv_width), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    bad = torch.zeros(1, dtype=torch.int32, device=device)
    for pattern, slots in patterns.items():
        slots = slots.to(torch.int32).contiguous()
        slots[::97] = -1  # padded positions are skipped

        def ours(slots=slots):
            for layer in range(w.layers):
                ops.store_kvcache(keys[layer], values[layer], caches[0, layer],
                                  caches[1, layer], slots)

        valid = slots >= 0
        idx = slots[valid].long()

        def torch_scatter(valid=valid, idx=idx):  # the reference kernel's semantics
            for layer in range(w.layers):
                caches[0, layer].view(-1, kv_width)[idx] = keys[layer].reshape(tokens, -1)[valid]
                caches[1, layer].view(-1, kv_width)[idx] = values[layer].reshape(tokens, -1)[valid]

        def reference(slots=slots):  # the reference's Triton kernel, unchanged
            for layer in range(w.layers):
                ref_store(keys[layer], values[layer], caches[0, layer], caches[1, layer], slots)

        # Eager: one Python call per layer, as in a prefill forward. Graph: the
        # same 36 launches captured in a CUDA graph, which isolates the kernel
        # from the host launch path (decode steps run this way under the
        # engine's graphs).
        def captured(fn):
            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                fn()  # first call outside the capture (Triton compiles here)
                with torch.cuda.graph(graph, stream=side):
                    fn()
            stream.wait_stream(side)
            return graph

        def forward(store_layer):
            def run():
                for layer in range(w.layers):
                    qkv[layer].mul_(1.0)  # the kernel that writes the layer's rows
                    store_layer(layer)
                    sink[layer].copy_(qkv[layer, :, :kv_width])  # a kernel after it
            return run

        def ours_layer(layer, slots=slots):
            ops.store_kvcache(keys[layer], values[layer], caches[0, layer], caches[1, layer],
                              slots)

        def reference_layer(layer, slots=slots):
            ref_store(keys[layer], values[layer], caches[0, layer], caches[1, layer], slots)

        arms = [("kvoff", ours, ours_layer)]
        if callable(ref_store):
            arms.append(("reference_triton", reference, reference_layer))
        res = {}
        graph = captured(forward(lambda layer: None))
        bare_ms = Timer(torch, stream, 1).run(graph.replay, args.steps, args.warmup) / args.steps
        del graph
        for arm, fn, layer_fn in arms:
            graph = captured(fn)
            for mode, run in (("eager", fn), ("graph", graph.replay)):
                ms = Timer(torch, stream, 1).run(run, args.steps, args.warmup) / args.steps
                res[f"{arm}_{mode}"] = {"ms_per_step": ms, "GBps": per_step / (ms / 1e3) / 1e9,
                                        "us_per_launch": 1e3 * ms / w.layers,
                                        "frac_of_hbm_peak": per_step / (ms / 1e3) / 1e9
                                        / hbm_peak}
            del graph
            graph = captured(forward(layer_fn))
            ms = Timer(torch, stream, 1).run(graph.replay, args.steps, args.warmup) / args.steps
            added = ms - bare_ms
            res[f"{arm}_forward"] = {"ms_per_step": ms, "ms_without_store": bare_ms,
                                     "us_added_per_layer": 1e3 * added / w.layers,
                                     "GBps": per_step / (added / 1e3) / 1e9}
            del graph
        ms = Timer(torch, stream, 1).run(torch_scatter, args.steps, args.warmup) / args.steps
        res["torch_index_put"] = {"ms_per_step": ms, "GBps": per_step / (ms / 1e3) / 1e9,
                                  "us_per_launch": 1e3 * ms / w.layers}
        if not callable(ref_store):
            res["reference_triton"] = {"unavailable": str(ref_store)[:200]}
        ops.store_kvcache(keys[0], values[0], caches[0, 0], caches[1, 0], slots, bad_slots=bad)
        out[pattern] = res
    torch.cuda.synchronize()
    out["bad_slots"] = int(bad.item())
    del keys, values, qkv, sink
    return out


def reference_store_kvcache():
    """The reference's store_kvcache (nanovllm/layers/attention.py:10-40: its
    Triton store_kvcache_kernel and launcher) from its installed copy, or the
    reason it cannot run here."""
    try:
        if reference_module("nanovllm.utils.context") is None:
            return "the reference's installed copy (baseline/_ref) is absent"
        return reference_module("nanovllm.layers.attention").store_kvcache
    except Exception as exc:  # e.g. its flash_attn or triton import failing
        return f"{type(exc).__name__}: {exc}"


def bf16_kernel_rates(torch, ops, w: Workload, pool, ids, hbm_peak: float, kernel_alone,
                      stream) -> dict:
    """The BF16 passthrough copy kernels on device memory: up to 64 blocks
    gathered from the pool into dense device slots (save) and scattered back
    (restore). Algorithmic HBM bytes: each block read once and written once
    (2 x 37.7 MB per config-2 block). The TMA bulk-copy kernel and the SM
    vector-copy kernel are ours; the copy engine (one cudaMemcpy2DAsync per
    block) is listed beside them.
    """
    n = min(64, len(ids))
    ids = ids[:n]
    slots = torch.empty((n, w.bf16_block), dtype=torch.uint8, device=pool.device)
    ptrs = [slots[i].data_ptr() for i in range(n)]
    nbytes = 2 * n * w.bf16_block
    out = {"blocks_per_launch": n, "bytes_per_launch": nbytes, "peak": hbm_peak}
    for name, code in (("tma_copy_kernel", ops.COPY_TMA), ("sm_copy_kernel", ops.COPY_SM),
                       ("copy_engine", ops.COPY_ENGINE)):
        for direction, restore in (("save", False), ("restore", True)):
            ms = kernel_alone(lambda code=code, restore=restore: ops.copy_blocks(
                pool, ids, ptrs, restore=restore, method=code, stream=stream), stream)
            achieved = nbytes / (ms / 1e3) / 1e9
            out[f"{name}_{direction}"] = {"launch_ms": ms, "achieved": achieved,
                                          "frac": achieved / hbm_peak}
    del slots
    return out


def handoff_bench(torch, w: Workload, pool, args) -> dict:
    """KV handoff of one sequence (nanovllm/engine/kv_handoff.py:34-135): export
    its written tokens from 32 random pool blocks into a dense host snapshot
    [2, L, tokens, H, D], and import a snapshot into 32 other blocks. 8191
    tokens, so the last block is partial. Ours: one strided DMA per block
    between the pool and pinned memory (ops.copy_tokens, what the drop-in
    export_kv / import_kv run). Reference path, as torch ops on this GPU:
    index_select + contiguous + pageable .cpu(), and .to(device) + one copy_ per
    block. Both are timed with the host waiting for the result, as export_kv
    returns a finished snapshot; the exported bytes are checked equal.
    """
    from kvoff import ops

    device = pool.device
    nblocks = 32
    count = nblocks * w.block_size - 1
    gen = torch.Generator().manual_seed(11)
    perm = torch.randperm(w.num_blocks, generator=gen)
    src, dst = perm[:nblocks].tolist(), perm[nblocks:2 * nblocks].tolist()
    shape = (2, w.layers, count, w.heads, w.head_dim)
    nbytes = 2 * w.layers * count * w.heads * w.head_dim * pool.element_size()
    pinned = torch.empty(shape, dtype=pool.dtype, pin_memory=True)
    index = torch.tensor(src, dtype=torch.int64, device=device)

    def ours_export():
        ops.copy_tokens(pool, src, count, pinned.data_ptr())
        torch.cuda.current_stream(device).synchronize()

    def ours_import():
        ops.copy_tokens(pool, dst, count, pinned.data_ptr(), restore=True)
        torch.cuda.current_stream(device).synchronize()

    snapshot = {}

    def ref_export():
        packed = pool.index_select(2, index).flatten(2, 3)
        snapshot["kv"] = packed[:, :, :count].contiguous().cpu()

    def ref_import():
        payload = snapshot["kv"].to(device=device)
        for logical, physical in enumerate(dst):
            start = logical * w.block_size
            end = min(start + w.block_size, count)
            pool[:, :, physical, :end - start].copy_(payload[:, :, start:end])
        torch.cuda.current_stream(device).synchronize()

    def seconds(fn, reps=5):
        fn()
        t = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t) / reps

    out = {"tokens": count, "blocks": nblocks, "bytes": nbytes}
    for name, fn in (("kvoff_export", ours_export), ("kvoff_import", ours_import),
                     ("torch_export", ref_export), ("torch_import", ref_import)):
        sec = seconds(fn)
        out[name] = {"ms": 1e3 * sec, "GBps": nbytes / sec / 1e9}
    out["export_bytes_equal"] = bool(torch.equal(pinned.view(torch.int16),
                                                 snapshot["kv"].view(torch.int16)))
    # verify_imported_kv after the import (dst now holds the snapshot): kvoff's
    # drop-in against the reference's own function, on the same blocks.
    ours_import()
    out["verify"] = handoff_verify(torch, w, pool, dst, count, pinned, seconds)
    out["verify_ms"] = out["verify"].get("kvoff", {}).get("ms")
    del pinned, snapshot
    return out


def handoff_verify(torch, w: Workload, pool, block_ids, count, snapshot_kv, seconds) -> dict:
    """Time verify_imported_kv (nanovllm/engine/kv_handoff.py:63-78) on an
    imported sequence: kvoff's drop-in (chunked native readback) and the
    reference's (one synchronous block readback at a time), both loaded with
    the reference's own engine modules from its installed copy."""
    import importlib
    from types import SimpleNamespace

    try:
        for dep in ("nanovllm.sampling_params", "nanovllm.engine.sequence",
                    "nanovllm.engine.handoff_timing"):
            if reference_module(dep) is None:
                return {"unavailable": "the reference's installed copy (baseline/_ref) is absent"}
        ours = importlib.import_module("kvoff.kv_handoff")
        reference = reference_module("nanovllm.engine.kv_handoff")
    except Exception as exc:  # context only; never fails the bench
        return {"error": f"{type(exc).__name__}: {str(exc)[:200]}"}
    runner = SimpleNamespace(world_size=1, block_size=w.block_size, kv_cache=pool)
    seq = SimpleNamespace(block_table=list(block_ids))
    snap = SimpleNamespace(num_cached_tokens=count, kv=snapshot_kv)
    nbytes = snapshot_kv.numel() * snapshot_kv.element_size()
    out = {}
    for name, module in (("kvoff", ours), ("reference", reference)):
        result = {}

        def run(module=module, result=result):
            result["equal"] = bool(module.verify_imported_kv(runner, seq, snap))

        sec = seconds(run, reps=3)
        out[name] = {"ms": 1e3 * sec, "GBps": nbytes / sec / 1e9, "verified": result["equal"]}
    return out


class _Block:
    def __init__(self, block_id: int):
        self.block_id, self.hash, self.token_ids = block_id, -1, []


REFERENCE_TREE = ROOT / "baseline" / "_ref" / "nanovllm_upstream" / "nanovllm"


def reference_module(name: str):
    """A module of the reference's installed copy (baseline/_ref), loaded by
    file path under its own package names without running the package's
    __init__ (which imports the model stack). None when the copy is absent."""
    import importlib.util
    import types

    relative = name.split(".", 1)[1].replace(".", "/") + ".py"
    path = REFERENCE_TREE / relative
    if not path.exists():
        return None
    if name in sys.modules:
        return sys.modules[name]
    parts = name.split(".")
    for depth in range(1, len(parts)):  # namespace stand-ins for the packages
        package = ".".join(parts[:depth])
        if package not in sys.modules:
            module = types.ModuleType(package)
            module.__path__ = [str(REFERENCE_TREE.joinpath(*parts[1:depth]))]
            sys.modules[package] = module
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def reference_cache_class():
    """The reference's own CPUBlockCache (nanovllm/engine/cpu_prefix_cache.py)."""
    for dep in ("nanovllm.sampling_params", "nanovllm.engine.sequence",
                "nanovllm.engine.block_manager"):
        if reference_module(dep) is None:
            return None
    module = reference_module("nanovllm.engine.cpu_prefix_cache")
    return module.CPUBlockCache if module is not None else None


def dropin_e2e(torch, w: Workload, pool, save_ids, restore_ids, args, timer, main,
               cache_cls=None) -> dict:
    """FP8 save + restore of the step's blocks through a CPUBlockCache.

    cache_cls None is kvoff's drop-in; the reference's own class gives the
    like-for-like comparator (same calls, same split streams and pinned slots,
    its torch quantizer and copies). per_block: one save_block / _copy_entry per
    block, the block manager's call pattern; batched (kvoff only): one
    save_blocks and one _copy_entries per step; staged_form: whether kvoff ran
    its staged calls serially (the default) or pipelined. The step joins both
    copy streams into the timing stream; each step discards the saved entries
    so that the next step saves them again.
    """
    from types import SimpleNamespace

    ours = cache_cls is None
    if ours:
        from kvoff.cpu_prefix_cache import CPUBlockCache as cache_cls

    B = len(save_ids)
    blocks = [_Block(i) for i in range(w.num_blocks)]
    manager = SimpleNamespace(blocks=blocks, block_size=w.block_size, hash_to_block_id={},
                              _cpu_prefix_cache=None, admission_blocked=False)
    runner = SimpleNamespace(world_size=1, block_size=w.block_size, kv_cache=pool)
    cache = cache_cls(runner, manager, 2 * B * (w.fp8_block + 4096), split_streams=True,
                      fp8=True, preallocate=True)

    def publish(block_id: int, tag: int) -> int:
        h = 1_000_000 + tag
        blocks[block_id].hash, blocks[block_id].token_ids = h, [tag] * w.block_size
        manager.hash_to_block_id[h] = block_id
        return h

    saves = [publish(b, i) for i, b in enumerate(save_ids)]
    sources = [publish(b, B + i) for i, b in enumerate(restore_ids)]
    for h in sources:
        cache.save_block(h)
    entries = [cache._entries[h] for h in sources]
    cache.synchronize()

    def join():
        for b in restore_ids:  # the engine's first use of each restored block
            cache.before_block_use(b)
        main.wait_stream(cache._copy_stream)  # the drains to host
        for h in saves:
            cache.discard(h)

    def per_block():
        for h, e, b in zip(saves, entries, restore_ids):
            cache.save_block(h)
            cache._copy_entry(e, b, wait=False)
        join()

    def batched():
        cache.save_blocks(saves)
        cache._copy_entries(entries, restore_ids, wait=False)
        join()

    out = {}
    steps = [("per_block", per_block)] + ([("batched", batched)] if ours else [])
    for name, step in steps:
        ms = timer.run(step, args.steps, args.warmup) / args.steps
        out[name] = 2 * B * w.bf16_block / (ms / 1e3) / 1e9
    # Host time per call on the engine thread (the GPU work is asynchronous):
    # 64 save_block calls, then 64 _copy_entry calls.
    n = min(64, B)
    main.synchronize()
    t0 = time.perf_counter()
    for h in saves[:n]:
        cache.save_block(h)
    t1 = time.perf_counter()
    for e, b in zip(entries[:n], restore_ids[:n]):
        cache._copy_entry(e, b, wait=False)
    t2 = time.perf_counter()
    join()
    main.synchronize()
    out["host_us_per_call"] = {"save_block": 1e6 * (t1 - t0) / n,
                               "_copy_entry": 1e6 * (t2 - t1) / n}
    if not ours:
        cache.close()
        return out
    # How long the compute stream waits before it may rewrite a block it just
    # saved (save_block, then before_block_reuse), against the wait for the
    # whole drain to host (the saved entry's event). Device time on the compute
    # stream; a sleep ahead of it keeps host enqueue time out of the interval.
    waits = {"reuse_wait_ms": [], "drain_ms": []}
    for i, h in enumerate(saves[:16] * 2):
        for name in waits:
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            main.synchronize()
            torch.cuda._sleep(4_000_000)  # about 2 ms, longer than the host calls below
            start.record(main)
            cache.save_block(h)
            if name == "reuse_wait_ms":
                cache.before_block_reuse(manager.hash_to_block_id[h])
            else:
                main.wait_event(cache._entries[h].saved)
            end.record(main)
            end.synchronize()
            if i >= 16:  # the first pass warms up
                waits[name].append(start.elapsed_time(end))
            cache.synchronize()
            cache.discard(h)
    out.update({name: statistics.median(v) for name, v in waits.items()})
    # The hybrid planner's restore cost at the batch sizes admission restores.
    out["restore_ms_per_block"] = {
        str(b): 1e3 * cache.measure_restore_s_per_block(repeats=max(1, 64 // b), batch=b)
        for b in SWEEP_BATCHES if b <= B}
    # The drop-in's staged-call form: serial (default) or pipelined (KVOFF_COPY_YIELD=0).
    out["staged_form"] = "serial" if cache._serial else "pipelined"
    cache.close()
    return out


def init_ranks(args):
    """One process per GPU: pick this rank's device and, for N > 1, join the
    process group (used only for barriers and the max-over-ranks timing)."""
    import torch

    rank, local_rank, world = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300),
                                             device_id=device)
    return rank, local_rank, world, device


def pcie_ceiling(torch, timer, concurrent, dev_buf, d2h_host, h2d_host, n_bytes: int,
                 block: int) -> dict:
    """Pinned cudaMemcpyAsync between `dev_buf` and two host ranges, per
    direction and in duplex, in several arrangements: one copy per direction
    issued D2H first or H2D first, one copy per block, and 4 MiB pieces. The
    best duplex total is the link's ceiling for concurrent save and restore."""
    cp = lambda d, s_: d.copy_(s_, non_blocking=True)  # noqa: E731
    dev_d2h, dev_h2d = dev_buf[:n_bytes], dev_buf[n_bytes:2 * n_bytes]

    def pieces(dst, src, size):
        return lambda: [cp(dst[k:k + size], src[k:k + size]) for k in range(0, n_bytes, size)]

    def rate(step, directions):
        ms = timer.run(step, 5, 3) / 5
        return directions * n_bytes / (ms / 1e3) / 1e9

    d2h = lambda: cp(d2h_host, dev_d2h)  # noqa: E731
    h2d = lambda: cp(dev_h2d, h2d_host)  # noqa: E731
    out = {"d2h": rate(concurrent(d2h, lambda: None), 1),
           "h2d": rate(concurrent(lambda: None, h2d), 1),
           "duplex_total": rate(concurrent(d2h, h2d), 2),
           "duplex_total_h2d_first": rate(concurrent(d2h, h2d, restore_first=True), 2),
           "duplex_total_block_copies": rate(concurrent(pieces(d2h_host, dev_d2h, block),
                                                        pieces(dev_h2d, h2d_host, block)), 2),
           "duplex_total_4mib_copies": rate(concurrent(pieces(d2h_host, dev_d2h, 4 << 20),
                                                       pieces(dev_h2d, h2d_host, 4 << 20)), 2),
           "bytes_per_direction": n_bytes}
    out["duplex_best"] = max(v for k, v in out.items() if k.startswith("duplex_total"))
    return out


def run_ours(args, w: Workload, rank: int, local_rank: int, world: int, device,
             extras: bool) -> dict:
    """Time `w` on this rank's GPU and return the bench line (rank 0 prints it).

    extras adds the single-GPU characterizations (mode and staging sweeps, BF16
    kernels, slot store, handoff, drop-in caches, torch-op comparison); the
    multi-GPU runs time only the contract's steps.
    """
    import numpy as np
    import torch

    from kvoff import ops
    from kvoff.slab import PinnedSlab

    B = w.batch
    if not 1 <= B <= w.num_blocks // 2:
        raise SystemExit("the batch must be at most half the pool")
    main = torch.cuda.current_stream(device)
    save_stream = torch.cuda.Stream(device)
    restore_stream = torch.cuda.Stream(device)
    timer = Timer(torch, main, world)
    sweep_batches = [b for b in SWEEP_BATCHES if b <= B] if extras and not args.no_sweep else []
    bf16_batch = max(sweep_batches, default=0)

    pool = torch.empty((2, w.layers, w.num_blocks, w.block_size, w.heads, w.head_dim),
                       dtype=torch.bfloat16, device=device)
    fill_pool(pool, w.heads, seed=1000 + rank)
    rng = np.random.default_rng(rank)
    perm = rng.permutation(w.num_blocks)
    save_ids = [int(i) for i in perm[:B]]
    restore_ids = [int(i) for i in perm[B:2 * B]]

    # Host slab: FP8 slots for B saves + B restore sources (payloads first,
    # then scales, as in a CPU-tier slab chunk), then BF16 slots for the sweep.
    fp8_bytes = 2 * B * w.fp8_block
    need = fp8_bytes + 2 * bf16_batch * w.bf16_block
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    budget = int(0.6 * mem_available_bytes() / max(1, local_world))
    slab_bytes = int(args.slab_gib * (1 << 30))
    if budget:
        slab_bytes = min(slab_bytes, max(need, budget))
    slab_bytes = max(slab_bytes, need)
    t0 = time.perf_counter()
    slab = PinnedSlab(slab_bytes, device=local_rank)
    pin_s = time.perf_counter() - t0

    def fp8_slot(i):
        return (slab.view(i * w.fp8_payload, (w.fp8_payload,), torch.uint8),
                slab.view(2 * B * w.fp8_payload + i * w.fp8_scale, (w.fp8_scale,), torch.uint8))

    save_slots = [fp8_slot(i) for i in range(B)]
    restore_slots = [fp8_slot(B + i) for i in range(B)]
    host_ptr = lambda slots, k: [s[k].data_ptr() for s in slots]  # noqa: E731
    mapped_ptr = lambda slots, k: [slab.device_alias(s[k]) for s in slots]  # noqa: E731
    bf16_slots = [slab.view(fp8_bytes + i * w.bf16_block, (w.bf16_block,), torch.uint8)
                  for i in range(2 * bf16_batch)]

    def fp8_staging(blocks):
        return {name: (torch.empty((blocks, w.fp8_payload), dtype=torch.uint8, device=device),
                       torch.empty((blocks, w.fp8_scale), dtype=torch.uint8, device=device))
                for name in ("save", "restore")}

    staging_blocks = min(B, args.staging_blocks)
    staging = fp8_staging(staging_blocks)
    bf16_staging = {name: torch.empty((min(B, 16), w.bf16_block), dtype=torch.uint8,
                                      device=device) for name in ("save", "restore")} \
        if bf16_batch else {}

    # Restore sources hold real FP8 blocks (saved once, untimed).
    ops.save_fp8_staged(pool, restore_ids, host_ptr(restore_slots, 0),
                        host_ptr(restore_slots, 1), *staging["save"], stream=main)
    torch.cuda.synchronize()

    # ---- device-resident step (value): slots in HBM -------------------------
    # A ring of at most 128 device slots per direction (reused round robin when
    # the batch is larger: same bytes moved, far more than L2 holds).
    ring = min(B, 128)
    dev_save = (torch.empty((ring, w.fp8_payload), dtype=torch.uint8, device=device),
                torch.empty((ring, w.fp8_scale), dtype=torch.uint8, device=device))
    dev_src = (torch.empty((ring, w.fp8_payload), dtype=torch.uint8, device=device),
               torch.empty((ring, w.fp8_scale), dtype=torch.uint8, device=device))
    for i in range(ring):
        dev_src[0][i].copy_(restore_slots[i][0])
        dev_src[1][i].copy_(restore_slots[i][1])
    dsp = [dev_save[0][i % ring].data_ptr() for i in range(B)]
    dss = [dev_save[1][i % ring].data_ptr() for i in range(B)]
    drp = [dev_src[0][i % ring].data_ptr() for i in range(B)]
    drs = [dev_src[1][i % ring].data_ptr() for i in range(B)]

    def concurrent(save_fn, restore_fn, restore_first=False):
        def step():
            save_stream.wait_stream(main)
            restore_stream.wait_stream(main)
            order = ((restore_stream, restore_fn), (save_stream, save_fn))
            for stream, fn in (order if restore_first else order[::-1]):
                with torch.cuda.stream(stream):
                    fn()
            main.wait_stream(save_stream)
            main.wait_stream(restore_stream)
        return step

    device_step = concurrent(
        lambda: ops.save_fp8(pool, save_ids, dsp, dss, stream=save_stream),
        lambda: ops.restore_fp8(pool, restore_ids, drp, drs, stream=restore_stream))

    gpu_name = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    with ClockSampler(gpu_name) as clocks_dev:
        ms = timer.run(device_step, args.steps, args.warmup)
    dev_ms_per_step = max_over_ranks(torch, ms, device) / args.steps
    value = world * 2 * B * w.bf16_block / (dev_ms_per_step / 1e3) / 1e9

    # ---- roofline: each kernel alone, timed on its own stream ----------------
    def kernel_alone(fn, stream):
        t = Timer(torch, stream, 1)
        with torch.cuda.stream(stream):
            return t.run(fn, args.steps, args.warmup) / args.steps

    launches_per_call = -(-B // 128)
    save_ms = kernel_alone(lambda: ops.save_fp8(pool, save_ids, dsp, dss, stream=save_stream),
                           save_stream)
    restore_ms = kernel_alone(lambda: ops.restore_fp8(pool, restore_ids, drp, drs,
                                                      stream=restore_stream), restore_stream)
    peaks = measured_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    peak_source = ("MEASURED_PEAKS.json hbm_gbs (burst copy)" if "hbm_gbs" in peaks
                   else "fallback 6650 GB/s")
    save_launch_ms = save_ms / launches_per_call
    blocks_per_launch = B / launches_per_call
    achieved = blocks_per_launch * w.kernel_bytes / (save_launch_ms / 1e3) / 1e9
    restore_launch_ms = restore_ms / launches_per_call
    restore_achieved = blocks_per_launch * w.kernel_bytes / (restore_launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak,
                "traffic": SAVE_KERNEL_DRAM_BYTES_PER_BF16_BYTE * w.bf16_block * blocks_per_launch,
                "traffic_source": TRAFFIC_SOURCE,
                "kernel": f"fp8_save_kernel (gather + quantize, {int(blocks_per_launch)} blocks "
                          "per launch)",
                "peak_source": peak_source, "algorithmic_bytes_per_block": w.kernel_bytes,
                "launch_ms": save_launch_ms,
                "restore_kernel": {"achieved": restore_achieved,
                                   "frac": restore_achieved / hbm_peak,
                                   "launch_ms": restore_launch_ms}}

    # ---- BF16 passthrough kernels, device-resident (pool <-> device slots) ----
    bf16_kernels = bf16_kernel_rates(torch, ops, w, pool, save_ids, hbm_peak, kernel_alone,
                                     save_stream) if extras else None

    # ---- end to end through the C ABI with pinned host slots -----------------
    def e2e_fns(batch, save_mode, restore_mode, stage=None):
        stage = stage or staging
        sids, rids = save_ids[:batch], restore_ids[:batch]
        ss, rs = save_slots[:batch], restore_slots[:batch]
        if save_mode == "mapped":
            sp, sc = mapped_ptr(ss, 0), mapped_ptr(ss, 1)
            save = lambda: ops.save_fp8(pool, sids, sp, sc, stream=save_stream)  # noqa: E731
        else:
            sp, sc = host_ptr(ss, 0), host_ptr(ss, 1)
            save = lambda: ops.save_fp8_staged(pool, sids, sp, sc,  # noqa: E731
                                               *stage["save"], stream=save_stream)
        if restore_mode == "mapped":
            rp, rc = mapped_ptr(rs, 0), mapped_ptr(rs, 1)
            restore = lambda: ops.restore_fp8(pool, rids, rp, rc,  # noqa: E731
                                              stream=restore_stream)
        else:
            rp, rc = host_ptr(rs, 0), host_ptr(rs, 1)
            restore = lambda: ops.restore_fp8_staged(pool, rids, rp, rc,  # noqa: E731
                                                     *stage["restore"], stream=restore_stream)
        return save, restore

    def bf16_fns(batch, method):
        sids, rids = save_ids[:batch], restore_ids[:batch]
        ss, rs = bf16_slots[:batch], bf16_slots[bf16_batch:bf16_batch + batch]
        if method == "tma":
            st_s, st_r = bf16_staging["save"], bf16_staging["restore"]
            depth = st_s.shape[0]

            def save():
                for k in range(0, batch, depth):
                    n = min(depth, batch - k)
                    ops.copy_blocks(pool, sids[k:k + n], [x.data_ptr() for x in st_s[:n]],
                                    method=ops.COPY_TMA, stream=save_stream)
                    ops.memcpy(ss[k].data_ptr(), st_s.data_ptr(), n * w.bf16_block,
                               device=device, stream=save_stream)

            def restore():
                for k in range(0, batch, depth):
                    n = min(depth, batch - k)
                    ops.memcpy(st_r.data_ptr(), rs[k].data_ptr(), n * w.bf16_block,
                               device=device, stream=restore_stream)
                    ops.copy_blocks(pool, rids[k:k + n], [x.data_ptr() for x in st_r[:n]],
                                    restore=True, method=ops.COPY_TMA, stream=restore_stream)
            return save, restore
        if method == "staged":
            sp, rp = [x.data_ptr() for x in ss], [x.data_ptr() for x in rs]
            save = lambda: ops.copy_blocks_staged(  # noqa: E731
                pool, sids, sp, bf16_staging["save"], stream=save_stream)
            restore = lambda: ops.copy_blocks_staged(  # noqa: E731
                pool, rids, rp, bf16_staging["restore"], restore=True, stream=restore_stream)
            return save, restore
        code = ops.COPY_SM if method == "sm" else ops.COPY_ENGINE
        sp = [slab.device_alias(x) if method == "sm" else x.data_ptr() for x in ss]
        rp = [slab.device_alias(x) if method == "sm" else x.data_ptr() for x in rs]
        save = lambda: ops.copy_blocks(pool, sids, sp, method=code, stream=save_stream)  # noqa
        restore = lambda: ops.copy_blocks(pool, rids, rp, restore=True,  # noqa: E731
                                          method=code, stream=restore_stream)
        return save, restore

    def rate(step, batch, directions, steps, warmup):
        ms = timer.run(step, steps, warmup) / steps
        return directions * batch * w.bf16_block / (ms / 1e3) / 1e9

    sweep = {}
    few = dict(steps=4, warmup=3)
    for batch in sweep_batches:
        row = {}
        for mode in ("staged", "mapped"):
            save, restore = e2e_fns(batch, mode, mode)
            row[f"fp8_{mode}"] = {
                "save": rate(concurrent(save, lambda: None), batch, 1, **few),
                "restore": rate(concurrent(lambda: None, restore), batch, 1, **few),
                "duplex": rate(concurrent(save, restore), batch, 2, **few)}
        for save_m, restore_m in (("mapped", "staged"), ("staged", "mapped")):
            save, restore = e2e_fns(batch, save_m, restore_m)
            row[f"fp8_save_{save_m}_restore_{restore_m}"] = {
                "duplex": rate(concurrent(save, restore), batch, 2, **few)}
        for method in ("staged", "engine", "tma", "sm"):
            save, restore = bf16_fns(batch, method)
            row[f"bf16_{method}"] = {
                "save": rate(concurrent(save, lambda: None), batch, 1, **few),
                "restore": rate(concurrent(lambda: None, restore), batch, 1, **few),
                "duplex": rate(concurrent(save, restore), batch, 2, **few)}
        sweep[str(batch)] = row
    best = sweep.get(str(bf16_batch), {})

    def duplex(save_m, restore_m):
        key = (f"fp8_{save_m}" if save_m == restore_m
               else f"fp8_save_{save_m}_restore_{restore_m}")
        return best.get(key, {}).get("duplex", 0.0)

    combos = [(a, b) for a in ("staged", "mapped") for b in ("staged", "mapped")]
    save_mode, restore_mode = max(combos, key=lambda c: duplex(*c)) if best else \
        ("staged", "staged")

    # Staging depth of the staged calls (blocks per staging buffer; each half
    # is drained by one cudaMemcpyAsync per run of consecutive slots), and the
    # issue order of the two directions, at the full batch.
    arrangement = {}
    if extras and not args.no_sweep and "staged" in (save_mode, restore_mode):
        for depth in sorted({8, 16, 32, 64} & set(range(2, B + 1)) | {staging_blocks}):
            stage = staging if depth == staging_blocks else fp8_staging(depth)
            save, restore = e2e_fns(B, save_mode, restore_mode, stage)
            for first in ("save", "restore"):
                arrangement[f"depth{depth}_{first}_first"] = rate(
                    concurrent(save, restore, restore_first=first == "restore"), B, 2, **few)
            del stage
    best_arrangement = max(arrangement, key=arrangement.get) if arrangement else None
    restore_first = bool(best_arrangement) and best_arrangement.endswith("restore_first")
    if best_arrangement:
        depth = int(best_arrangement[5:].split("_")[0])
        if depth != staging_blocks:
            staging_blocks, staging = depth, fp8_staging(depth)

    save, restore = e2e_fns(B, save_mode, restore_mode)
    e2e_step = concurrent(save, restore, restore_first=restore_first)
    with ClockSampler(gpu_name) as clocks_e2e:
        ms = timer.run(e2e_step, args.steps, args.warmup)
    e2e_ms = max_over_ranks(torch, ms, device) / args.steps
    e2e_value = world * 2 * B * w.bf16_block / (e2e_ms / 1e3) / 1e9
    groups = -(-B // max(1, staging_blocks // 2))
    launches = (launches_per_call if save_mode == "mapped" else groups) + \
        (launches_per_call if restore_mode == "mapped" else groups)

    # ---- prefill slot store (store_kvcache) ------------------------------------
    store = store_kvcache_bench(torch, w, pool, args, hbm_peak) \
        if extras and not args.no_store else None

    # ---- KV handoff export / import of one sequence ---------------------------
    handoff = handoff_bench(torch, w, pool, args) \
        if extras and not args.no_handoff and w.num_blocks >= 64 else None

    # ---- through drop-in caches: kvoff's (per-block and batched calls) and the
    # reference's own CPUBlockCache on the same GPU (like for like) -------------
    dropin = None
    if extras and w.batch <= 256 and not args.no_dropin:
        dropin = dropin_e2e(torch, w, pool, save_ids, restore_ids, args, timer, main)
        try:
            stock_cls = reference_cache_class()
            dropin["stock"] = (dropin_e2e(torch, w, pool, save_ids, restore_ids, args, timer,
                                          main, cache_cls=stock_cls) if stock_cls is not None
                               else {"unavailable": "the reference's installed copy "
                                                    "(baseline/_ref) is absent"})
        except Exception as exc:  # context only; never fails the bench
            dropin["stock"] = {"error": f"{type(exc).__name__}: {str(exc)[:200]}"}

    # ---- PCIe ceiling: pinned memcpy per direction and duplex -------------------
    # The slab's pages (mmap + cudaHostRegister, kvoff_host_alloc) and, beside
    # them, pages from cudaHostAlloc (torch's pinned allocator); every rank
    # copies at once, so at N > 1 this is the host's shared ceiling.
    blocks = min(B, 64, max(1, int(2.5e9 // w.fp8_block)))
    n_bytes = blocks * w.fp8_block
    dev_buf = torch.empty(2 * n_bytes, dtype=torch.uint8, device=device)
    ceiling = pcie_ceiling(torch, timer, concurrent, dev_buf, slab.bytes[:n_bytes],
                           slab.bytes[n_bytes:2 * n_bytes], n_bytes, w.fp8_block)
    host_alloc = torch.empty(2 * n_bytes, dtype=torch.uint8, pin_memory=True)
    ceiling["cuda_host_alloc"] = pcie_ceiling(torch, timer, concurrent, dev_buf,
                                              host_alloc[:n_bytes], host_alloc[n_bytes:],
                                              n_bytes, w.fp8_block)
    del dev_buf, host_alloc
    pcie_per_dir = B * w.fp8_block / (e2e_ms / 1e3) / 1e9

    # ---- the reference's device path (torch ops) for context ------------------
    ref_gpu = None
    try:
        if not extras:
            raise StopIteration  # measured at N=1 only
        from kvoff.cpu_prefix_cache import fp8_dequantize, fp8_quantize

        shape = (2, w.layers, w.block_size, w.heads, w.head_dim)
        stage_p = torch.empty(shape, dtype=torch.float8_e4m3fn, device=device)
        stage_s = torch.empty((*shape[:-1], 1), dtype=torch.bfloat16, device=device)
        few_ids = save_ids[:8]

        def aten_step():
            for b in few_ids:
                fp8_quantize(pool[:, :, b], stage_p, stage_s)
                fp8_dequantize(stage_p, stage_s, pool[:, :, restore_ids[0]])
        ms = Timer(torch, main, 1).run(aten_step, 3, 3) / 3
        ref_gpu = {"what": "reference fp8_quantize + fp8_dequantize as torch ops on this GPU",
                   "GBps": 2 * len(few_ids) * w.bf16_block / (ms / 1e3) / 1e9}
    except StopIteration:
        pass
    except Exception as exc:  # context only; never fails the bench
        ref_gpu = {"error": str(exc)[:200]}

    return {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,1) bf16 with 1% x20 outlier channels per (K/V, layer, KV head)",
        "config": {"workload": w.describe(), "batch_blocks": B, "pool_blocks": w.num_blocks,
                   "pool_bytes": pool.numel() * 2, "slab_bytes": slab_bytes,
                   "slab_pin_s": pin_s, "numa_node": slab.numa_node,
                   "staging_blocks": staging_blocks,
                   "l2": f"inputs larger than L2 ({2 * B * w.bf16_block / 1e9:.1f} GB of KV "
                         "per step)",
                   "parallelism": f"dp{world} (independent per-GPU pools and slabs, no "
                                  "collective)"},
        "tokens_per_s": world * 2 * B * w.block_size / (dev_ms_per_step / 1e3),
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": B * w.fp8_block,
                "d2h_bytes_per_step": B * w.fp8_block, "ms_per_step": e2e_ms,
                "tokens_per_s": world * 2 * B * w.block_size / (e2e_ms / 1e3),
                "save_mode": save_mode, "restore_mode": restore_mode,
                "issue_order": "restore first" if restore_first else "save first",
                "pcie_GBps_per_direction": pcie_per_dir,
                "pcie_frac_of_memcpy_d2h": pcie_per_dir / ceiling["d2h"],
                "pcie_frac_of_memcpy_h2d": pcie_per_dir / ceiling["h2d"],
                "pcie_frac_of_memcpy_duplex": 2 * pcie_per_dir / ceiling["duplex_total"],
                "pcie_frac_of_memcpy_duplex_best": 2 * pcie_per_dir / ceiling["duplex_best"],
                "memcpy_duplex_best_frac_of_solo": {
                    "d2h": ceiling["duplex_best"] / 2 / ceiling["d2h"],
                    "h2d": ceiling["duplex_best"] / 2 / ceiling["h2d"]}},
        "roofline": roofline,
        "bf16_kernels": bf16_kernels,
        "clocks": clocks_e2e.summary() or clocks_dev.summary(),
        # kvoff kernels launched inside the two timed regions (device step: one
        # save and one restore launch per 128 blocks; e2e: one kernel per
        # staging half, or per 128 blocks for mapped slots).
        "gpu_launches": (2 * launches_per_call + launches) * args.steps,
        "gpu_launches_by_region": {"value": 2 * launches_per_call * args.steps,
                                   "e2e": launches * args.steps},
        "pcie_memcpy_ceiling_GBps": ceiling,
        "e2e_arrangement_GBps": arrangement or None,
        "sweep_GBps": sweep,
        "dropin_e2e_GBps": dropin,
        "store_kvcache": store,
        "kv_handoff": handoff,
        "reference_gpu_path": ref_gpu,
    }


CONFIG4_KEYS = ("value", "ms_per_step", "tokens_per_s", "e2e", "roofline", "clocks",
                "pcie_memcpy_ceiling_GBps", "gpu_launches", "config")


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    rank, _, world = dist_env()
    w = make_workload(args, world)
    # The host-core baseline runs first, before the pool, the pinned slab and
    # the GPU work exist, so it sees the host as the reference arm does.
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_sample(w, args.cpu_seconds)
        cpu["torch_ops_cpu"] = torch_ops_sample(w, min(5.0, args.cpu_seconds))
    import gc

    import torch

    rank, local_rank, world, device = init_ranks(args)
    line = run_ours(args, w, rank, local_rank, world, device, extras=world == 1)
    line["cpu_baseline"] = cpu
    if world > 1 and args.workload == "config2" and not args.no_config4:
        # BASELINE config 4 on the same ranks: each rank's KV-head shard of a
        # Qwen3-32B pool, 512-block restore || 512-block save (weak in blocks
        # per rank; the pool shard shrinks as 8 / N heads).
        gc.collect()
        torch.cuda.empty_cache()
        args4 = argparse.Namespace(**{**vars(args), "workload": "config4", "tp": 0, "batch": 0,
                                      "pool_blocks": 0, "slab_gib": 0.0})
        w4 = make_workload(args4, world)
        line4 = run_ours(args4, w4, rank, local_rank, world, device, extras=False)
        line["config4"] = {k: line4[k] for k in CONFIG4_KEYS}
    if rank == 0:
        emit(line)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
