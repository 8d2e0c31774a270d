"""Multi-rank logic on CPU with the gloo backend (world size 2).

Under tensor parallelism the KV pool shards by KV head (each rank holds
[2, L, NB, BS, H / t, D], nanovllm/engine/model_runner.py:110), and the FP8
codec keeps one scale per (token, KV head). So every rank can save and restore
its own heads with no exchange: the slots a rank produces for its heads are
exactly the head-slice of the unsharded slots. The test checks that property
with the oracle on each rank, plus the max-over-ranks timing reduction that
bench.py uses (the only collective it issues, and only for timing).
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    for p in (ROOT, ROOT / "tests", ROOT / "kv-cache-offloading_b200"):
        sys.path.insert(0, str(p))
    import torch
    import torch.distributed as dist

    import bench
    import workloads
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, num_blocks, block_size, heads, dim = 2, 3, 16, 8, 128
        full = workloads.pool_with_blocks(range(num_blocks), layers, num_blocks, block_size,
                                          heads, dim, seed=3)
        per = heads // world
        shard = np.ascontiguousarray(full[:, :, :, :, rank * per:(rank + 1) * per])
        payload, scale = oracle.fp8_save_blocks(shard, [2, 0])
        want_p, want_s = oracle.fp8_save_blocks(full, [2, 0])
        ok = (np.array_equal(payload, want_p[..., rank * per:(rank + 1) * per, :]) and
              np.array_equal(scale, want_s[..., rank * per:(rank + 1) * per, :]))
        # Restores of each rank's own slots rebuild its shard of the restored pool.
        oracle.fp8_restore_blocks(shard, [1], payload[:1], scale[:1])
        oracle.fp8_restore_blocks(full, [1], want_p[:1], want_s[:1])
        ok = ok and np.array_equal(shard, full[:, :, :, :, rank * per:(rank + 1) * per])
        slowest = bench.max_over_ranks(torch, float(10 + rank), "cpu")
        queue.put((rank, bool(ok), slowest))
    finally:
        dist.destroy_process_group()


def test_kv_head_shards_need_no_exchange_and_timing_takes_the_max():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(r for r, _, _ in results) == [0, 1]
    assert all(ok for _, ok, _ in results)
    assert all(slowest == 11.0 for _, _, slowest in results)
