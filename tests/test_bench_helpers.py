"""bench.py's host-side helpers, on CPU.

The host-core baseline must take its thread count from the process's CPU
affinity set (torchrun exports OMP_NUM_THREADS=1 to every rank), and the
comparators that run the reference's own code on the GPU must find it in its
installed copy: its CPUBlockCache, its Triton store_kvcache and its KV handoff
module, each loaded by file path without the package's model imports. The
loader is checked here without a GPU; it is skipped when the copy is absent.
"""

from __future__ import annotations

import os

import pytest

import bench

needs_copy = pytest.mark.skipif(not bench.REFERENCE_TREE.is_dir(),
                                reason="the reference's installed copy (baseline/_ref) is absent")


def test_host_threads_follow_the_affinity_set(monkeypatch):
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    assert bench.host_threads() == len(os.sched_getaffinity(0))


def test_cpu_sample_runs_on_the_requested_threads():
    w = bench.Workload("tiny", layers=2, num_blocks=8, heads=1, batch=2)
    sample = bench.cpu_sample(w, 0.05, threads=2)
    assert sample["cores"] == 2 and sample["value"] > 0 and sample["kind"] == "port"


@needs_copy
def test_reference_comparators_load_from_the_installed_copy():
    cache_cls = bench.reference_cache_class()
    assert cache_cls is not None and cache_cls.__module__ == "nanovllm.engine.cpu_prefix_cache"
    assert hasattr(cache_cls, "save_block") and not hasattr(cache_cls, "save_blocks")
    store = bench.reference_store_kvcache()
    assert callable(store), store
    assert store.__module__ == "nanovllm.layers.attention"
    handoff = bench.reference_module("nanovllm.engine.kv_handoff")
    assert callable(handoff.verify_imported_kv)
