"""Shared pytest setup: import paths, the `gpu` marker and build-on-demand.

`-m "not gpu"` tests run anywhere (CPU only); `-m gpu` tests need a CUDA
device and call the hot path through libkvoff's C ABI.
"""

from __future__ import annotations

import gc
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_PARENT = ROOT / "kv-cache-offloading_b200"
for path in (ROOT, PACKAGE_PARENT, ROOT / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")
    # Build the native library and the oracle when sources are newer (no-op on a
    # box that received prebuilt files and has no compiler changes).
    from kvoff import build as kvoff_build
    from oracle import build as oracle_build

    if not kvoff_build.up_to_date():
        try:
            kvoff_build.build()
        except RuntimeError as exc:  # no nvcc: tests that need the library fail loudly
            print(f"warning: libkvoff build skipped: {exc}", file=sys.stderr)
    oracle_build.build()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device unavailable")
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _release_test_garbage():
    """Collect each test's garbage when it ends.

    Caches that sit in reference cycles (an automatic cache and its block
    manager, a cache whose copy methods a test wrapped) keep their pinned
    slabs until the cyclic garbage collector runs. Unpinning a slab
    (cudaHostUnregister) waits for the device, so a collection that happened
    to run inside a later test's timed region would stall its host thread
    behind that test's queued work. Collecting here frees them between tests.
    """
    yield
    gc.collect()
