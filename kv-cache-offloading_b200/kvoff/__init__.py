"""kvoff - B200-native KV-cache offload copy path.

Drop-in replacements for the nano-vllm engine's block save / restore
(kvoff.cpu_prefix_cache, replacing nanovllm/engine/cpu_prefix_cache.py) and
slot-mapping store (kvoff.attention.store_kvcache, replacing
nanovllm/layers/attention.py:store_kvcache), running hand-written sm_100a
kernels from libkvoff.so through its C ABI (include/kvoff.h).
"""

from kvoff._lib import KvoffError, debug_fail_next, device_error, lib  # noqa: F401

__all__ = ["KvoffError", "debug_fail_next", "device_error", "lib"]
