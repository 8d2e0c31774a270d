"""Drop-in store_kvcache for nanovllm/layers/attention.py.

The reference writes each new token's K and V rows into the paged cache with
a Triton kernel launched once per layer per step (attention.py:10-40). This
module keeps its signature and layout assertions and runs libkvoff's
16-byte-vectorized scatter instead: one launch, 64-bit slot offsets, slots of
-1 skipped, no allocation or host synchronization (CUDA-graph capturable).
"""

from __future__ import annotations

import torch

from kvoff import ops


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor):
    ops.store_kvcache(key, value, k_cache, v_cache, slot_mapping)
