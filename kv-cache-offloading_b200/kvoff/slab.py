"""Pinned, NUMA-local host slabs exposed as torch tensors.

A slab is one anonymous mapping placed on the NUMA node closest to the GPU
and page-locked with cudaHostRegister(Portable | Mapped) by kvoff_host_alloc.
It is wrapped as a uint8 CPU tensor (torch.frombuffer over the mapping), so
typed views of it behave like the reference's pin_memory=True slab chunks
(nanovllm/engine/cpu_prefix_cache.py:199-208) while copies see true pinned
memory, and zero-copy kernels get its device alias. The mapping is unpinned
and unmapped when the last tensor view of it is garbage collected.
"""

from __future__ import annotations

import ctypes
import weakref

import torch

from kvoff import _lib


def device_numa_node(device: int) -> int:
    """NUMA node of CUDA device `device` (-1 when the platform does not say)."""
    node = ctypes.c_int32(-1)
    _lib.call("kvoff_device_numa_node", int(device), ctypes.byref(node))
    return node.value


def _release(host_ptr: int) -> None:
    try:
        _lib.lib().kvoff_host_free(ctypes.c_void_p(host_ptr))
    except Exception:  # interpreter shutdown: the process exit frees it anyway
        pass


class PinnedSlab:
    """`nbytes` of pinned host memory with a device alias for zero-copy kernels."""

    def __init__(self, nbytes: int, device: int | None = None, numa_node: int | None = None):
        if nbytes <= 0:
            raise ValueError("slab size must be positive")
        if numa_node is None:
            numa_node = device_numa_node(device) if device is not None else -1
        host, dev = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.call("kvoff_host_alloc", int(nbytes), int(numa_node), ctypes.byref(host),
                  ctypes.byref(dev))
        self.nbytes = int(nbytes)
        self.host_ptr = int(host.value)
        self.device_ptr = int(dev.value)
        self.numa_node = numa_node
        buffer = (ctypes.c_uint8 * self.nbytes).from_address(self.host_ptr)
        weakref.finalize(buffer, _release, self.host_ptr)
        self.bytes = torch.frombuffer(buffer, dtype=torch.uint8)

    def view(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """Typed tensor of `shape` starting `offset` bytes into the slab."""
        count = 1
        for s in shape:
            count *= int(s)
        size = count * dtype.itemsize
        if offset < 0 or offset + size > self.nbytes or offset % dtype.itemsize:
            raise ValueError("view outside the slab or misaligned")
        return self.bytes[offset:offset + size].view(dtype).view(tuple(shape))

    def device_alias(self, tensor: torch.Tensor) -> int:
        """Device address of a host tensor inside this slab (for zero-copy kernels)."""
        offset = tensor.data_ptr() - self.host_ptr
        if not 0 <= offset < self.nbytes:
            raise ValueError("tensor is not inside this slab")
        return self.device_ptr + offset
