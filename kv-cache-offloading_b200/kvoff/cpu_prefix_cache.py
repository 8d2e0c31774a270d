"""Drop-in CPU block tier for the nano-vllm engine, with B200-native copies.

This module replaces nanovllm/engine/cpu_prefix_cache.py of the reference
(xxdydx/KV-Cache-Offloading). Its surface is unchanged: CPUBlockCache with the
same constructor, properties, public methods, the hooks the block manager calls
(_preserve_before_recycle, _preserve_on_release, before_block_reuse,
before_block_use, _entry_for, _copy_entry, _prefetched_blocks) and the private
attributes the reference tests read (_copy_stream, _restore_stream, _slabs,
_scale_slabs, _slot_view, _entries, _SLAB_CHUNK_BYTES). Bookkeeping - keys,
budget, slot recycling, publish-after-copy, error behaviour and messages -
follows the reference (cpu_prefix_cache.py:44-448).

What changes is the copy path for a CUDA pool. Instead of about ten ATen
launches plus torch copies per block, a save is one libkvoff call on the copy
stream: a fused gather + FP8 quantize kernel feeding a DMA drain into a
NUMA-local pinned slab slot (or writing the slot directly over PCIe), or one
strided DMA for BF16. Restores mirror it on the restore stream. Stream and
event ordering is the reference's: a save starts after the current stream's
writes of the block and after earlier restores that read the slot; a restore
starts after its own save; block reuse waits for pending copies. A pool on the
CPU (the reference's host-only test mode) keeps the reference's synchronous
torch copies and quantizer below.
"""

from __future__ import annotations

import contextlib

import os
from dataclasses import dataclass
from math import prod

import torch

# Pinned memory is allocated in chunks of about this size: one allocation and
# one page-locking call cover many slots.
_SLAB_CHUNK_BYTES = 1 << 30


# Largest finite float8_e4m3fn magnitude.
_FP8_MAX = 448.0


def fp8_quantize(source: torch.Tensor, payload: torch.Tensor, scale: torch.Tensor):
    """float8_e4m3fn payload plus one scale (in scale's dtype) per last-dim vector.

    The scale is rounded to its storage dtype first and the payload divides by
    the rounded value, so dequantization is its exact inverse up to e4m3 rounding.
    """
    amax = source.abs().amax(dim=-1, keepdim=True).to(torch.float32)
    scale.copy_(torch.clamp_min(amax / _FP8_MAX, 1e-30))
    ratio = source.to(torch.float32) / scale.to(torch.float32)
    payload.copy_(ratio.clamp_(-_FP8_MAX, _FP8_MAX))


def fp8_dequantize(payload: torch.Tensor, scale: torch.Tensor, target: torch.Tensor):
    """target = payload * scale, computed in target's dtype."""
    torch.mul(payload.to(target.dtype), scale, out=target)


@dataclass(frozen=True)
class _CPUBlock:
    token_ids: tuple[int, ...]
    kv: torch.Tensor  # slot view [K/V, layer, token, KV head, head dim]
    slot: int
    scale: torch.Tensor | None = None  # FP8: [K/V, layer, token, KV head, 1]
    saved: torch.cuda.Event | None = None  # CUDA: the save into `slot` has finished


class CPUCacheFullError(MemoryError):
    """The configured payload budget cannot admit another block."""


class _FollowerManager:
    """Layout-only stand-in for the block manager of a tensor-parallel follower
    rank (its bookkeeping lives on rank 0)."""

    def __init__(self, num_blocks: int, block_size: int):
        self.blocks = range(num_blocks)
        self.block_size = block_size
        self.hash_to_block_id: dict[int, int] = {}
        self._cpu_prefix_cache = None
        self.admission_blocked = False


# Copy methods for CUDA pools. FP8: "staged" (kernel into device staging,
# DMA drain) or "mapped" (kernel reads/writes the pinned slot over PCIe).
# BF16: "staged" (TMA gather / scatter kernels on one half of a device staging
# buffer while plain DMA moves the other half, one native call), "engine" (one
# strided DMA per block), "tma" (the TMA kernel and the DMA as separate calls
# in stream order) or "sm" (vector-copy kernel over PCIe). Override with
# KVOFF_FP8_SAVE / KVOFF_FP8_RESTORE / KVOFF_BF16_SAVE / KVOFF_BF16_RESTORE.
# BF16 defaults to "staged": a strided (2D) DMA straight into or out of the
# pool holds up the compute stream's own small copies queued behind it, so a
# prefill that overlaps a run of restores stalls until they drain; and a
# staged save frees its block for reuse once the gather kernel has read it,
# not after the drain to host.
DEFAULT_MODES = {"fp8_save": "staged", "fp8_restore": "staged",
                 "bf16_save": "staged", "bf16_restore": "staged"}
_MODE_CHOICES = {"fp8_save": ("staged", "mapped"), "fp8_restore": ("staged", "mapped"),
                 "bf16_save": ("staged", "engine", "tma", "sm"),
                 "bf16_restore": ("staged", "engine", "tma", "sm")}


def _transfer_modes() -> dict[str, str]:
    modes = {}
    for key, default in DEFAULT_MODES.items():
        value = os.environ.get(f"KVOFF_{key.upper()}", default)
        if value not in _MODE_CHOICES[key]:
            raise ValueError(f"KVOFF_{key.upper()} must be one of {_MODE_CHOICES[key]}")
        modes[key] = value
    return modes


class CPUBlockCache:
    """Bounded pinned-host store of full KV blocks keyed by chained prefix hash.

    Call from the engine-owning thread between steps. The byte budget counts
    payloads (FP8: e4m3 payload plus one bf16 scale per token and KV head).
    Restored GPU blocks are ordinary recyclable blocks; the CPU copy lives until
    discard / clear / close. On CUDA all copies are asynchronous on the copy
    stream (and a separate restore stream with split_streams=True, so both PCIe
    directions run at once); call synchronize() before reading slots on the
    host. automatic / save_on_release / prefetch / hybrid integrate with the
    block manager exactly as in the reference engine.
    """

    def __init__(self, runner, block_manager, max_bytes: int, *,
                 automatic: bool = False, save_on_release: bool = False, preallocate: bool = False,
                 prefetch: bool = False, split_streams: bool = False, fp8: bool = False,
                 hybrid: tuple[float, float, float] | None = None):
        if type(max_bytes) is not int or max_bytes <= 0:
            raise ValueError("max_bytes must be a positive integer")
        tensor_parallel = runner.world_size != 1
        if tensor_parallel and not callable(getattr(runner, "kvoff_tier", None)):
            # Per-rank tiers need the engine's runner to forward kvoff_tier calls.
            raise NotImplementedError("CPU prefix blocks currently require TP=1")
        if not automatic and (save_on_release or prefetch or hybrid):
            raise ValueError("save_on_release, prefetch and hybrid require automatic=True")
        if hybrid is not None and (len(hybrid) != 3 or min(hybrid) < 0):
            raise ValueError("hybrid needs three nonnegative cost coefficients")
        pool = runner.kv_cache
        layout_ok = (pool.ndim == 6 and pool.shape[0] == 2 and min(pool.shape) > 0
                     and pool.shape[2] == len(block_manager.blocks)
                     and pool.shape[3] == block_manager.block_size
                     and runner.block_size == block_manager.block_size)
        if not layout_ok:
            raise ValueError("KV pool layout does not match the block manager")
        if pool.device.type not in ("cpu", "cuda"):
            raise ValueError("KV pool must be on CPU or CUDA")
        if tensor_parallel and pool.device.type != "cuda":
            raise ValueError("a tensor-parallel CPU tier needs CUDA KV pools")
        self._manager = block_manager
        self._setup_storage(pool, fp8, split_streams)
        # Under tensor parallelism every rank stores its own KV heads of each
        # block; the budget counts the block's payload over all ranks.
        self._tp_runner = runner if tensor_parallel else None
        self._block_bytes = self._slot_bytes * runner.world_size
        self._max_bytes = max_bytes
        self._capacity = max_bytes // self._block_bytes
        self._entries: dict[int, _CPUBlock] = {}
        self._hybrid = hybrid
        self._save_on_release = save_on_release
        self._prefetch = prefetch
        self._prefetched_blocks = 0
        self._saved_blocks = 0
        self._restored_blocks = 0
        self._budget_skips = 0
        if tensor_parallel:
            self._rpc("init", fp8, split_streams)
        if automatic:
            if block_manager._cpu_prefix_cache is not None:
                raise RuntimeError("block manager already has an automatic CPU cache")
            block_manager._cpu_prefix_cache = self
        if preallocate:
            while self._num_slots < self._capacity:
                self._grow()

    def _setup_storage(self, pool: torch.Tensor, fp8: bool, split_streams: bool):
        """Slot layout, slabs, copy streams and ordering events for `pool`."""
        self._cache = pool
        self._fp8 = fp8
        self._shape = (2, pool.shape[1], *pool.shape[3:])
        self._scale_shape = (*self._shape[:-1], 1)
        self._dtype = torch.float8_e4m3fn if fp8 else pool.dtype
        self._payload_bytes = prod(self._shape) * self._dtype.itemsize
        self._scale_bytes = prod(self._scale_shape) * pool.element_size() if fp8 else 0
        self._slot_bytes = self._payload_bytes + self._scale_bytes
        self._slabs: list[torch.Tensor] = []
        self._scale_slabs: list[torch.Tensor] = []
        self._slab_owners: list = []  # PinnedSlab per chunk (CUDA pools)
        self._free_slots: list[int] = []
        self._num_slots = 0
        self._slot_loc: list[tuple[int, int]] = []  # slot -> (slab chunk, index in it)
        # slot -> (payload, scale) host pointers and their device aliases (CUDA pools)
        self._slot_ptrs: list[tuple[int, int, int, int]] = []
        self._on_cuda = pool.device.type == "cuda"
        self._copy_stream = self._restore_stream = None
        self._slot_reads: dict[int, torch.cuda.Event] = {}  # slot -> last restore reading it
        self._slot_saved: dict[int, torch.cuda.Event] = {}  # slot -> its save (TP followers)
        self._pending_saves: dict[int, torch.cuda.Event] = {}  # GPU block -> save done
        self._pending_restores: dict[int, torch.cuda.Event] = {}  # GPU block -> restore done
        self._staging: dict = {}
        if self._on_cuda:
            from kvoff import ops  # the native library is required for CUDA pools

            self._ops = ops
            self._geometry = ops.geometry(pool)
            if fp8 and pool.dtype != torch.bfloat16:
                raise ValueError("fp8=True needs a bf16 KV pool")
            self._modes = _transfer_modes()
            self._staging_blocks = max(1, int(os.environ.get("KVOFF_STAGING_BLOCKS", "2")))
            self._batch_staging_blocks = max(
                1, int(os.environ.get("KVOFF_BATCH_STAGING_BLOCKS", "8")))
            self._copy_stream = torch.cuda.Stream(pool.device)
            self._restore_stream = (torch.cuda.Stream(pool.device) if split_streams
                                    else self._copy_stream)
            self._ready = torch.cuda.Event()  # re-recorded before each staged save
            # Serial staged calls (staging_blocks = 1 at the C ABI) leave the
            # copy engine idle while each block's kernel runs, so the engine's
            # per-step input and sampled-token copies are not held behind a run
            # of block transfers; KVOFF_COPY_YIELD=0 pipelines the kernels on
            # the library's stream instead (more raw throughput, measured
            # slower inside the engine).
            self._serial = os.environ.get("KVOFF_COPY_YIELD", "1") != "0"

    # -- tensor parallelism ----------------------------------------------------
    #
    # Rank 0's cache (the leader) keeps all bookkeeping and copies its own KV
    # heads; every device operation is mirrored to the other ranks through the
    # engine's runner RPC (runner.call("kvoff_tier", op, ...), see
    # kvoff.tp_tier), where a follower cache performs the same ordered copies on
    # that rank's shard of the pool, into the same slot numbers.

    @classmethod
    def _follower(cls, runner, fp8: bool, split_streams: bool) -> "CPUBlockCache":
        self = cls.__new__(cls)
        pool = runner.kv_cache
        self._manager = _FollowerManager(pool.shape[2], pool.shape[3])
        self._setup_storage(pool, fp8, split_streams)
        self._tp_runner = None
        self._block_bytes = self._slot_bytes
        self._max_bytes = self._capacity = 1 << 62  # slots are chosen by the leader
        self._entries = {}
        self._hybrid = None
        self._save_on_release = self._prefetch = False
        self._prefetched_blocks = self._saved_blocks = self._restored_blocks = 0
        self._budget_skips = 0
        return self

    def _rpc(self, op: str, *args):
        if self._tp_runner is not None:
            from kvoff.tp_tier import send

            send(self._tp_runner, op, *args)

    def _tp_grow(self, count: int):
        self._grow(count)

    def _tp_save(self, block_ids, slots):
        done = self._save_on_device(block_ids, slots)
        for slot in slots:
            self._slot_saved[slot] = done

    def _tp_restore(self, slots, block_ids, wait: bool):
        entries = [_CPUBlock((), None, slot, None, self._slot_saved.get(slot)) for slot in slots]
        self._copy_entries(entries, block_ids, wait)

    def _tp_before_reuse(self, block_ids):
        for block_id in block_ids:
            self.before_block_reuse(block_id)

    def _tp_before_use(self, block_ids):
        for block_id in block_ids:
            self.before_block_use(block_id)

    def _tp_synchronize(self):
        self.synchronize()

    # -- properties ---------------------------------------------------------

    @property
    def max_bytes(self) -> int:
        return self._max_bytes

    @property
    def block_bytes(self) -> int:
        return self._block_bytes

    @property
    def bytes_used(self) -> int:
        return len(self._entries) * self._block_bytes

    @property
    def reserved_bytes(self) -> int:
        return self._num_slots * self._block_bytes

    @property
    def closed(self) -> bool:
        return self._cache is None

    @property
    def automatic(self) -> bool:
        return not self.closed and self._manager._cpu_prefix_cache is self

    @property
    def prefetch_enabled(self) -> bool:
        return self._prefetch

    @property
    def hybrid(self) -> tuple[float, float, float] | None:
        return self._hybrid

    @hybrid.setter
    def hybrid(self, costs: tuple[float, float, float] | None):
        """Split-admission costs, e.g. after measure_restore_s_per_block()."""
        if costs is not None:
            if not self.automatic:
                raise ValueError("hybrid requires an automatic cache")
            if len(costs) != 3 or min(costs) < 0:
                raise ValueError("hybrid needs three nonnegative cost coefficients")
            costs = tuple(float(c) for c in costs)
        self._hybrid = costs

    @property
    def fp8(self) -> bool:
        return self._fp8

    @property
    def prefetched_blocks(self) -> int:
        return self._prefetched_blocks

    @property
    def stats(self) -> dict[str, int]:
        return {"saved_blocks": self._saved_blocks, "restored_blocks": self._restored_blocks,
                "budget_skips": self._budget_skips}

    def __len__(self):
        return len(self._entries)

    def __contains__(self, prefix_hash: int):
        return prefix_hash in self._entries

    def _require_open(self):
        if self.closed:
            raise RuntimeError("CPU prefix cache is closed")

    # -- slots ----------------------------------------------------------------

    def _grow(self, count: int | None = None):
        """Add one slab chunk of slots (pinned and NUMA-local for CUDA pools)."""
        if count is None:
            count = min(max(1, _SLAB_CHUNK_BYTES // self._block_bytes),
                        self._capacity - self._num_slots)
            self._rpc("grow", count)
        if self._on_cuda:
            from kvoff.slab import PinnedSlab

            scale_offset = -(-count * self._payload_bytes // 256) * 256
            slab = PinnedSlab(scale_offset + count * self._scale_bytes,
                              device=self._cache.device.index)
            payload = slab.view(0, (count, *self._shape), self._dtype)
            scales = (slab.view(scale_offset, (count, *self._scale_shape), self._cache.dtype)
                      if self._fp8 else None)
            self._slab_owners.append(slab)
        else:
            payload = torch.empty((count, *self._shape), dtype=self._dtype, device="cpu")
            scales = (torch.empty((count, *self._scale_shape), dtype=self._cache.dtype,
                                  device="cpu") if self._fp8 else None)
        chunk = len(self._slabs)
        self._slabs.append(payload)
        if self._fp8:
            self._scale_slabs.append(scales)
        self._slot_loc.extend((chunk, i) for i in range(count))
        if self._on_cuda:
            pb, sb = self._payload_bytes, self._scale_bytes
            p0, pa = payload.data_ptr(), slab.device_alias(payload)
            s0, sa = (scales.data_ptr(), slab.device_alias(scales)) if self._fp8 else (0, 0)
            self._slot_ptrs.extend(
                (p0 + i * pb, s0 + i * sb if sb else 0, pa + i * pb, sa + i * sb if sb else 0)
                for i in range(count))
        first = self._num_slots
        self._free_slots.extend(range(first + count - 1, first - 1, -1))
        self._num_slots += count

    def _locate(self, slot: int) -> tuple[int, int]:
        if slot < 0:
            raise IndexError(slot)
        return self._slot_loc[slot]

    def _slot_view(self, slot: int) -> tuple[torch.Tensor, torch.Tensor | None]:
        chunk, index = self._locate(slot)
        return self._slabs[chunk][index], self._scale_slabs[chunk][index] if self._fp8 else None

    def _stage(self, stream, blocks: int = 0,
               serial: bool = False) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Per-stream device staging (FP8 payloads + scales, or raw blocks).

        Work on one stream runs in order, so reusing its staging is safe. It
        holds _staging_blocks blocks (2 by default: the staged FP8 calls then
        overlap the kernel of one block with the DMA of the previous one); a
        batched call grows it to min(blocks, _batch_staging_blocks) so a run of
        blocks drains in few, large DMA copies. serial=True (the staged calls'
        serial form) needs one block. A replaced buffer is released in stream
        order, after every copy that used it.
        """
        want = 1 if serial else max(self._staging_blocks, min(blocks, self._batch_staging_blocks))
        staged = self._staging.get(stream)
        if staged is None or staged[0].shape[0] < want:
            device = self._cache.device
            if staged is not None:  # kernels of earlier calls may still use it
                self._ops.join_pipeline(device, stream)
            with torch.cuda.stream(stream):  # owned by, and reused in order on, `stream`
                scales = (torch.empty((want, self._scale_bytes), dtype=torch.uint8,
                                      device=device) if self._fp8 else None)
                staged = (torch.empty((want, self._payload_bytes), dtype=torch.uint8,
                                      device=device), scales)
            self._staging[stream] = staged
        return staged

    # -- device copies (CUDA pools) ---------------------------------------------

    def _slot_pointers(self, slot: int, mapped: bool) -> tuple[int, int]:
        payload, scale, payload_alias, scale_alias = self._slot_ptrs[slot]
        return (payload_alias, scale_alias) if mapped else (payload, scale)

    def _pointers(self, slots, mapped: bool) -> tuple[list[int], list[int]]:
        pairs = [self._slot_pointers(slot, mapped) for slot in slots]
        return [p for p, _ in pairs], [s for _, s in pairs]

    def _device_save(self, pool: torch.Tensor, block_ids, slots, stream, wait_events=None,
                     source_done=None):
        """Enqueue pool blocks -> slots on `stream` (one native call per method).

        wait_events / source_done apply to staged saves (FP8 and BF16).
        """
        ops, modes = self._ops, self._modes
        if self._fp8:
            mapped = modes["fp8_save"] == "mapped"
            payload, scale = self._pointers(slots, mapped)
            if mapped:
                ops.save_fp8(pool, block_ids, payload, scale, stream=stream)
            else:
                self._staged_call(True, pool, block_ids, payload, scale, stream,
                                  wait_events or (), source_done)
            return
        method = modes["bf16_save"]
        payload, _ = self._pointers(slots, method == "sm")
        if method == "staged":
            self._staged_call(True, pool, block_ids, payload, None, stream, wait_events or (),
                              source_done)
        elif method == "tma":
            staged, _ = self._stage(stream, len(block_ids))
            for first in range(0, len(block_ids), len(staged)):
                ids = block_ids[first:first + len(staged)]
                ops.copy_blocks(pool, ids, [staged[i].data_ptr() for i in range(len(ids))],
                                method=ops.COPY_TMA, stream=stream)
                for i in range(len(ids)):
                    ops.memcpy(payload[first + i], staged[i].data_ptr(), self._payload_bytes,
                               device=pool.device, stream=stream)
        else:
            ops.copy_blocks(pool, block_ids, payload, stream=stream,
                            method=ops.COPY_SM if method == "sm" else ops.COPY_ENGINE)

    def _device_restore(self, pool: torch.Tensor, block_ids, plain, mapped, stream,
                        done_event=None):
        """Enqueue slots -> pool blocks on `stream`; plain / mapped are the slots'
        (payload, scale) host pointers and device aliases. done_event applies to
        staged restores (FP8 and BF16)."""
        ops, modes = self._ops, self._modes
        if self._fp8:
            if modes["fp8_restore"] == "mapped":
                ops.restore_fp8(pool, block_ids, *mapped, stream=stream)
            else:
                self._staged_call(False, pool, block_ids, *plain, stream, (), done_event)
            return
        method = modes["bf16_restore"]
        if method == "staged":
            self._staged_call(False, pool, block_ids, plain[0], None, stream, (), done_event)
        elif method == "tma":
            staged, _ = self._stage(stream, len(block_ids))
            for first in range(0, len(block_ids), len(staged)):
                ids = block_ids[first:first + len(staged)]
                for i in range(len(ids)):
                    ops.memcpy(staged[i].data_ptr(), plain[0][first + i], self._payload_bytes,
                               device=pool.device, stream=stream)
                ops.copy_blocks(pool, ids, [staged[i].data_ptr() for i in range(len(ids))],
                                restore=True, method=ops.COPY_TMA, stream=stream)
        elif method == "sm":
            ops.copy_blocks(pool, block_ids, mapped[0], restore=True, method=ops.COPY_SM,
                            stream=stream)
        else:
            ops.copy_blocks(pool, block_ids, plain[0], restore=True, stream=stream)

    def _staged_call(self, save: bool, pool: torch.Tensor, block_ids, payload, scale, stream,
                     wait_events, event):
        """One staged call (FP8: ops._fp8_staged_ev; BF16: ops._copy_staged_ev,
        with scale None) with raw handles, the cache's own geometry and no
        per-call tensor checks. wait_events and event are recorded
        torch.cuda.Events or None."""
        staged_payload, staged_scale = self._stage(stream, len(block_ids), self._serial)
        blocks = 1 if self._serial else staged_payload.shape[0]
        if scale is not None:
            blocks = min(blocks, staged_scale.shape[0])
        g = self._geometry if pool is self._cache else self._ops.geometry(pool)
        waits = [e.cuda_event for e in wait_events]
        handle = event.cuda_event if event is not None else 0
        index = pool.device.index
        guard = (contextlib.nullcontext() if torch.cuda.current_device() == index
                 else torch.cuda.device(index))
        with guard:
            if scale is None:
                self._ops._copy_staged_ev(save, g, pool.data_ptr(), block_ids, payload,
                                          staged_payload.data_ptr(), blocks, stream.cuda_stream,
                                          waits, handle)
            else:
                self._ops._fp8_staged_ev(save, g, pool.data_ptr(), block_ids, payload, scale,
                                         staged_payload.data_ptr(), staged_scale.data_ptr(),
                                         blocks, stream.cuda_stream, waits, handle)

    def _restore_slots(self, slots, block_ids, stream) -> torch.cuda.Event:
        """Restore slots into pool blocks on `stream`; returns the done event.

        A staged restore (FP8 or BF16) records the event after its last
        dequantize or scatter kernel (on the library's kernel stream), so
        `stream` is free to start the next restore's copies while those kernels
        run; other methods record it on `stream` after the copies.
        """
        done = torch.cuda.Event()
        done.record(stream)  # creates the CUDA event; a staged restore re-records it
        staged = self._modes["fp8_restore" if self._fp8 else "bf16_restore"] == "staged"
        self._device_restore(self._cache, block_ids, self._pointers(slots, False),
                             self._pointers(slots, True), stream,
                             done_event=done if staged else None)
        if not staged:
            done.record(stream)
        return done

    # -- host copies (CPU pools: the reference's synchronous path) ---------------

    def _host_save(self, source: torch.Tensor, payload: torch.Tensor, scale):
        if self._fp8:
            fp8_quantize(source, payload, scale)
        else:
            payload.copy_(source)

    def _host_restore(self, entry: _CPUBlock, target: torch.Tensor):
        if self._fp8:
            fp8_dequantize(entry.kv, entry.scale, target)
        else:
            target.copy_(entry.kv)

    # -- engine API -------------------------------------------------------------

    @torch.inference_mode()
    def measure_restore_s_per_block(self, repeats: int = 8, batch: int = 1) -> float:
        """Seconds per block of this cache's restore path (H2D, plus FP8 dequant).

        batch > 1 times restores issued `batch` blocks per call (as _copy_entries
        does for a run of CPU hits), so hybrid admission can use the per-block
        cost at the batch size it actually restores; batch=1 is the per-block
        call of _copy_entry.
        """
        self._require_open()
        if not self._on_cuda:
            raise RuntimeError("restore timing needs a CUDA KV pool")
        if repeats < 1 or batch < 1:
            raise ValueError("repeats and batch must be positive")
        from kvoff.slab import PinnedSlab

        pool = self._cache
        scratch_pool = torch.empty((2, pool.shape[1], batch, *pool.shape[3:]), dtype=pool.dtype,
                                   device=pool.device)
        n = repeats * batch
        scale_offset = -(-n * self._payload_bytes // 256) * 256
        slab = PinnedSlab(scale_offset + n * self._scale_bytes, device=pool.device.index)
        payload = slab.view(0, (n, self._payload_bytes), torch.uint8)
        payload.zero_()
        scale = None
        if self._fp8:
            scale = slab.view(scale_offset, (n, self._scale_bytes // 2), pool.dtype)
            scale.fill_(1.0)

        def pointers(rows, alias):
            ptr = slab.device_alias if alias else (lambda t: t.data_ptr())
            return ([ptr(payload[i]) for i in rows],
                    [ptr(scale[i]) if scale is not None else 0 for i in rows])

        calls = [range(r * batch, (r + 1) * batch) for r in range(repeats)]
        args = [(pointers(rows, False), pointers(rows, True)) for rows in calls]
        targets = list(range(batch))
        stream = self._restore_stream
        stream.wait_stream(torch.cuda.current_stream(pool.device))
        for _ in range(2):  # the first pass warms up kernels and clocks
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                start.record(stream)
                for plain, mapped in args:
                    self._device_restore(scratch_pool, targets, plain, mapped, stream)
                end.record(stream)
            end.synchronize()
        return start.elapsed_time(end) / 1000 / n

    def synchronize(self):
        """Wait for every pending host<->device copy (needed before host reads)."""
        for stream in {self._copy_stream, self._restore_stream} - {None}:
            self._ops.join_pipeline(self._cache.device, stream)
            stream.synchronize()
        self._rpc("synchronize")

    @torch.inference_mode()
    def save_block(self, prefix_hash: int) -> bool:
        """Save a published full block; False if it is already saved.

        A full budget raises CPUCacheFullError before any allocation. A failed
        copy leaves CPU entries and GPU metadata unchanged. Partial tail blocks
        cannot be saved.
        """
        self._require_open()
        entry = self._entries.get(prefix_hash)
        block_id = self._manager.hash_to_block_id.get(prefix_hash)
        if block_id is None:
            if entry is not None:
                return False
            raise KeyError(f"GPU prefix block {prefix_hash} is not cached")
        block = self._manager.blocks[block_id]
        tokens = tuple(block.token_ids)
        if block.hash != prefix_hash or len(tokens) != self._manager.block_size:
            raise ValueError("source must be a published full prefix block")
        if entry is not None:
            if entry.token_ids != tokens:
                raise ValueError("prefix hash has conflicting token metadata")
            return False
        if self.bytes_used + self._block_bytes > self._max_bytes:
            raise CPUCacheFullError("CPU prefix cache payload budget exceeded")
        if not self._free_slots:
            self._grow()
        slot = self._free_slots.pop()
        done = None
        try:
            payload, scale = self._slot_view(slot)
            if self._on_cuda:
                done = self._save_on_device([block_id], [slot])
            else:
                self._host_save(self._cache[:, :, block_id], payload, scale)
        except BaseException:
            self._free_slots.append(slot)
            raise
        self._entries[prefix_hash] = _CPUBlock(tokens, payload, slot, scale, done)
        self._saved_blocks += 1
        return True

    @torch.inference_mode()
    def save_blocks(self, prefix_hashes) -> list[bool]:
        """Save several published full blocks with one copy call; True per new save.

        Each hash follows save_block's rules (KeyError, ValueError, False when
        already saved). The batch is checked in full - keys, metadata, budget -
        before any slot is taken, and a failed copy saves none of it. On CUDA
        the blocks move in one native call and share one completion event,
        instead of one launch, one DMA pair and one event per block.
        """
        self._require_open()
        todo, results, seen = [], [], set()
        for prefix_hash in prefix_hashes:
            entry = self._entries.get(prefix_hash)
            block_id = self._manager.hash_to_block_id.get(prefix_hash)
            if block_id is None:
                if entry is not None:
                    results.append(False)
                    continue
                raise KeyError(f"GPU prefix block {prefix_hash} is not cached")
            block = self._manager.blocks[block_id]
            tokens = tuple(block.token_ids)
            if block.hash != prefix_hash or len(tokens) != self._manager.block_size:
                raise ValueError("source must be a published full prefix block")
            if entry is not None and entry.token_ids != tokens:
                raise ValueError("prefix hash has conflicting token metadata")
            new = entry is None and prefix_hash not in seen
            results.append(new)
            if new:
                seen.add(prefix_hash)
                todo.append((prefix_hash, block_id, tokens))
        if not todo:
            return results
        if self.bytes_used + len(todo) * self._block_bytes > self._max_bytes:
            raise CPUCacheFullError("CPU prefix cache payload budget exceeded")
        while len(self._free_slots) < len(todo) and self._num_slots < self._capacity:
            self._grow()
        slots = [self._free_slots.pop() for _ in todo]
        done = None
        try:
            if self._on_cuda:
                done = self._save_on_device([b for _, b, _ in todo], slots)
            else:
                for (_, block_id, _), slot in zip(todo, slots):
                    payload, scale = self._slot_view(slot)
                    self._host_save(self._cache[:, :, block_id], payload, scale)
        except BaseException:
            self._free_slots.extend(reversed(slots))
            raise
        for (prefix_hash, _, tokens), slot in zip(todo, slots):
            payload, scale = self._slot_view(slot)
            self._entries[prefix_hash] = _CPUBlock(tokens, payload, slot, scale, done)
        self._saved_blocks += len(todo)
        return results

    def _save_on_device(self, block_ids, slots) -> torch.cuda.Event:
        """Enqueue the save of pool blocks into slots; returns the slots-filled event.

        The copies follow the kernels that wrote the blocks and, with split
        streams, earlier restores that read these slots. before_block_reuse
        orders each block's next writer after the point where the save has read
        it: for a staged save that is the quantize or gather kernel (the
        library records `read` after it, while the copies to host still
        drain); otherwise the returned event.
        """
        pool = self._cache
        current = torch.cuda.current_stream(pool.device)
        copy = self._copy_stream
        staged = self._modes["fp8_save" if self._fp8 else "bf16_save"] == "staged"
        waits = read = None
        if staged:
            # The kernels wait only for the blocks' writers (and restores still
            # filling them), not for earlier saves' copies on the copy stream.
            # One event serves every call: a wait takes its latest record.
            ready = self._ready
            ready.record(current)
            waits = [ready]
            for block_id in dict.fromkeys(block_ids):
                restoring = self._pending_restores.get(block_id)
                if restoring is not None:
                    waits.append(restoring)
            read = torch.cuda.Event()
            read.record(copy)  # creates the CUDA event; the library re-records it
        else:
            copy.wait_stream(current)
        for slot in slots:
            slot_read = self._slot_reads.pop(slot, None)
            if slot_read is not None and self._restore_stream is not copy:
                copy.wait_event(slot_read)
        self._device_save(pool, list(block_ids), list(slots), copy, waits, read)
        done = torch.cuda.Event()
        done.record(copy)
        for block_id in block_ids:
            self._pending_saves[block_id] = read if read is not None else done
        self._rpc("save", list(block_ids), list(slots))
        return done

    def _preserve(self, prefix_hash: int):
        # Only a full budget is an expected, silent skip; device and copy
        # errors propagate.
        try:
            self.save_block(prefix_hash)
        except CPUCacheFullError:
            self._budget_skips += 1

    def _preserve_before_recycle(self, prefix_hash: int):
        self._preserve(prefix_hash)

    def _preserve_on_release(self, prefix_hash: int):
        # Save eagerly only while a request waits for blocks; otherwise the
        # block likely stays a GPU hit and the D2H traffic would only delay
        # small per-step copies.
        if self._save_on_release and self._manager.admission_blocked:
            self._preserve(prefix_hash)

    def before_block_reuse(self, block_id: int):
        """Order later writes of a GPU block after its pending copies (no host sync)."""
        waited = False
        for pending in (self._pending_saves, self._pending_restores):
            done = pending.pop(block_id, None)
            if done is not None:
                torch.cuda.current_stream(self._cache.device).wait_event(done)
                waited = True
        if waited:  # the other ranks hold the same pending copies
            self._rpc("before_reuse", [block_id])

    def before_block_use(self, block_id: int):
        """Order later reads of a prefetched GPU block after its restore."""
        done = self._pending_restores.pop(block_id, None)
        if done is not None:
            torch.cuda.current_stream(self._cache.device).wait_event(done)
            self._rpc("before_use", [block_id])

    def _entry_for(self, prefix_hash: int, token_ids):
        """Pure lookup for admission planning; entries stay valid during copies."""
        entry = self._entries.get(prefix_hash)
        if entry is None or entry.token_ids != tuple(token_ids):
            return None
        return entry

    @torch.inference_mode()
    def _copy_entry(self, entry: _CPUBlock, block_id: int, wait: bool = True):
        self._require_open()
        if not self._on_cuda:
            self._host_restore(entry, self._cache[:, :, block_id])
            self._restored_blocks += 1
            return
        pool = self._cache
        current = torch.cuda.current_stream(pool.device)
        stream = self._restore_stream
        # The target may still be read by queued kernels, and the slot may
        # still be filling from its own save.
        stream.wait_stream(current)
        if entry.saved is not None and stream is not self._copy_stream:
            stream.wait_event(entry.saved)
        done = self._restore_slots([entry.slot], [block_id], stream)
        self._slot_reads[entry.slot] = done
        if wait:
            current.wait_event(done)
        else:
            self._pending_restores[block_id] = done
        self._rpc("restore", [entry.slot], [block_id], wait)
        self._restored_blocks += 1

    @torch.inference_mode()
    def _copy_entries(self, entries, block_ids, wait: bool = True):
        """_copy_entry for several entries with one copy call and one event.

        For callers that restore a run of blocks at once (an admission's CPU
        hits, a prefetch): the same ordering as _copy_entry per block, with the
        copies issued as one native call on the restore stream.
        """
        self._require_open()
        entries, block_ids = list(entries), list(block_ids)
        if len(entries) != len(block_ids):
            raise ValueError("one target block per entry")
        if not entries:
            return
        if not self._on_cuda:
            for entry, block_id in zip(entries, block_ids):
                self._host_restore(entry, self._cache[:, :, block_id])
            self._restored_blocks += len(entries)
            return
        pool = self._cache
        current = torch.cuda.current_stream(pool.device)
        stream = self._restore_stream
        stream.wait_stream(current)
        if stream is not self._copy_stream:
            waited = set()
            for entry in entries:
                if entry.saved is not None and id(entry.saved) not in waited:
                    waited.add(id(entry.saved))
                    stream.wait_event(entry.saved)
        done = self._restore_slots([e.slot for e in entries], block_ids, stream)
        for entry in entries:
            self._slot_reads[entry.slot] = done
        if wait:
            current.wait_event(done)
        else:
            for block_id in block_ids:
                self._pending_restores[block_id] = done
        self._rpc("restore", [e.slot for e in entries], block_ids, wait)
        self._restored_blocks += len(entries)

    @torch.inference_mode()
    def restore_block(self, prefix_hash: int) -> int:
        """Restore a CPU hit; return the GPU block it now occupies.

        GPU hits are reused without a copy. On copy failure the destination is
        freed and the hash stays unpublished; the CPU entry remains for retry.
        """
        self._require_open()
        entry = self._entries[prefix_hash]
        return self._manager.restore_cached_block(
            prefix_hash, entry.token_ids, lambda block_id: self._copy_entry(entry, block_id))

    def discard(self, prefix_hash: int) -> bool:
        """Release one CPU payload without changing GPU cache state."""
        self._require_open()
        entry = self._entries.pop(prefix_hash, None)
        if entry is None:
            return False
        # A later save into the slot is ordered after a pending restore of it
        # by the slot-read event (split streams) or by stream order.
        self._free_slots.append(entry.slot)
        return True

    def clear(self):
        self._free_slots.extend(entry.slot for entry in self._entries.values())
        self._entries.clear()

    def close(self):
        """Release payloads and pool references; idempotent."""
        if self.closed:
            return
        if self.automatic:
            self._manager._cpu_prefix_cache = None
        self.synchronize()
        self._rpc("close")
        self._tp_runner = None
        self.clear()
        for table in (self._pending_saves, self._pending_restores, self._slot_reads,
                      self._slot_saved, self._staging):
            table.clear()
        self._slabs.clear()
        self._scale_slabs.clear()
        self._slab_owners.clear()
        self._free_slots.clear()
        self._num_slots = 0
        self._cache = None
        self._manager = None
