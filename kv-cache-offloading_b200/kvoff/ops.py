"""Tensor-level wrappers over the libkvoff C ABI.

Every function enqueues work on a CUDA stream (default: the current stream of
the pool's device) and never synchronizes the host. Slots are addressed by raw
pointers so that one call can target pinned host slabs, their device aliases
(zero-copy) or device staging buffers.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from kvoff import _lib
from kvoff._lib import COPY_ENGINE, COPY_SM, COPY_TMA  # noqa: F401  (re-exported)


@dataclass(frozen=True)
class PoolGeometry:
    """Geometry of a paged pool [2, L, NB, BS, H, D] (strides in elements).

    Chunk c = kv * L + layer of block b starts at c * chunk_stride +
    b * block_stride and holds rows_per_chunk = BS * H dense rows of D.
    """

    num_chunks: int
    chunk_stride: int
    block_stride: int
    num_blocks: int
    rows_per_chunk: int
    head_dim: int
    elem_size: int

    @property
    def rows(self) -> int:
        return self.num_chunks * self.rows_per_chunk

    @property
    def chunk_bytes(self) -> int:
        return self.rows_per_chunk * self.head_dim * self.elem_size

    @property
    def block_bytes(self) -> int:
        """Raw (BF16-mode) bytes of one block."""
        return self.num_chunks * self.chunk_bytes

    @property
    def fp8_payload_bytes(self) -> int:
        return self.rows * self.head_dim

    @property
    def fp8_scale_bytes(self) -> int:
        return self.rows * 2


def geometry(pool: torch.Tensor) -> PoolGeometry:
    """Validate a pool's layout and return its geometry."""
    if pool.ndim != 6 or pool.shape[0] != 2 or min(pool.shape) <= 0:
        raise ValueError("KV pool must be a non-empty [2, L, NB, BS, H, D] tensor")
    _, layers, num_blocks, block_size, heads, dim = pool.shape
    s = pool.stride()
    if s[5] != 1 or s[4] != dim or s[3] != heads * dim:
        raise ValueError("each KV block chunk [BS, H, D] must be dense")
    if layers > 1 and s[0] != layers * s[1]:
        raise ValueError("(K/V, layer) chunks of the pool must be evenly strided")
    chunk_stride = s[1] if layers > 1 else s[0]
    return PoolGeometry(2 * layers, chunk_stride, s[2], num_blocks, block_size * heads, dim,
                        pool.element_size())


def _stream(device: torch.device, stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream(device)
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor")


def _require_bf16(pool: torch.Tensor) -> None:
    if pool.dtype != torch.bfloat16:
        raise ValueError("the FP8 codec quantizes bf16 KV pools")


def save_fp8(pool: torch.Tensor, block_ids, payload_ptrs, scale_ptrs, *, stream=None,
             max_ctas: int = 0) -> None:
    """Quantize blocks into device-accessible slots (device staging or mapped host)."""
    _require_cuda(pool, "pool")
    _require_bf16(pool)
    g = geometry(pool)
    n = len(block_ids)
    if len(payload_ptrs) != n or len(scale_ptrs) != n:
        raise ValueError("one payload and scale pointer per block")
    with torch.cuda.device(pool.device):
        _lib.call("kvoff_fp8_save_blocks", pool.data_ptr(), g.num_chunks, g.chunk_stride,
                  g.block_stride, g.num_blocks, g.rows_per_chunk, g.head_dim,
                  _lib.int64_array(block_ids), n, _lib.pointer_array(payload_ptrs),
                  _lib.pointer_array(scale_ptrs), max_ctas, _stream(pool.device, stream))


def restore_fp8(pool: torch.Tensor, block_ids, payload_ptrs, scale_ptrs, *, stream=None,
                max_ctas: int = 0) -> None:
    """Dequantize device-accessible slots into pool blocks."""
    _require_cuda(pool, "pool")
    _require_bf16(pool)
    g = geometry(pool)
    n = len(block_ids)
    if len(payload_ptrs) != n or len(scale_ptrs) != n:
        raise ValueError("one payload and scale pointer per block")
    with torch.cuda.device(pool.device):
        _lib.call("kvoff_fp8_restore_blocks", pool.data_ptr(), g.num_chunks, g.chunk_stride,
                  g.block_stride, g.num_blocks, g.rows_per_chunk, g.head_dim,
                  _lib.int64_array(block_ids), n, _lib.pointer_array(payload_ptrs),
                  _lib.pointer_array(scale_ptrs), max_ctas, _stream(pool.device, stream))


def _staging_blocks(g: PoolGeometry, staging_payload: torch.Tensor,
                    staging_scale: torch.Tensor) -> int:
    _require_cuda(staging_payload, "staging payload")
    _require_cuda(staging_scale, "staging scale")
    count = min(staging_payload.numel() * staging_payload.element_size() // g.fp8_payload_bytes,
                staging_scale.numel() * staging_scale.element_size() // g.fp8_scale_bytes)
    if count < 1:
        raise ValueError("staging buffers hold less than one block")
    return count


def _event(event) -> int:
    """Raw cudaEvent_t of a recorded torch.cuda.Event (or a raw handle)."""
    handle = int(getattr(event, "cuda_event", event))
    if handle == 0:  # torch creates the CUDA event on its first record
        raise ValueError("pass an event that has been recorded at least once")
    return handle


def save_fp8_staged(pool: torch.Tensor, block_ids, host_payload_ptrs, host_scale_ptrs,
                    staging_payload: torch.Tensor, staging_scale: torch.Tensor, *,
                    stream=None, wait_events=None, source_done=None) -> None:
    """Quantize into device staging, then cudaMemcpyAsync each slot to pinned host.

    By default the quantize kernels follow all earlier work on `stream`. With
    `wait_events` (recorded torch.cuda.Events) they follow only those, so they
    can overlap the host copies of earlier calls; `source_done` is re-recorded
    once the kernels have read every pool block of the call.
    """
    _require_cuda(pool, "pool")
    _require_bf16(pool)
    g = geometry(pool)
    n = len(block_ids)
    if len(host_payload_ptrs) != n or len(host_scale_ptrs) != n:
        raise ValueError("one payload and scale pointer per block")
    staged = _staging_blocks(g, staging_payload, staging_scale)
    common = (pool.data_ptr(), g.num_chunks, g.chunk_stride, g.block_stride, g.num_blocks,
              g.rows_per_chunk, g.head_dim, _lib.int64_array(block_ids), n,
              _lib.pointer_array(host_payload_ptrs), _lib.pointer_array(host_scale_ptrs),
              staging_payload.data_ptr(), staging_scale.data_ptr(), staged)
    with torch.cuda.device(pool.device):
        if wait_events is None and source_done is None:
            _lib.call("kvoff_fp8_save_blocks_staged", *common, _stream(pool.device, stream))
            return
        waits = [_event(e) for e in (wait_events or ())]
        _lib.call("kvoff_fp8_save_blocks_staged_ev", *common,
                  _lib.pointer_array(waits) if waits else None, len(waits),
                  _event(source_done) if source_done is not None else None,
                  _stream(pool.device, stream))


def restore_fp8_staged(pool: torch.Tensor, block_ids, host_payload_ptrs, host_scale_ptrs,
                       staging_payload: torch.Tensor, staging_scale: torch.Tensor, *,
                       stream=None, done_event=None) -> None:
    """cudaMemcpyAsync each pinned slot into device staging, then dequantize.

    By default `stream` waits for the dequantize kernels before it returns to
    the caller's later work. With `done_event` (a recorded torch.cuda.Event)
    the event is re-recorded after the last pool write instead and `stream` is
    left free to start the next call's copies; order readers on the event, or
    call join_pipeline(stream) before synchronizing `stream`.
    """
    _require_cuda(pool, "pool")
    _require_bf16(pool)
    g = geometry(pool)
    n = len(block_ids)
    if len(host_payload_ptrs) != n or len(host_scale_ptrs) != n:
        raise ValueError("one payload and scale pointer per block")
    staged = _staging_blocks(g, staging_payload, staging_scale)
    common = (pool.data_ptr(), g.num_chunks, g.chunk_stride, g.block_stride, g.num_blocks,
              g.rows_per_chunk, g.head_dim, _lib.int64_array(block_ids), n,
              _lib.pointer_array(host_payload_ptrs), _lib.pointer_array(host_scale_ptrs),
              staging_payload.data_ptr(), staging_scale.data_ptr(), staged)
    with torch.cuda.device(pool.device):
        if done_event is None:
            _lib.call("kvoff_fp8_restore_blocks_staged", *common, _stream(pool.device, stream))
        else:
            _lib.call("kvoff_fp8_restore_blocks_staged_ev", *common, _event(done_event),
                      _stream(pool.device, stream))


def _fp8_staged_ev(save: bool, g: PoolGeometry, pool_ptr: int, block_ids, payload_ptrs,
                   scale_ptrs, staging_payload_ptr: int, staging_scale_ptr: int,
                   staging_blocks: int, stream: int, wait_events=(), event: int = 0) -> None:
    """Lean form of save_fp8_staged / restore_fp8_staged for a caller that
    already holds a checked geometry, raw pointers, raw stream and event
    handles, and has the pool's device current (the drop-in cache's per-block
    path, which runs once per saved or restored block on the engine thread).

    Save: the kernels wait for `wait_events` (none: all earlier work on the
    stream) and `event`, when non-zero, is recorded once the pool blocks are
    read. Restore: `event`, when non-zero, is recorded after the last pool
    write and the stream is not joined (see restore_fp8_staged).
    """
    so = _lib.lib()
    n = len(block_ids)
    ids = (ctypes.c_int64 * n)(*block_ids)
    payload = (ctypes.c_void_p * n)(*payload_ptrs)
    scale = (ctypes.c_void_p * n)(*scale_ptrs)
    if save:
        waits = (ctypes.c_void_p * max(1, len(wait_events)))(*wait_events)
        rc = so.kvoff_fp8_save_blocks_staged_ev(
            pool_ptr, g.num_chunks, g.chunk_stride, g.block_stride, g.num_blocks,
            g.rows_per_chunk, g.head_dim, ids, n, payload, scale, staging_payload_ptr,
            staging_scale_ptr, staging_blocks, waits, len(wait_events), event or None, stream)
        _lib.check(rc, "kvoff_fp8_save_blocks_staged_ev")
    else:
        rc = so.kvoff_fp8_restore_blocks_staged_ev(
            pool_ptr, g.num_chunks, g.chunk_stride, g.block_stride, g.num_blocks,
            g.rows_per_chunk, g.head_dim, ids, n, payload, scale, staging_payload_ptr,
            staging_scale_ptr, staging_blocks, event or None, stream)
        _lib.check(rc, "kvoff_fp8_restore_blocks_staged_ev")


def join_pipeline(device, stream=None) -> None:
    """Make `stream` wait for the staged calls' kernels queued on its behalf."""
    device = torch.device(device)
    with torch.cuda.device(device):
        _lib.call("kvoff_stream_join_pipeline", _stream(device, stream))


def copy_blocks(pool: torch.Tensor, block_ids, slot_ptrs, *, restore: bool = False,
                method: int = COPY_ENGINE, stream=None, max_ctas: int = 0) -> None:
    """Byte-exact block moves pool <-> dense slots (BF16 passthrough)."""
    _require_cuda(pool, "pool")
    g = geometry(pool)
    e = g.elem_size
    n = len(block_ids)
    if len(slot_ptrs) != n:
        raise ValueError("one slot pointer per block")
    with torch.cuda.device(pool.device):
        _lib.call("kvoff_copy_blocks", pool.data_ptr(), g.num_chunks, g.chunk_stride * e,
                  g.block_stride * e, g.num_blocks, g.chunk_bytes, _lib.int64_array(block_ids), n,
                  _lib.pointer_array(slot_ptrs), _lib.RESTORE if restore else _lib.SAVE, method,
                  max_ctas, _stream(pool.device, stream))


def copy_blocks_staged(pool: torch.Tensor, block_ids, host_slot_ptrs, staging: torch.Tensor, *,
                       restore: bool = False, stream=None, wait_events=(), event=None) -> None:
    """Byte-exact block moves pool <-> pinned host slots through device staging.

    staging is a [n, block_bytes] uint8 device buffer; with n >= 2 the gather /
    scatter kernels of one half overlap the DMA of the other (a library-owned
    kernel stream; see join_pipeline). Save: the kernels wait for wait_events
    (recorded torch.cuda.Events; none: earlier work on the stream) and `event`
    is recorded once the pool blocks are read. Restore: `event` is recorded
    after the last pool write and the stream is not joined; without it the
    stream waits for the kernels.
    """
    _require_cuda(pool, "pool")
    _require_cuda(staging, "staging")
    g = geometry(pool)
    n = len(block_ids)
    if len(host_slot_ptrs) != n:
        raise ValueError("one slot pointer per block")
    if staging.dtype != torch.uint8 or staging.dim() != 2 or staging.shape[1] != g.block_bytes:
        raise ValueError(f"staging must be uint8 [n, {g.block_bytes}]")
    if restore and wait_events:
        raise ValueError("wait_events apply to saves only")
    with torch.cuda.device(pool.device):
        _copy_staged_ev(not restore, g, pool.data_ptr(), block_ids, host_slot_ptrs,
                        staging.data_ptr(), staging.shape[0], _stream(pool.device, stream),
                        [_event(e) for e in wait_events], _event(event) if event is not None else 0)


def _copy_staged_ev(save: bool, g: PoolGeometry, pool_ptr: int, block_ids, slot_ptrs,
                    staging_ptr: int, staging_blocks: int, stream: int, wait_events=(),
                    event: int = 0) -> None:
    """Lean form of copy_blocks_staged for the drop-in cache's per-block path
    (checked geometry, raw pointers, stream and event handles, the pool's
    device current)."""
    n = len(block_ids)
    ids = (ctypes.c_int64 * n)(*block_ids)
    slots = (ctypes.c_void_p * n)(*slot_ptrs)
    waits = (ctypes.c_void_p * max(1, len(wait_events)))(*wait_events)
    e = g.elem_size
    rc = _lib.lib().kvoff_copy_blocks_staged(
        pool_ptr, g.num_chunks, g.chunk_stride * e, g.block_stride * e, g.num_blocks,
        g.chunk_bytes, ids, n, slots, staging_ptr, staging_blocks,
        _lib.SAVE if save else _lib.RESTORE, waits, len(wait_events), event or None, stream)
    _lib.check(rc, "kvoff_copy_blocks_staged")


def copy_tokens(pool: torch.Tensor, block_ids, num_tokens: int, dense_ptr: int, *,
                restore: bool = False, stream=None) -> None:
    """Tokens [0, num_tokens) of a sequence's blocks <-> dense [2, L, num_tokens, H, D]."""
    _require_cuda(pool, "pool")
    g = geometry(pool)
    block_size = pool.shape[3]
    token_bytes = pool.shape[4] * pool.shape[5] * g.elem_size
    needed = -(-num_tokens // block_size)
    if len(block_ids) < needed:
        raise ValueError("sequence is missing KV blocks")
    with torch.cuda.device(pool.device):
        _lib.call("kvoff_copy_tokens", pool.data_ptr(), g.num_chunks, g.chunk_stride * g.elem_size,
                  g.block_stride * g.elem_size, g.num_blocks, block_size, token_bytes,
                  _lib.int64_array(block_ids[:needed]), int(num_tokens), int(dense_ptr),
                  _lib.RESTORE if restore else _lib.SAVE, _stream(pool.device, stream))


def memcpy(dst_ptr: int, src_ptr: int, nbytes: int, *, device, stream=None) -> None:
    """cudaMemcpyAsync(cudaMemcpyDefault) on `stream`."""
    device = torch.device(device)
    with torch.cuda.device(device):
        _lib.call("kvoff_memcpy", int(dst_ptr), int(src_ptr), int(nbytes), _stream(device, stream))


_raw_current_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _fast_stream(device: torch.device, stream) -> int:
    """Raw handle of `stream`, or of the device's current stream (cheap path)."""
    if stream is None and _raw_current_stream is not None:
        return _raw_current_stream(device.index)
    return _stream(device, stream)


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor, *,
                  bad_slots: torch.Tensor | None = None, stream=None) -> None:
    """Write row i of key/value [N, H, D] to cache slot slot_mapping[i] (-1: skip).

    Same contract as nanovllm/layers/attention.py:33-40 (including its layout
    assertions); the scatter is one CUDA-graph-capturable kernel launch. This
    runs once per layer per forward, so the host path is kept short: one
    stride tuple per tensor, the raw current-stream handle, and a device
    switch only when the tensors live on another device than the current one.
    """
    num_tokens, num_heads, head_dim = key.shape
    row = num_heads * head_dim
    ks, vs = key.stride(), value.stride()
    if ks[2] != 1 or vs[2] != 1:
        raise AssertionError("key/value last dim must be contiguous")
    if ks[1] != head_dim or vs[1] != head_dim:
        raise AssertionError("key/value heads must be dense")
    if k_cache.stride(1) != row or v_cache.stride(1) != row:
        raise AssertionError("cache slots must hold dense [H, D] rows")
    if slot_mapping.numel() != num_tokens:
        raise AssertionError("one slot per token")
    if value.shape != key.shape:
        raise ValueError("key and value shapes differ")
    dtype = key.dtype
    if value.dtype != dtype or k_cache.dtype != dtype or v_cache.dtype != dtype:
        raise ValueError("key, value and caches must share a dtype")
    if slot_mapping.dtype != torch.int32:
        raise ValueError("slot_mapping must be int32")
    if not (key.is_cuda and value.is_cuda and k_cache.is_cuda and v_cache.is_cuda
            and slot_mapping.is_cuda):
        raise ValueError("key, value, caches and slot_mapping must be CUDA tensors")
    if bad_slots is not None and (bad_slots.dtype != torch.int32 or not bad_slots.is_cuda):
        raise ValueError("bad_slots must be a CUDA int32 tensor")
    e = key.element_size()
    num_slots = k_cache.numel() // row if row else 0
    device = key.device
    args = (key.data_ptr(), ks[0] * e, value.data_ptr(), vs[0] * e, k_cache.data_ptr(),
            v_cache.data_ptr(), row * e, slot_mapping.data_ptr(), num_tokens, num_slots,
            bad_slots.data_ptr() if bad_slots is not None else None)
    if device.index == torch.cuda.current_device():
        status = _store_fn()(*args, _fast_stream(device, stream))
    else:
        with torch.cuda.device(device):
            status = _store_fn()(*args, _fast_stream(device, stream))
    if status:
        _lib.check(status, "kvoff_store_kvcache")


_STORE = None


def _store_fn():
    global _STORE
    if _STORE is None:
        _STORE = _lib.lib().kvoff_store_kvcache
    return _STORE
