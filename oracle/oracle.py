"""numpy front end of the C oracle (oracle/kvoff_oracle.c) - TEST INFRASTRUCTURE.

Arrays of bf16 values are carried as uint16 bit patterns and FP8 payloads as
uint8, so every comparison against the CUDA library is a bit comparison.
Layouts follow the reference (nanovllm/engine/cpu_prefix_cache.py:94-100):
pool [2, L, NB, BS, H, D], slot [2, L, BS, H, D], scales [2, L, BS, H, 1].
"""

from __future__ import annotations

import ctypes

import numpy as np

from oracle.build import build

__all__ = [
    "lib", "set_threads", "max_threads", "f32_to_bf16_bits", "bf16_bits_to_f32",
    "fp8_quantize_rows", "fp8_dequantize_rows", "fp8_save_blocks", "fp8_restore_blocks",
    "copy_blocks", "store_kvcache", "e4m3_from_f32", "bf16_from_f32", "e4m3_value",
]

_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int64


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        so = ctypes.CDLL(str(build()))
        so.kvo_set_threads.argtypes = [ctypes.c_int]
        so.kvo_max_threads.restype = ctypes.c_int
        so.kvo_bf16_from_f32.argtypes = [ctypes.c_float]
        so.kvo_bf16_from_f32.restype = ctypes.c_uint16
        so.kvo_e4m3_from_f32.argtypes = [ctypes.c_float]
        so.kvo_e4m3_from_f32.restype = ctypes.c_uint8
        so.kvo_e4m3_value.argtypes = [ctypes.c_uint8]
        so.kvo_e4m3_value.restype = ctypes.c_float
        so.kvo_fp8_quantize_rows.argtypes = [_P, _I, _I, _I, _P, _P]
        so.kvo_fp8_dequantize_rows.argtypes = [_P, _P, _I, _I, _P, _I]
        so.kvo_fp8_save_blocks.argtypes = [_P, _I, _I, _I, _I, _I, _P, _I, _P, _P]
        so.kvo_fp8_restore_blocks.argtypes = [_P, _I, _I, _I, _I, _I, _P, _I, _P, _P]
        so.kvo_fp8_save_blocks_fast.argtypes = [_P, _I, _I, _I, _I, _I, _P, _I, _P, _P]
        so.kvo_fp8_restore_blocks_fast.argtypes = [_P, _I, _I, _I, _I, _I, _P, _I, _P, _P]
        so.kvo_copy_blocks.argtypes = [_P, _I, _I, _I, _I, _P, _I, _P, ctypes.c_int]
        so.kvo_store_kvcache.argtypes = [_P, _I, _P, _I, _P, _P, _I, _P, _I, _I]
        _lib = so
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().kvo_set_threads(int(n))


def max_threads() -> int:
    return int(lib().kvo_max_threads())


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_from_f32(x: float) -> int:
    return int(lib().kvo_bf16_from_f32(x))


def e4m3_from_f32(x: float) -> int:
    return int(lib().kvo_e4m3_from_f32(x))


def e4m3_value(v: int) -> float:
    return float(lib().kvo_e4m3_value(v))


def fp8_quantize_rows(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Reference fp8_quantize on the last dim: bf16 bits [..., D] -> (payload, scale)."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    d = x.shape[-1]
    rows = x.size // d if d else 0
    payload = np.empty(x.shape, dtype=np.uint8)
    scale = np.empty((*x.shape[:-1], 1), dtype=np.uint16)
    lib().kvo_fp8_quantize_rows(_ptr(x), rows, d, d, _ptr(payload), _ptr(scale))
    return payload, scale


def fp8_dequantize_rows(payload: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Reference fp8_dequantize: (payload [..., D], scale [..., 1]) -> bf16 bits."""
    p = np.ascontiguousarray(payload, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    d = p.shape[-1]
    rows = p.size // d if d else 0
    out = np.empty(p.shape, dtype=np.uint16)
    lib().kvo_fp8_dequantize_rows(_ptr(p), _ptr(s), rows, d, _ptr(out), d)
    return out


def _geometry(pool: np.ndarray) -> tuple[int, int, int, int, int]:
    """(num_chunks, chunk_stride, block_stride, rows_per_chunk, D) in elements."""
    if pool.ndim != 6 or pool.shape[0] != 2 or not pool.flags.c_contiguous:
        raise ValueError("pool must be a contiguous [2, L, NB, BS, H, D] array")
    _, layers, nb, bs, h, d = pool.shape
    return 2 * layers, nb * bs * h * d, bs * h * d, bs * h, d


def fp8_save_blocks(pool: np.ndarray, ids, fast: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """Quantize pool[:, :, id] for each id -> payload [n, 2, L, BS, H, D], scale [n, ..., 1].

    fast=True runs the single-pass port (same bits) used as the timed CPU baseline.
    """
    pool = np.asarray(pool)
    chunks, cs, bst, rpc, d = _geometry(pool)
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    _, layers, _, bs, h, _ = pool.shape
    payload = np.empty((len(ids), 2, layers, bs, h, d), dtype=np.uint8)
    scale = np.empty((len(ids), 2, layers, bs, h, 1), dtype=np.uint16)
    fn = lib().kvo_fp8_save_blocks_fast if fast else lib().kvo_fp8_save_blocks
    fn(_ptr(pool.view(np.uint16)), chunks, cs, bst, rpc, d, _ptr(ids), len(ids), _ptr(payload),
       _ptr(scale))
    return payload, scale


def fp8_restore_blocks(pool: np.ndarray, ids, payload: np.ndarray, scale: np.ndarray,
                       fast: bool = False) -> None:
    """Dequantize slot i into pool[:, :, ids[i]] in place (fast=True: the timed port)."""
    chunks, cs, bst, rpc, d = _geometry(pool)
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    p = np.ascontiguousarray(payload, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint16)
    if p.shape[0] != len(ids) or s.shape[0] != len(ids):
        raise ValueError("one payload and scale slot per block id")
    fn = lib().kvo_fp8_restore_blocks_fast if fast else lib().kvo_fp8_restore_blocks
    fn(_ptr(pool.view(np.uint16)), chunks, cs, bst, rpc, d, _ptr(ids), len(ids), _ptr(p), _ptr(s))


def copy_blocks(pool: np.ndarray, ids, slots: np.ndarray | None = None, restore: bool = False):
    """Byte moves of whole blocks: pool -> new slots (save) or slots -> pool (restore)."""
    if pool.ndim != 6 or pool.shape[0] != 2 or not pool.flags.c_contiguous:
        raise ValueError("pool must be a contiguous [2, L, NB, ...] array")
    _, layers, nb = pool.shape[:3]
    item = pool.itemsize
    chunk_bytes = int(np.prod(pool.shape[3:])) * item
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    if slots is None:
        slots = np.empty((len(ids), 2, layers, *pool.shape[3:]), dtype=pool.dtype)
    slots = np.ascontiguousarray(slots)
    lib().kvo_copy_blocks(_ptr(pool), 2 * layers, nb * chunk_bytes, chunk_bytes, chunk_bytes,
                          _ptr(ids), len(ids), _ptr(slots), 1 if restore else 0)
    return slots


def store_kvcache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                  slot_mapping: np.ndarray) -> None:
    """attention.store_kvcache restated: row i of key/value -> cache row slot_mapping[i]."""
    n, h, d = key.shape
    item = key.itemsize
    for t in (key, value):
        if t.strides[2] != item or t.strides[1] != d * item:
            raise ValueError("key/value rows must be [H, D] contiguous")
    if not (k_cache.flags.c_contiguous and v_cache.flags.c_contiguous):
        raise ValueError("caches must be contiguous")
    slots = np.ascontiguousarray(slot_mapping, dtype=np.int32)
    if slots.shape != (n,):
        raise ValueError("one slot per token")
    row = h * d * item
    lib().kvo_store_kvcache(key.ctypes.data, key.strides[0], value.ctypes.data, value.strides[0],
                            _ptr(k_cache), _ptr(v_cache), row, _ptr(slots), n,
                            k_cache.size * item // row)
