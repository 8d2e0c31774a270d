"""ctypes binding of libkvoff.so (the C ABI declared in include/kvoff.h).

The library is loaded from this package directory. There is no fallback: if
it is missing or stale, every call raises, so a CUDA pool can never silently
run on another code path.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY = Path(__file__).resolve().with_name("libkvoff.so")
ABI_VERSION = 1

KVOFF_OK, KVOFF_EINVAL, KVOFF_ECUDA, KVOFF_EINJECTED, KVOFF_ENOMEM, KVOFF_EDEVICE = range(6)
SAVE, RESTORE = 0, 1
COPY_ENGINE, COPY_TMA, COPY_SM = 0, 1, 2

_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_PI64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); must match include/kvoff.h.
SIGNATURES = {
    "kvoff_abi_version": (_I32, []),
    "kvoff_last_error": (ctypes.c_char_p, []),
    "kvoff_debug_fail_next": (ctypes.c_int, [ctypes.c_char_p, _I32]),
    "kvoff_device_error": (ctypes.c_int, [_I32, ctypes.POINTER(_I32), _I32]),
    "kvoff_fp8_save_blocks": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _PI64, _I64,
                                             _PP, _PP, _I32, _P]),
    "kvoff_fp8_restore_blocks": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _PI64,
                                                _I64, _PP, _PP, _I32, _P]),
    "kvoff_fp8_save_blocks_staged": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _PI64,
                                                    _I64, _PP, _PP, _P, _P, _I64, _P]),
    "kvoff_fp8_save_blocks_staged_noalloc": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64,
                                                            _I64, _PI64, _I64, _PP, _PP, _P]),
    "kvoff_fp8_restore_blocks_staged": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64,
                                                       _PI64, _I64, _PP, _PP, _P, _P, _I64, _P]),
    "kvoff_fp8_save_blocks_staged_ev": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64,
                                                       _PI64, _I64, _PP, _PP, _P, _P, _I64, _PP,
                                                       _I32, _P, _P]),
    "kvoff_fp8_restore_blocks_staged_ev": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64,
                                                          _PI64, _I64, _PP, _PP, _P, _P, _I64, _P,
                                                          _P]),
    "kvoff_stream_join_pipeline": (ctypes.c_int, [_P]),
    "kvoff_debug_bounded_wait": (ctypes.c_int, [_I64, _P]),
    "kvoff_copy_blocks": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _PI64, _I64, _PP, _I32,
                                         _I32, _I32, _P]),
    "kvoff_copy_blocks_staged": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _PI64, _I64,
                                                _PP, _P, _I64, _I32, _PP, _I32, _P, _P]),
    "kvoff_copy_tokens": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _PI64, _I64, _P,
                                         _I32, _P]),
    "kvoff_store_kvcache": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I64, _I64, _P,
                                           _P]),
    "kvoff_host_alloc": (ctypes.c_int, [ctypes.c_uint64, _I32, _PP, _PP]),
    "kvoff_host_free": (ctypes.c_int, [_P]),
    "kvoff_device_numa_node": (ctypes.c_int, [_I32, ctypes.POINTER(_I32)]),
    "kvoff_memcpy": (ctypes.c_int, [_P, _P, ctypes.c_uint64, _P]),
}


class KvoffError(RuntimeError):
    """A libkvoff call failed; `status` is its kvoff_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise RuntimeError(
                    f"{LIBRARY.name} is not built; run `python -m kvoff.build` or "
                    "__graft_entry__.build() (the CUDA path has no fallback)")
            so = ctypes.CDLL(str(LIBRARY))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(so, name)
                fn.restype, fn.argtypes = restype, argtypes
            version = so.kvoff_abi_version()
            if version != ABI_VERSION:
                raise RuntimeError(f"{LIBRARY} has ABI {version}, expected {ABI_VERSION}")
            _lib = so
    return _lib


def last_error() -> str:
    return lib().kvoff_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != KVOFF_OK:
        raise KvoffError(status, f"{what}: {last_error()}")


def call(name: str, *args) -> None:
    """Call entry point `name` and raise KvoffError on a non-zero status."""
    check(getattr(lib(), name)(*args), name)


def int64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(values)))(*values)


def pointer_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_void_p * max(1, len(values)))(*values)


def debug_fail_next(op: str, count: int = 1) -> None:
    """Make the next `count` calls of entry point `op` fail (test hook)."""
    call("kvoff_debug_fail_next", op.encode(), count)


def device_error(device: int, clear: bool = True) -> int:
    """Device-side error flags of bounded waits on `device` (synchronizes it)."""
    flags = _I32(0)
    call("kvoff_device_error", device, ctypes.byref(flags), 1 if clear else 0)
    return flags.value
