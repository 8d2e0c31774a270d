"""The C ABI library loads on a CPU-only host and exports every declared entry.

No test here launches GPU work: argument validation and fault injection run
before any CUDA call, so they are host logic.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from kvoff import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "kvoff.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"KVOFF_API\s+[\w\s\*]*?\b(kvoff_\w+)\s*\(", text)


def test_header_declares_the_hot_path_entry_points():
    names = set(declared())
    for required in ("kvoff_fp8_save_blocks", "kvoff_fp8_restore_blocks",
                     "kvoff_fp8_save_blocks_staged", "kvoff_fp8_restore_blocks_staged",
                     "kvoff_copy_blocks", "kvoff_store_kvcache", "kvoff_host_alloc",
                     "kvoff_host_free", "kvoff_last_error", "kvoff_debug_fail_next"):
        assert required in names


def test_library_exports_every_declared_symbol():
    so = ctypes.CDLL(str(_lib.LIBRARY))
    names = declared()
    assert names
    for name in names:
        assert hasattr(so, name), name
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes binding"
    assert set(_lib.SIGNATURES) == set(names)


def test_abi_version_and_error_text():
    so = _lib.lib()
    assert so.kvoff_abi_version() == _lib.ABI_VERSION
    rc = so.kvoff_copy_blocks(None, 1, 0, 0, 1, 16, None, 1, None, 7, 0, 0, None)
    assert rc == _lib.KVOFF_EINVAL
    assert "direction" in _lib.last_error()


def test_fault_injection_fires_once_before_any_device_work():
    so = _lib.lib()
    _lib.debug_fail_next("memcpy", 1)
    assert so.kvoff_memcpy(None, None, 0, None) == _lib.KVOFF_EINJECTED
    assert "injected" in _lib.last_error()
    assert so.kvoff_memcpy(None, None, 0, None) == _lib.KVOFF_OK  # disarmed
    _lib.debug_fail_next("fp8_save_blocks", 2)
    _lib.debug_fail_next("fp8_save_blocks", 0)  # cleared
    ids = _lib.int64_array([0])
    assert so.kvoff_fp8_save_blocks(None, 2, 0, 0, 1, 1, 1, ids, -1, None, None, 0,
                                    None) == _lib.KVOFF_EINVAL
    with pytest.raises(_lib.KvoffError, match="empty op"):
        _lib.call("kvoff_debug_fail_next", b"", 1)


@pytest.mark.parametrize("block_id", [-1, 4])
def test_block_ids_are_range_checked_on_the_host(block_id):
    so = _lib.lib()
    ids = _lib.int64_array([block_id])
    slots = _lib.pointer_array([16])
    rc = so.kvoff_fp8_restore_blocks(ctypes.c_void_p(256), 4, 4096, 1024, 4, 8, 128, ids, 1,
                                     slots, slots, 0, None)
    assert rc == _lib.KVOFF_EINVAL and "out of range" in _lib.last_error()
    rc = so.kvoff_copy_blocks(ctypes.c_void_p(256), 4, 4096, 1024, 4, 1024, ids, 1, slots, 0, 0,
                              0, None)
    assert rc == _lib.KVOFF_EINVAL and "out of range" in _lib.last_error()


def test_store_kvcache_rejects_bad_sizes_and_skips_empty_batches():
    so = _lib.lib()
    assert so.kvoff_store_kvcache(None, 0, None, 0, None, None, 0, None, 1, 1, None,
                                  None) == _lib.KVOFF_EINVAL
    assert so.kvoff_store_kvcache(None, 0, None, 0, None, None, 16, None, 0, 1, None,
                                  None) == _lib.KVOFF_OK


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIBRARY", tmp_path / "libkvoff.so")
    with pytest.raises(RuntimeError, match="not built"):
        _lib.lib()


def test_event_ordered_entry_points_check_their_arguments_on_the_host():
    so = _lib.lib()
    ids = _lib.int64_array([0])
    slots = _lib.pointer_array([16])
    # A wait-event count with no list is rejected before any device work.
    rc = so.kvoff_fp8_save_blocks_staged_ev(ctypes.c_void_p(256), 4, 4096, 1024, 4, 8, 128, ids,
                                            1, slots, slots, ctypes.c_void_p(512),
                                            ctypes.c_void_p(512), 2, None, 1, None, None)
    assert rc == _lib.KVOFF_EINVAL and "wait event" in _lib.last_error()
    rc = so.kvoff_fp8_save_blocks_staged_ev(ctypes.c_void_p(256), 4, 4096, 1024, 4, 8, 128, ids,
                                            1, slots, slots, ctypes.c_void_p(512),
                                            ctypes.c_void_p(512), 2, None, -1, None, None)
    assert rc == _lib.KVOFF_EINVAL
    # Empty batches are a no-op; out-of-range ids fail like the plain staged calls.
    assert so.kvoff_fp8_restore_blocks_staged_ev(ctypes.c_void_p(256), 4, 4096, 1024, 4, 8, 128,
                                                 ids, 0, slots, slots, None, None, 2, None,
                                                 None) == _lib.KVOFF_OK
    bad = _lib.int64_array([9])
    rc = so.kvoff_fp8_restore_blocks_staged_ev(ctypes.c_void_p(256), 4, 4096, 1024, 4, 8, 128,
                                               bad, 1, slots, slots, ctypes.c_void_p(512),
                                               ctypes.c_void_p(512), 2, None, None)
    assert rc == _lib.KVOFF_EINVAL and "out of range" in _lib.last_error()


def test_staged_block_copies_check_their_arguments_on_the_host():
    so = _lib.lib()
    ids = _lib.int64_array([0])
    slots = _lib.pointer_array([16])
    geom = (ctypes.c_void_p(256), 4, 4096, 1024, 4, 1024)
    # Bad direction, wait events on a restore, and a null staging buffer are
    # rejected before any device work; an empty batch is a no-op.
    rc = so.kvoff_copy_blocks_staged(*geom, ids, 1, slots, ctypes.c_void_p(512), 2, 7, None, 0,
                                     None, None)
    assert rc == _lib.KVOFF_EINVAL and "direction" in _lib.last_error()
    rc = so.kvoff_copy_blocks_staged(*geom, ids, 1, slots, ctypes.c_void_p(512), 2, _lib.RESTORE,
                                     slots, 1, None, None)
    assert rc == _lib.KVOFF_EINVAL and "wait event" in _lib.last_error()
    rc = so.kvoff_copy_blocks_staged(*geom, ids, 1, slots, None, 2, _lib.SAVE, None, 0, None,
                                     None)
    assert rc == _lib.KVOFF_EINVAL and "staging" in _lib.last_error()
    assert so.kvoff_copy_blocks_staged(*geom, ids, 0, slots, None, 2, _lib.SAVE, None, 0, None,
                                       None) == _lib.KVOFF_OK
    bad = _lib.int64_array([4])
    rc = so.kvoff_copy_blocks_staged(*geom, bad, 1, slots, ctypes.c_void_p(512), 2, _lib.SAVE,
                                     None, 0, None, None)
    assert rc == _lib.KVOFF_EINVAL and "out of range" in _lib.last_error()


def test_ops_rejects_events_that_were_never_recorded():
    from kvoff import ops

    with pytest.raises(ValueError, match="recorded"):
        ops._event(0)
    assert ops._event(1234) == 1234


def test_bounded_wait_hook_rejects_limits_outside_its_range():
    so = _lib.lib()
    assert so.kvoff_debug_bounded_wait(0, None) == _lib.KVOFF_EINVAL
    assert so.kvoff_debug_bounded_wait(3_000_000_000, None) == _lib.KVOFF_EINVAL
    assert "limit" in _lib.last_error()
