"""The device quantizer divides without a division instruction; prove it exact.

csrc/codec.cuh quant_input replaces IEEE x / s by a correctly rounded
reciprocal, one multiply and two FMAs. This checks, for every (x, scale) pair
an FP8 row can produce, that the resulting e4m3 byte equals the one IEEE
division gives (the oracle runs the check in C over all 929,598,054 pairs).
"""

from __future__ import annotations

import ctypes

from oracle import oracle


def test_division_free_quotient_matches_ieee_division_on_every_reachable_pair():
    lib = oracle.lib()
    lib.kvo_fast_quotient_mismatches.argtypes = [ctypes.POINTER(ctypes.c_int64)]
    lib.kvo_fast_quotient_mismatches.restype = ctypes.c_int64
    pairs = ctypes.c_int64(0)
    assert lib.kvo_fast_quotient_mismatches(ctypes.byref(pairs)) == 0
    assert pairs.value == 929_598_054
