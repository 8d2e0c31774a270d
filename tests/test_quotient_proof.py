"""The device quantizer divides without a division instruction; prove it exact.

csrc/codec.cuh quant_input replaces IEEE x / s by a correctly rounded
reciprocal, one multiply and two FMAs, and scale_from_amax replaces amax / 448
by a multiply with RN(1/448). These tests check, for every (x, scale) pair an
FP8 row can produce and for every bf16 amax, that the resulting e4m3 byte and
bf16 scale equal the ones IEEE division gives (the oracle runs the checks in C
over all 929,598,054 pairs and all 32,640 amax values).
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


def test_scale_multiply_matches_ieee_division_for_every_amax():
    lib = oracle.lib()
    lib.kvo_scale_multiply_mismatches.restype = ctypes.c_int32
    assert lib.kvo_scale_multiply_mismatches() == 0
