"""Properties of the b-posit formats that the device kernels rely on, checked
over every code with the oracle's decoder."""
from __future__ import annotations

import ctypes

import pytest


def _me(orc, fmt, c):
    m, e = ctypes.c_int64(), ctypes.c_int()
    orc.lib().orc_decode_me(fmt, c, ctypes.byref(m), ctypes.byref(e))
    return m.value, e.value


@pytest.mark.parametrize("fmt,top", [(8, 0x7F), (16, 0x7FFF)])
def test_lsb_and_binade_monotone_in_magnitude(orc, fmt, top):
    """The tensor-core prep takes a row's min lsb exponent and max binade from
    its smallest and largest nonzero code magnitude: both must be
    non-decreasing in the magnitude code, and a negative code must decode to
    the negation of its two's complement."""
    prev_l = prev_h = -10 ** 9
    for c in range(1, top + 1):
        m, e = _me(orc, fmt, c)
        hb = e + abs(m).bit_length() - 1
        assert e >= prev_l and hb >= prev_h, c
        prev_l, prev_h = e, hb
    for c in range(top + 2, 2 * (top + 1)):
        m, e = _me(orc, fmt, c)
        m2, e2 = _me(orc, fmt, 2 * (top + 1) - c)
        assert m == -m2 and e == e2, c
