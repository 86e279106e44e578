"""CPU checks of the packed-integer identities the tensor-core preparation
kernels rely on (csrc/bp_gemm_tc.cu), evaluated with numpy on every input they
can see:

* k_tc_prep's row statistics (unscaled bp8): two codes per register in 16-bit
  lanes, |c| = min(c, 0x100 - c) and (|c| + 0x7FFF) & 0x7FFF (= |c| - 1, zero
  -> 0x7FFF) computed on the whole register without a carry or borrow between
  the lanes; the row's min and max code magnitude over nonzero, non-NaR codes
  follow, a NaR showing as a lane value of 128;
* k_kmajor_bp8's keep mask and E bytes: per byte, (lw | 0x80) - L and
  (lw | 0x80) - la never borrow from the next byte, bit 7 of the first is
  lw >= L, and the low 7 bits of the second are lw - la.
"""
from __future__ import annotations

import numpy as np

M32 = 0xFFFFFFFF


def _lanes(x):
    return x & 0xFFFF, x >> 16


def test_prep_code_magnitudes_in_16bit_lanes():
    c = np.arange(256, dtype=np.int64)
    c0, c1 = np.meshgrid(c, c, indexing="ij")
    x = (c0 | (c1 << 16)).ravel()                         # two codes per register (zero-extended bytes)
    t = (0x01000100 - x) & M32                           # 0x100 - c per lane, no borrow: c <= 0xFF
    assert (((t & 0xFFFF) == 0x100 - (x & 0xFFFF))).all() and ((t >> 16) == 0x100 - (x >> 16)).all()
    lo = np.minimum(x & 0xFFFF, t & 0xFFFF)
    hi = np.minimum(x >> 16, t >> 16)
    mag = lo | (hi << 16)                                # min.u16x2(x, 0x01000100 - x)
    m1 = ((mag + 0x7FFF7FFF) & M32) & 0x7FFF7FFF
    ref = np.where(c0 >= 128, 256 - c0, c0).ravel(), np.where(c1 >= 128, 256 - c1, c1).ravel()
    for lane, (got, r) in enumerate(zip(_lanes(mag), ref)):
        assert (got == r).all(), lane
    for lane, (got, r) in enumerate(zip(_lanes(m1), ref)):
        assert (got == np.where(r == 0, 0x7FFF, r - 1)).all(), lane
    # the only code with |c| = 128 is NaR; every other nonzero code has |c| <= 127
    assert set(np.nonzero(np.where(c >= 128, 256 - c, c) == 128)[0]) == {0x80}


def test_prep_row_min_max_match_the_per_code_rule():
    rng = np.random.default_rng(5)
    for _ in range(2000):
        n = int(rng.integers(1, 64))
        pool = np.array([0, 0x80, 1, 0x7F, 0x81, 0xFF, 0x40, 0xC0], np.int64)
        codes = np.where(rng.random(n) < 0.3, rng.choice(pool, n), rng.integers(0, 256, n))
        mag = np.where(codes >= 128, 256 - codes, codes)
        mx = int(mag.max())
        mn = int(np.where(mag == 0, 0x7FFF, mag - 1).min()) + 1
        valid = mag[(codes & 0x7F) != 0]
        if mx == 128:   # a NaR: the kernel redoes the span code by code
            continue
        assert mx == (int(valid.max()) if valid.size else 0)
        if valid.size:
            assert mn == int(valid.min())


def test_kmajor_keep_mask_and_e_bytes():
    lsb = np.arange(-24, 25)
    lw = np.concatenate([[0], lsb + 64])                 # a byte: 0 for zero / NaR, else lsb + 64
    Lb = np.arange(1, 128)                                # clamp(L + 64, 1, 127)
    lab = lsb + 64                                        # la + 64
    w, L, a = np.meshgrid(lw, Lb, lab, indexing="ij")
    w, L, a = w.ravel(), L.ravel(), a.ravel()
    x = w | 0x80
    d1 = x - L
    d2 = x - a
    assert (d1 >= 1).all() and (d1 <= 0xFF).all()         # no borrow out of the byte
    assert (d2 >= 1).all() and (d2 <= 0xFF).all()
    keep = (d1 & 0x80) != 0
    assert (keep == ((w >= L) & (w != 0))).all()
    kept = keep & (w >= a)                                # la is the row's minimum lsb of kept elements
    assert ((d2[kept] & 0x7F) == (w[kept] - a[kept])).all()
    # whole 32-bit words: four independent bytes
    rng = np.random.default_rng(9)
    idx = rng.integers(0, w.size, (4096, 4))
    W = sum(w[idx[:, i]].astype(np.int64) << (8 * i) for i in range(4))
    LL = sum(L[idx[:, i]].astype(np.int64) << (8 * i) for i in range(4))
    X = W | 0x80808080
    D = (X - LL) & M32
    for i in range(4):
        assert (((D >> (8 * i)) & 0xFF) == (x[idx[:, i]] - L[idx[:, i]])).all()
