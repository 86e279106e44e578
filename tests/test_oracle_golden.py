"""Pin the CPU oracle (oracle/bposit_oracle.c) to the reference's own outputs.

Every fixture under tests/golden/ was produced by running the reference
(tests/golden/make_golden.py); these tests check the oracle against all of
them, so that the GPU parity tests can trust it at sizes the reference's
Python cannot reach.
"""
from __future__ import annotations

import numpy as np

from conftest import golden


def test_encoder_vectors_quire_to_bp32(orc):
    """reference/gen_encoder_vectors.py: 132,811 quire256 -> bposit32 pairs."""
    g = golden("encoder_vectors")
    got = orc.quire_to_bp32(g["quire"])
    assert np.array_equal(got, g["bp32"])


def test_bp8_exhaustive_products(orc):
    """reference/gen_bp8_exhaustive.py: every bp8 x bp8 product (K=1)."""
    g = golden("bp8_exhaustive")
    A = g["a"].reshape(256, 256)[:, :1]   # a-code varies along the first axis
    B = np.arange(256, dtype=np.uint8).reshape(256, 1)
    got = orc.quire_gemm(A, B, 8)          # [256 a, 256 b]
    assert np.array_equal(got.ravel(), g["bp32"])


def test_rtl_bp8_roms_and_dots(orc):
    """reference/gen_rtl_vectors.py:288-325: the bp8 (mant, exp) ROMs and 22
    K=32 dots with their 256-bit quires and bposit32 results."""
    g = golden("rtl_bp8")
    L = orc.lib()
    import ctypes
    for c in range(256):
        m = ctypes.c_int64(); e = ctypes.c_int()
        L.orc_decode_me(8, c, ctypes.byref(m), ctypes.byref(e))
        assert m.value == int(g["mant"][c]) and (e.value if m.value else 0) == int(g["exp"][c]), c
    a, b = g["a"], g["b"]
    for i in range(a.shape[0]):
        bp32, q = orc.quire_gemm(a[i:i + 1], b[i:i + 1], 8, nlimbs=8)
        assert np.array_equal(q[0, 0], g["quire"][i]), i
        assert int(bp32[0, 0]) == int(g["bp32"][i]), i


def test_fast_selftest_dots(orc):
    """reference/bposit_fast.py:181-197: the 300 seeded bp8 dots."""
    g = golden("fast_selftest")
    off = g["off"]
    for i in range(len(off) - 1):
        a = g["a"][off[i]:off[i + 1]][None, :]
        b = g["b"][off[i]:off[i + 1]][None, :]
        assert int(orc.quire_gemm(a, b, 8)[0, 0]) == int(g["bp32"][i]), i


def test_fast_selftest_quantize_trunc(orc):
    """reference/bposit_fast.py:199-212: truncating quantize == per-element
    encode_bposit8 over the seeded multi-scale sample."""
    g = golden("fast_selftest")
    got = orc.quantize_bp8_f64(g["xs"], nearest=False)
    assert np.array_equal(got, g["enc_codes"])


def test_quantize_bp8_nearest_and_trunc(orc):
    """bposit_fast.quantize_bp8(nearest=True/False) on every midpoint and grid
    point +-1 ulp, the specials and a seeded sample."""
    g = golden("quantize_bp8")
    cn, vn = orc.quantize_bp8(g["x"], nearest=True)
    ct, _ = orc.quantize_bp8(g["x"], nearest=False)
    assert np.array_equal(cn, g["codes_nearest"])
    assert np.array_equal(ct, g["codes_trunc"])
    assert np.array_equal(vn, orc.decode_f32(cn, 8))


def test_bp16_decode_all_codes(orc):
    g = golden("bp16")
    dec = g["decoded"]
    got = orc.decode_f32(np.arange(65536, dtype=np.uint16), 16).astype(np.float64)
    ok = np.where(np.isnan(dec), got == 0, got == dec)
    assert ok.all()


def test_bp16_encode_rtne_and_trunc(orc):
    """encode_bposit16(Fraction(x), "rtne" / "truncate")."""
    g = golden("bp16")
    assert np.array_equal(orc.encode_bp16(g["x"], rtne=True), g["rtne"])
    assert np.array_equal(orc.encode_bp16(g["x_trunc"], rtne=False), g["trunc"])


def test_bp32_decode(orc):
    g = golden("bp32_decode")
    got = orc.bp32_to_double(g["codes"])
    v = g["values"]
    assert np.array_equal(np.isnan(got), np.isnan(v))
    assert np.array_equal(got[~np.isnan(v)], v[~np.isnan(v)])


def test_w8a8_linear_group_scaled(orc):
    """The group-scaled bp8 W8A8 linear (16x576x576): scales, RTN codes, every
    256-bit quire and every bposit32 output word."""
    g = golden("w8a8_linear")
    X, W = g["X"], g["W"]
    sx, sw = orc.group_scales(X), orc.group_scales(W)
    assert np.array_equal(sx, g["sx"]) and np.array_equal(sw, g["sw"])
    xc = orc.quantize_bp8_grouped(X, sx)
    wc = orc.quantize_bp8_grouped(W, sw)
    assert np.array_equal(xc, g["xc"]) and np.array_equal(wc, g["wc"])
    bp32, q = orc.quire_gemm(xc, wc, 8, sa=sx, sb=sw, nlimbs=8)
    assert np.array_equal(q, g["quire"])
    assert np.array_equal(bp32, g["bp32"])


def test_quantize_w8a8_fixture_present():
    g = golden("quantize_w8a8")
    assert g["Y"].shape == (4, 16)


def test_quire_to_bp16(orc):
    """quire256_to_bposit16 (reference/bposit_ref.py:620-635): the encoder-vector
    quires plus power-of-two, saturation and seeded quires."""
    g = golden("quire_bp16")
    ev = golden("encoder_vectors")
    assert np.array_equal(orc.quire_to_bp16(ev["quire"]), g["ev_bp16"])
    assert np.array_equal(orc.quire_to_bp16(g["quire"]), g["bp16"])


NB = {"bp4": 4, "aip5": 5, "bp8": 8, "bp16": 16}


def test_rungs_values_and_transcode(orc):
    """Every bposit4 / AI-posit5 code: its value (code_value) is the value of its
    bp8 and bp16 transcodes."""
    g = golden("rungs")
    for fmt in ("bp4", "aip5"):
        codes = np.arange(1 << NB[fmt], dtype=np.uint8)
        for out in (8, 16):
            t = orc.transcode(codes, NB[fmt], out)
            v = orc.decode_f32(t, out).astype(np.float64)
            assert np.array_equal(v, g[f"{fmt}_values"]), (fmt, out)


def test_rungs_quantize(orc):
    """quantize_vec (reference/bposit_ref.py:1017-1019) for bp4, aip5 and bp8."""
    g = golden("rungs")
    x = g["q_in"]
    assert np.array_equal(orc.quantize_small(x, 4), g["q_bp4"])
    assert np.array_equal(orc.quantize_small(x, 5), g["q_aip5"])
    c8 = orc.quantize_bp8_f64(x, nearest=False)
    c8 = np.where(np.abs(x) <= 4.999999999999999e-09, 0, c8)   # limit_denominator(10**8) zero cut
    assert np.array_equal(c8, g["q_bp8"])


def test_rungs_dot_at_precision(orc):
    """dot_at_precision (reference/bposit_ref.py:1028-1035) for bp4, aip5, bp8 with
    bp32 and bp16 outputs: the bp8 quire GEMM on transcoded codes."""
    g = golden("rungs")
    for fmt in ("bp4", "aip5", "bp8"):
        lens = g[f"dot_{fmt}_len"]
        off = np.concatenate([[0], np.cumsum(lens)])
        for i in range(len(lens)):
            a = g[f"dot_{fmt}_a"][off[i]:off[i + 1]]
            b = g[f"dot_{fmt}_b"][off[i]:off[i + 1]]
            if fmt != "bp8":
                a, b = orc.transcode(a, NB[fmt], 8), orc.transcode(b, NB[fmt], 8)
            out, q = orc.quire_gemm(a[None, :], b[None, :], 8, nlimbs=16)
            assert int(out[0, 0]) == int(g[f"dot_{fmt}_bp32"][i]), (fmt, i)
            assert int(orc.quire_to_bp16(q.reshape(1, 16))[0]) == int(g[f"dot_{fmt}_bp16"][i]), (fmt, i)


def test_rungs_mixed_precision_sum(orc):
    """mixed_precision_sum (reference/bposit_ref.py:995-1002) over bp4/aip5/bp8/bp16
    items: every item transcoded to bp16, one bp16 quire row against 1.0."""
    g = golden("rungs")
    fm = (4, 5, 8, 16)
    lens = g["mix_len"]
    off = np.concatenate([[0], np.cumsum(lens)])
    for i in range(len(lens)):
        f = g["mix_fmt"][off[i]:off[i + 1]]
        c = g["mix_code"][off[i]:off[i + 1]]
        row = np.empty(len(c), np.uint16)
        for j in range(4):
            m = f == j
            row[m] = c[m] if fm[j] == 16 else orc.transcode(c[m].astype(np.uint8), fm[j], 16)
        ones = np.full((1, len(c)), 0x4000, np.uint16)
        out, q = orc.quire_gemm(row[None, :], ones, 16, nlimbs=16)
        assert int(out[0, 0]) == int(g["mix_bp32"][i]), i
        assert int(orc.quire_to_bp16(q.reshape(1, 16))[0]) == int(g["mix_bp16"][i]), i
