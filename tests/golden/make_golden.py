#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ by running the reference itself.

The reference (a pure-Python project) is imported read-only from
``--ref`` (its ``reference/`` directory is put on sys.path); its vector
generators are run in a temporary directory (they write into the current
directory).  Nothing from the reference is copied: only its outputs on the
inputs below are stored, as compressed .npz files.

    python tests/golden/make_golden.py --ref /root/reference

Fixtures
  encoder_vectors.npz  reference/gen_encoder_vectors.py: 132,811 quire256 -> bp32
  bp8_exhaustive.npz   reference/gen_bp8_exhaustive.py: all 65,536 bp8 products -> bp32
  rtl_bp8.npz          reference/gen_rtl_vectors.py: bp8 mant/exp ROMs, 22 K=32 dots
  fast_selftest.npz    reference/bposit_fast.py:179-212 self-test dots (bp8) and
                       the quantize_bp8 vs encode_bposit8 sample
  quantize_bp8.npz     bposit_fast.quantize_bp8 (nearest True/False) on mids +-1ulp,
                       grid +-1ulp, specials and a seeded sample
  bp16.npz             decode of all 65,536 bp16 codes; encode_bposit16(Fraction(x),
                       "rtne"/"truncate") on grid points, means +-1ulp, samples
  bp32_decode.npz      decode_bposit32 of the roundtrip_test.py code sample
  w8a8_linear.npz      the 16x576x576 group-scaled W8A8 linear, composed from
                       quantize_bp8(nearest=True), code_value, the per-term quire
                       rule of dot_at_precision and quire256_to_bposit32
  quantize_w8a8.npz    bposit_quantize.quantize_w8a8 on examples/smoke_test.sh's
                       W[16,32] / X[4,32] (seeds 0 / 1)
  quire_bp16.npz       quire256_to_bposit16 on the encoder-vector quires plus
                       saturation / regime-edge / seeded quires
  rungs.npz            bposit4 / AI-posit5: code values, quantize_vec on edge and
                       seeded floats, dot_at_precision (bp4, aip5, bp8 -> bp32,
                       bp16) and mixed_precision_sum over bp4/aip5/bp8/bp16 items
"""
from __future__ import annotations

import argparse
import math
import os
import random
import subprocess
import sys
import tempfile
import time
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "open-bposit_b200"))
from bposit_b200 import workloads  # noqa: E402


def hexlines(p: Path):
    return [ln.strip() for ln in p.read_text().splitlines() if ln.strip()]


def to_limbs(v: int, nl: int):
    return [(v >> (32 * i)) & 0xFFFFFFFF for i in range(nl)]


def run_gen(refdir: Path, script: str, tmp: Path):
    subprocess.run([sys.executable, str(refdir / "reference" / script)], cwd=tmp, check=True,
                   stdout=subprocess.DEVNULL)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    refdir = Path(args.ref)
    sys.path.insert(0, str(refdir / "reference"))
    import bposit_ref as bp  # noqa: E402
    import bposit_fast as bf  # noqa: E402
    import bposit_quantize as bq  # noqa: E402

    only = set(args.only.split(",")) if args.only else None

    def want(name):
        return only is None or name in only

    t0 = time.time()
    with tempfile.TemporaryDirectory() as td:
        tmp = Path(td)
        if want("encoder_vectors"):
            run_gen(refdir, "gen_encoder_vectors.py", tmp)
            q = hexlines(tmp / "qin.hex")
            e = hexlines(tmp / "ebp.hex")
            limbs = np.array([to_limbs(int(h, 16), 8) for h in q], dtype=np.uint32)
            np.savez_compressed(HERE / "encoder_vectors.npz", quire=limbs,
                                bp32=np.array([int(h, 16) for h in e], dtype=np.uint32))
            print("encoder_vectors", len(q), f"{time.time()-t0:.1f}s")
        if want("bp8_exhaustive"):
            run_gen(refdir, "gen_bp8_exhaustive.py", tmp)
            a = np.array([int(h, 16) for h in hexlines(tmp / "bp8x_a.hex")], np.uint8)
            b = np.array([int(h, 16) for h in hexlines(tmp / "bp8x_b.hex")], np.uint8)
            ebp = np.array([int(h, 16) for h in hexlines(tmp / "bp8x_ebp.hex")], np.uint32)
            np.savez_compressed(HERE / "bp8_exhaustive.npz", a=a, b=b, bp32=ebp)
            print("bp8_exhaustive", len(a), f"{time.time()-t0:.1f}s")
        if want("rtl_bp8"):
            run_gen(refdir, "gen_rtl_vectors.py", tmp)
            mant = np.array([int(h, 16) for h in hexlines(tmp / "bp8_mant.hex")], np.uint16).view(np.int16)
            expo = np.array([int(h, 16) for h in hexlines(tmp / "bp8_exp.hex")], np.uint8).view(np.int8)
            a = np.array([int(h, 16) for h in hexlines(tmp / "bp8_a.hex")], np.uint8)
            b = np.array([int(h, 16) for h in hexlines(tmp / "bp8_b.hex")], np.uint8)
            eq = np.array([to_limbs(int(h, 16), 8) for h in hexlines(tmp / "bp8_eq.hex")], np.uint32)
            ebp = np.array([int(h, 16) for h in hexlines(tmp / "bp8_ebp.hex")], np.uint32)
            n = len(ebp)
            np.savez_compressed(HERE / "rtl_bp8.npz", mant=mant, exp=expo, a=a.reshape(n, -1),
                                b=b.reshape(n, -1), quire=eq, bp32=ebp)
            print("rtl_bp8", n, f"{time.time()-t0:.1f}s")

    if want("fast_selftest"):
        # same generator draws as reference/bposit_fast.py:181-203 (seed 0)
        rng = np.random.default_rng(0)
        nb = {"bp4": 4, "aip5": 5, "bp8": 8}
        A, B, off, exp_bp32 = [], [], [0], []
        for fmt in ("bp4", "aip5", "bp8"):
            n = 1 << nb[fmt]
            for _ in range(300):
                K = int(rng.integers(1, 400))
                a = rng.integers(0, n, size=K, dtype=np.int64)
                b = rng.integers(0, n, size=K, dtype=np.int64)
                if fmt == "bp8":
                    A.append(a.astype(np.uint8)); B.append(b.astype(np.uint8))
                    off.append(off[-1] + K)
                    exp_bp32.append(bp.dot_at_precision(a.tolist(), b.tolist(), "bp8", "bp32"))
        _g, minpos = bf._grid("bp8")
        xs = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 0.05, 0.5, 5.0, 500.0, 1e5)])
        xs = xs[np.abs(xs) >= minpos]
        enc = np.array([bp.encode_bposit8(float(v)) for v in xs], dtype=np.uint8)
        qv = bf.quantize_bp8(xs)
        assert np.array_equal(qv, np.array([0.0 if c == 0x80 else float(bp.code_value(int(c), "bp8"))
                                            for c in enc]))
        np.savez_compressed(HERE / "fast_selftest.npz", a=np.concatenate(A), b=np.concatenate(B),
                            off=np.array(off, np.int64), bp32=np.array(exp_bp32, np.uint32),
                            xs=xs[::4], enc_codes=enc[::4])
        print("fast_selftest", len(exp_bp32), len(xs), f"{time.time()-t0:.1f}s")

    v2c = {float(bp.code_value(c, "bp8")): c for c in range(256) if c != 0x80}

    def codes_of(vals):
        return np.array([v2c[float(t)] for t in vals.ravel()], np.uint8).reshape(vals.shape)

    if want("quantize_bp8"):
        g, minpos = bf._grid("bp8")
        mids = bf._mids("bp8")
        f32 = np.float32
        pts = []
        for arr in (mids, g):
            v = arr.astype(f32)
            assert np.array_equal(v.astype(np.float64), arr), "grid/mids not exact in fp32"
            pts += [v, np.nextafter(v, f32(np.inf)), np.nextafter(v, f32(-np.inf))]
        specials = np.array([0.0, -0.0, np.inf, -np.inf, 2.0 ** 25, 2.0 ** 24 * 1.0625, 2.0 ** -25,
                             2.0 ** -26, 2.0 ** -24 * 0.75, 1e-38, 1e-45, 3e38, 2.0 ** 23 * 1.0625,
                             2.0 ** 17 * 1.25, 2.0 ** 19 * 1.25, 2.0 ** -21 * 1.0625,
                             2.0 ** -17 * 1.25, 2.0 ** -19 * 1.25], dtype=f32)
        pts.append(specials)
        rng = np.random.default_rng(1234)
        pts.append(rng.standard_normal(1 << 13).astype(f32))
        pts.append((np.exp2(rng.uniform(-27, 27, 1 << 13))).astype(f32))
        pts.append((rng.standard_normal(1 << 12) * 20).astype(f32))
        x = np.concatenate(pts).astype(f32)
        x = np.concatenate([x, -x])
        xd = x.astype(np.float64)
        vn = bf.quantize_bp8(xd, nearest=True)
        vt = bf.quantize_bp8(xd, nearest=False)
        np.savez_compressed(HERE / "quantize_bp8.npz", x=x, codes_nearest=codes_of(vn),
                            codes_trunc=codes_of(vt))
        print("quantize_bp8", len(x), f"{time.time()-t0:.1f}s")

    if want("bp16"):
        dec = np.empty(65536, np.float64)
        for c in range(65536):
            d = bp.decode_bposit16(c)
            dec[c] = np.nan if d.is_special == "nar" else float(bp.decoded_to_fraction(d))
        f32 = np.float32
        pos = dec[1:0x8000].astype(f32)
        assert np.array_equal(pos.astype(np.float64), dec[1:0x8000])
        means = ((dec[1:0x7FFF] + dec[2:0x8000]) / 2).astype(f32)
        rng = np.random.default_rng(4321)
        pts = [pos, means, np.nextafter(means, f32(np.inf)), np.nextafter(means, f32(-np.inf)),
               rng.standard_normal(1 << 14).astype(f32),
               np.exp2(rng.uniform(-118, 118, 1 << 14)).astype(f32),
               np.array([2.0 ** 113, 2.0 ** 112 * 1.5, 2.0 ** -113, 2.0 ** -112 * 1.5, 3e38, 1e-40,
                         2.0 ** -112, 2.0 ** 112], dtype=f32)]
        x = np.concatenate(pts)
        x = np.concatenate([x, -x[::7]])
        rt = np.array([bp.encode_bposit16(Fraction(float(v)), "rtne") for v in x], np.uint16)
        tr = np.array([bp.encode_bposit16(Fraction(float(v)), "truncate") for v in x[::4]], np.uint16)
        np.savez_compressed(HERE / "bp16.npz", decoded=dec, x=x, rtne=rt, x_trunc=x[::4], trunc=tr)
        print("bp16", len(x), f"{time.time()-t0:.1f}s")

    if want("bp32_decode"):
        rng = random.Random(20260720)  # reference/roundtrip_test.py:48-50
        codes = list(range(1, 64)) + list(range(0x7FFFFFFF - 64, 0x7FFFFFFF)) + \
            [rng.randrange(1, 1 << 32) for _ in range(200000)]
        codes = codes[::4] + [0, 0x80000000, 0x7FFFFFFF, 0x80000001, 0xFFFFFFFF, 1]
        vals = []
        for c in codes:
            d = bp.decode_bposit32(c)
            vals.append(np.nan if d.is_special == "nar" else float(bp.decoded_to_fraction_32(d)))
        np.savez_compressed(HERE / "bp32_decode.npz", codes=np.array(codes, np.uint32),
                            values=np.array(vals, np.float64))
        print("bp32_decode", len(codes), f"{time.time()-t0:.1f}s")

    if want("w8a8_linear"):
        X, W = workloads.w8a8_linear(seed=0)
        group = 128

        def scales(M):
            rows, K = M.shape
            G = (K + group - 1) // group
            s = np.zeros((rows, G), np.int32)
            for r in range(rows):
                for gi in range(G):
                    amax = float(np.max(np.abs(M[r, gi * group:(gi + 1) * group].astype(np.float64))))
                    if amax > 0:
                        m, e = math.frexp(amax)
                        s[r, gi] = (e - 1 if m == 0.5 else e) - 24
            return s

        sx, sw = scales(X), scales(W)
        Kk = X.shape[1]
        gidx = np.arange(Kk) // group
        xq = bf.quantize_bp8(X.astype(np.float64) * np.exp2(-sx[:, gidx].astype(np.float64)), nearest=True)
        wq = bf.quantize_bp8(W.astype(np.float64) * np.exp2(-sw[:, gidx].astype(np.float64)), nearest=True)
        xc, wc = codes_of(xq), codes_of(wq)
        cv = [bp.code_value(c, "bp8") for c in range(256)]
        two = Fraction(2)
        ONE96 = 1 << bp.QUIRE_FRAC_BITS
        M, N = X.shape[0], W.shape[0]
        out = np.zeros((M, N), np.uint32)
        quires = np.zeros((M, N, 8), np.uint32)
        pw = {}
        for m in range(M):
            for n in range(N):
                q = 0
                for k in range(Kk):
                    a, b = int(xc[m, k]), int(wc[n, k])
                    if a == 0 or b == 0 or a == 0x80 or b == 0x80:
                        continue
                    s = int(sx[m, gidx[k]] + sw[n, gidx[k]])
                    f = pw.get(s)
                    if f is None:
                        f = pw[s] = two ** s
                    q += int(cv[a] * cv[b] * f * ONE96)
                out[m, n] = bp.quire256_to_bposit32(q) & 0xFFFFFFFF
                quires[m, n] = to_limbs(q & ((1 << 256) - 1), 8)
            print(f"  w8a8_linear row {m} {time.time()-t0:.1f}s", flush=True)
        np.savez_compressed(HERE / "w8a8_linear.npz", X=X, W=W, sx=sx, sw=sw, xc=xc, wc=wc,
                            bp32=out, quire=quires)
        print("w8a8_linear", out.shape, f"{time.time()-t0:.1f}s")

    if want("quire_bp16"):
        # the encoder-vector quires are already in encoder_vectors.npz: store
        # only their bp16 rounds, plus the extra quires with theirs
        ev = np.load(HERE / "encoder_vectors.npz")
        qs = [sum(int(w) << (32 * i) for i, w in enumerate(row)) for row in ev["quire"]]
        qs = [q - (1 << 256) if q >> 255 else q for q in qs]
        ev16 = np.array([bp.quire256_to_bposit16(q) & 0xFFFF for q in qs], np.uint16)
        rng = random.Random(16)
        extra = [0, 1, -1, (1 << 255) - 1, -(1 << 255)]
        for t in range(0, 255):             # every power of two and its neighbours (all fit 256 bits)
            for d in (-1, 0, 1):
                v = (1 << t) + d
                extra += [v, -v]
        for _ in range(6000):               # seeded magnitudes over the whole quire
            nb = rng.randrange(1, 256)
            v = rng.getrandbits(nb)
            extra.append(-v if rng.random() < 0.5 else v)
        out = np.array([bp.quire256_to_bposit16(q) & 0xFFFF for q in extra], np.uint16)
        limbs = np.array([to_limbs(q & ((1 << 256) - 1), 8) for q in extra], np.uint32)
        np.savez_compressed(HERE / "quire_bp16.npz", ev_bp16=ev16, quire=limbs, bp16=out)
        print("quire_bp16", len(qs) + len(extra), f"{time.time()-t0:.1f}s")

    if want("rungs"):
        rng = np.random.default_rng(45)
        res = {}
        for fmt, nb in (("bp4", 4), ("aip5", 5)):
            res[f"{fmt}_values"] = np.array([float(bp.code_value(c, fmt)) for c in range(1 << nb)])
        edges = [0.0, -0.0, 1.0, 1.5, 3.0, 3.9, 4.0, 7.99, 8.0, 16.0, 17.0, 64.0, 100.0, 1e30, 0.25, 0.2, 0.0625,
                 0.05, 0.015625, 0.01, 1e-9, 5e-9, 4.999999999999999e-09, 1.0 / 3, 0.375, 0.74, 0.75, 2.0 ** -30]
        vals = np.array(edges + [-v for v in edges] +
                        list(rng.standard_normal(3000) * np.exp2(rng.integers(-8, 8, 3000))), np.float64)
        res["q_in"] = vals
        for fmt in ("bp4", "aip5", "bp8"):
            res[f"q_{fmt}"] = np.array(bp.quantize_vec([float(v) for v in vals], fmt), np.uint8)
        # dot_at_precision on random code vectors
        for fmt, nb in (("bp4", 4), ("aip5", 5), ("bp8", 8)):
            L = 40
            lens = rng.integers(1, 300, L)
            a = [rng.integers(0, 1 << nb, n) for n in lens]
            b = [rng.integers(0, 1 << nb, n) for n in lens]
            res[f"dot_{fmt}_len"] = lens
            res[f"dot_{fmt}_a"] = np.concatenate(a).astype(np.uint8)
            res[f"dot_{fmt}_b"] = np.concatenate(b).astype(np.uint8)
            for of in ("bp32", "bp16"):
                res[f"dot_{fmt}_{of}"] = np.array(
                    [bp.dot_at_precision(list(map(int, x)), list(map(int, y)), fmt, of) for x, y in zip(a, b)],
                    np.uint32)
        # mixed_precision_sum over all four rungs
        fm = ("bp4", "aip5", "bp8", "bp16")
        nbs = (4, 5, 8, 16)
        lens = rng.integers(1, 200, 60)
        fi = [rng.integers(0, 4, n) for n in lens]
        codes = [np.array([rng.integers(0, 1 << nbs[j]) for j in f]) for f in fi]
        res["mix_len"] = lens
        res["mix_fmt"] = np.concatenate(fi).astype(np.uint8)
        res["mix_code"] = np.concatenate(codes).astype(np.uint16)
        for of in ("bp32", "bp16"):
            res[f"mix_{of}"] = np.array([bp.mixed_precision_sum([(int(c), fm[j]) for c, j in zip(cs, f)], of)
                                         for cs, f in zip(codes, fi)], np.uint32)
        np.savez_compressed(HERE / "rungs.npz", **res)
        print("rungs", f"{time.time()-t0:.1f}s")

    if want("quantize_w8a8"):
        W = np.random.default_rng(0).standard_normal((16, 32)) * 0.05
        X = np.random.default_rng(1).standard_normal((4, 32)) * 0.5
        Y = bq.quantize_w8a8(W, X)
        np.savez_compressed(HERE / "quantize_w8a8.npz", W=W, X=X, Y=Y,
                            w_exp=bq.recommended_exponents(W), x_exp=bq.recommended_exponents(X))
        print("quantize_w8a8", Y.shape, f"{time.time()-t0:.1f}s")


if __name__ == "__main__":
    main()
