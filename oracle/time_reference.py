"""Times the reference's own Python (reference/bposit_fast.py, bposit_ref.py)
against the oracle port (oracle/bposit_oracle.c) on the same seeded samples,
one core each, in the container that holds the reference.  Test and
measurement infrastructure only: the reference does not exist where the GPU
benchmark runs, so the benchmark times the port there and this ratio says how
a port figure translates into the reference's own speed.

    python oracle/time_reference.py [--ref /root/reference/reference] [--out oracle/reference_timing.json]

Workloads (all from the benchmark's definitions):
  * quantize_bp8(x, nearest=True) on 2^22 values of the codec sweep
    (reference/bposit_fast.py:69-99) vs the port's quantize_bp8;
  * encode_bposit16(Fraction(x), "rtne") per element on 2^12 values
    (reference/bposit_ref.py:489-507) vs the port's encode_bp16 on 2^22;
  * matmul_quire + quire256_to_bposit32 per output (reference/bposit_fast.py:136-176,
    reference/bposit_ref.py:703-722) on the 16x576x576 W8A8 linear's codes and on
    2 rows of the 4096x65536 large-GEMM operands against 64 columns, vs the
    port's quire_gemm (one thread).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from fractions import Fraction

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_HERE = os.path.dirname(os.path.abspath(__file__))
# this file's own folder would shadow the oracle package with oracle/oracle.py
sys.path[:] = [REPO, os.path.join(REPO, "open-bposit_b200")] + [p for p in sys.path if os.path.abspath(p or ".") != _HERE]


def _t(fn, min_s=1.0):
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= min_s:
            return dt / n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference/reference")
    ap.add_argument("--out", default=os.path.join(REPO, "oracle", "reference_timing.json"))
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import bposit_fast as bf
    import bposit_ref as br

    from bposit_b200 import workloads
    from oracle import oracle as orc

    res = {"cores": 1, "host": os.uname().nodename, "python": sys.version.split()[0], "numpy": np.__version__}
    # quantize_bp8 nearest
    x = workloads.codec_sweep(1 << 22, "bp8", seed=0)
    tr = _t(lambda: bf.quantize_bp8(x, nearest=True))
    tp = _t(lambda: orc.quantize_bp8(x, True))
    assert np.array_equal(bf.quantize_bp8(x, nearest=True), orc.quantize_bp8(x, True)[1].astype(np.float64)), \
        "quantize_bp8 differs"
    res["quantize_bp8_nearest"] = {"elements": x.size, "reference_s": tr, "port_s": tp,
                                   "reference_GBps": 5 * x.size / tr / 1e9, "port_GBps": 5 * x.size / tp / 1e9,
                                   "ratio": tr / tp}
    # bp16 RTNE encode
    xs = workloads.codec_sweep(1 << 12, "bp16", seed=1)
    tr = _t(lambda: [br.encode_bposit16(Fraction(float(v)), "rtne") for v in xs]) / xs.size
    xb = workloads.codec_sweep(1 << 22, "bp16", seed=1)
    tp = _t(lambda: orc.encode_bp16(xb, True)) / xb.size
    ref_codes = np.array([br.encode_bposit16(Fraction(float(v)), "rtne") for v in xs], np.uint16)
    assert np.array_equal(ref_codes, orc.encode_bp16(xs, True)), "encode_bp16 differs"
    res["encode_bp16_rtne"] = {"reference_s_per_elem": tr, "port_s_per_elem": tp,
                               "reference_GBps": 6 / tr / 1e9, "port_GBps": 6 / tp / 1e9, "ratio": tr / tp}
    # quire GEMM + bp32 round
    X, W = workloads.w8a8_linear(seed=0)
    A, B = orc.quantize_bp8(X)[0], orc.quantize_bp8(W)[0]

    def ref_gemm(A_, B_):
        q = bf.matmul_quire(A_, B_, "bp8")
        return np.array([[br.quire256_to_bposit32(int(v)) for v in row] for row in q], np.uint32)

    tr = _t(lambda: ref_gemm(A, B), 2.0)
    tp = _t(lambda: orc.quire_gemm(A, B, 8, nthreads=1))
    assert np.array_equal(ref_gemm(A, B), orc.quire_gemm(A, B, 8, nthreads=1)), "quire GEMM differs"
    macs = A.shape[0] * B.shape[0] * A.shape[1]
    res["quire_gemm_16x576x576"] = {"reference_s": tr, "port_s": tp, "reference_TOPS": 2 * macs / tr / 1e12,
                                    "port_TOPS": 2 * macs / tp / 1e12, "ratio": tr / tp}
    rng = np.random.default_rng(0)
    K = 65536
    xa = (rng.standard_normal((2, K)) * np.exp2(rng.integers(-8, 9, (2, 1)))).astype(np.float32)
    xb = (rng.standard_normal((64, K)) * np.exp2(rng.integers(-8, 9, (64, 1)))).astype(np.float32)
    A2, B2 = orc.quantize_bp8(xa)[0], orc.quantize_bp8(xb)[0]
    tr = _t(lambda: ref_gemm(A2, B2), 2.0)
    tp = _t(lambda: orc.quire_gemm(A2, B2, 8, nthreads=1))
    assert np.array_equal(ref_gemm(A2, B2), orc.quire_gemm(A2, B2, 8, nthreads=1)), "large-K GEMM differs"
    macs = 2 * 64 * K
    res["quire_gemm_2x64x65536"] = {"reference_s": tr, "port_s": tp, "reference_TOPS": 2 * macs / tr / 1e12,
                                    "port_TOPS": 2 * macs / tp / 1e12, "ratio": tr / tp}
    with open(a.out, "w") as f:
        json.dump(res, f, indent=1)
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
