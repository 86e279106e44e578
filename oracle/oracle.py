"""ctypes front end of the CPU oracle (oracle/bposit_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check in
__graft_entry__.py and by the cpu_baseline / reference arm of bench.py, never by
the product package.  Each function names the reference function whose
semantics it restates (paths relative to the reference project root).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libbposit_oracle.so")
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or (
            os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_HERE, "bposit_oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_SO)
        vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        L.orc_decode_f32.argtypes = [i32, vp, sz, vp]
        L.orc_quantize_bp8.argtypes = [vp, sz, i32, vp, vp]
        L.orc_quantize_bp8_f64.argtypes = [vp, sz, i32, vp]
        L.orc_encode_bp16.argtypes = [vp, sz, i32, vp]
        L.orc_quire_to_bp32_batch.argtypes = [vp, i32, sz, vp]
        L.orc_quire_to_bp16_batch.argtypes = [vp, i32, sz, vp]
        L.orc_quantize_small.argtypes = [i32, vp, sz, vp]
        L.orc_transcode.argtypes = [i32, i32, vp, sz, vp]
        L.orc_group_scales.argtypes = [vp, i32, i32, i32, i32, vp]
        L.orc_quantize_bp8_grouped.argtypes = [vp, i32, i32, i32, vp, i32, vp]
        L.orc_quire_gemm.argtypes = [i32, vp, vp, i32, i32, i32, vp, vp, i32, vp, vp, i32, i32]
        L.orc_quire_gemm.restype = i32
        L.orc_bp32_to_double_batch.argtypes = [vp, sz, vp]
        L.orc_encode_bp8_exact.argtypes = [ctypes.c_double]
        L.orc_encode_bp8_exact.restype = ctypes.c_uint8
        L.orc_bp8_grid.argtypes = [vp, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def bp8_grid():
    """(grid[128], mids[127]) as float64 -- bposit_fast._grid / _mids
    (reference/bposit_fast.py:49-66)."""
    g = np.zeros(128, np.float64)
    m = np.zeros(127, np.float64)
    lib().orc_bp8_grid(_p(g), _p(m))
    return g, m


def decode_f32(codes: np.ndarray, fmt_bits: int) -> np.ndarray:
    """code -> fp32 value, NaR -> 0 (code_value, reference/bposit_ref.py:1022-1025)."""
    c = np.ascontiguousarray(codes, dtype=np.uint8 if fmt_bits == 8 else np.uint16)
    out = np.empty(c.shape, np.float32)
    lib().orc_decode_f32(fmt_bits, _p(c), c.size, _p(out))
    return out


def quantize_bp8(x: np.ndarray, nearest: bool = True):
    """(codes uint8, values fp32) of bposit_fast.quantize_bp8(x, nearest=...)
    (reference/bposit_fast.py:69-99); value->code as in
    examples/w8a8_rounding_demo.py:31."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.empty(x.shape, np.uint8)
    vals = np.empty(x.shape, np.float32)
    lib().orc_quantize_bp8(_p(x), x.size, int(bool(nearest)), _p(codes), _p(vals))
    return codes, vals


def quantize_bp8_f64(x: np.ndarray, nearest: bool = False) -> np.ndarray:
    """codes of quantize_bp8 on float64 input (the reference's own dtype)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    codes = np.empty(x.shape, np.uint8)
    lib().orc_quantize_bp8_f64(_p(x), x.size, int(bool(nearest)), _p(codes))
    return codes


def encode_bp16(x: np.ndarray, rtne: bool = True) -> np.ndarray:
    """encode_bposit16(Fraction(float(x)), "rtne"|"truncate")
    (reference/bposit_ref.py:382-507)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_encode_bp16(_p(x), x.size, int(bool(rtne)), _p(out))
    return out


def quire_to_bp32(limbs: np.ndarray) -> np.ndarray:
    """quire256_to_bposit32 (reference/bposit_ref.py:703-722) over [n, nlimbs]
    little-endian uint32 two's-complement limbs."""
    limbs = np.ascontiguousarray(limbs, dtype=np.uint32)
    n, nl = limbs.shape
    out = np.empty(n, np.uint32)
    lib().orc_quire_to_bp32_batch(_p(limbs), nl, n, _p(out))
    return out


def quire_to_bp16(limbs: np.ndarray) -> np.ndarray:
    """quire256_to_bposit16 (reference/bposit_ref.py:620-635) over [n, nlimbs]
    little-endian uint32 two's-complement limbs."""
    limbs = np.ascontiguousarray(limbs, dtype=np.uint32)
    n, nl = limbs.shape
    out = np.empty(n, np.uint16)
    lib().orc_quire_to_bp16_batch(_p(limbs), nl, n, _p(out))
    return out


def quantize_small(x: np.ndarray, nbits: int) -> np.ndarray:
    """Truncating float64 -> bposit4 (nbits 4) / AI-posit5 (nbits 5) codes, one per
    byte (encode_bposit4 / encode_aiposit5, reference/bposit_ref.py:806-925)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    out = np.empty(x.shape, np.uint8)
    lib().orc_quantize_small(nbits, _p(x), x.size, _p(out))
    return out


def transcode(codes: np.ndarray, fmt_in: int, fmt_out: int) -> np.ndarray:
    """Codes of fmt_in (4, 5 or 8 bits, one per byte) to the fmt_out (8 or 16)
    codes of the same values (exact; NaR -> NaR)."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(c.shape, np.uint8 if fmt_out == 8 else np.uint16)
    lib().orc_transcode(fmt_in, fmt_out, _p(c), c.size, _p(out))
    return out


def group_scales(x: np.ndarray, group: int = 128, maxpos_log2: int = 24) -> np.ndarray:
    """Per-(row, group) exponent ceil(log2(absmax / 2^maxpos_log2)); 0 for an
    all-zero group."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, K = x.shape
    G = (K + group - 1) // group
    s = np.empty((rows, G), np.int32)
    lib().orc_group_scales(_p(x), rows, K, group, maxpos_log2, _p(s))
    return s


def quantize_bp8_grouped(x: np.ndarray, s: np.ndarray, group: int = 128, nearest: bool = True):
    """codes of quantize_bp8(x / 2^s[row, k // group], nearest)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    s = np.ascontiguousarray(s, dtype=np.int32)
    rows, K = x.shape
    codes = np.empty((rows, K), np.uint8)
    lib().orc_quantize_bp8_grouped(_p(x), rows, K, group, _p(s), int(bool(nearest)), _p(codes))
    return codes


def quire_gemm(A: np.ndarray, B: np.ndarray, fmt_bits: int = 8, sa=None, sb=None, group: int = 128,
               nlimbs: int = 0, nthreads: int | None = None):
    """Exact quire GEMM A[M,K] @ B[N,K]^T with dot_at_precision's per-term rule
    (reference/bposit_ref.py:1028-1035) evaluated by shift classes as
    bposit_fast.dot_quire / matmul_quire do (reference/bposit_fast.py:102-176),
    plus optional per-group power-of-two exponents.  Returns bp32 codes [M,N]
    (quire256_to_bposit32), and the raw quires as [M,N,nlimbs] uint32 limbs
    when nlimbs > 0."""
    dt = np.uint8 if fmt_bits == 8 else np.uint16
    A = np.ascontiguousarray(A, dtype=dt)
    B = np.ascontiguousarray(B, dtype=dt)
    M, K = A.shape
    N = B.shape[0]
    sa_ = None if sa is None else np.ascontiguousarray(sa, dtype=np.int32)
    sb_ = None if sb is None else np.ascontiguousarray(sb, dtype=np.int32)
    out = np.empty((M, N), np.uint32)
    q = np.empty((M, N, nlimbs), np.uint32) if nlimbs else None
    if nthreads is None:
        nthreads = max(1, len(os.sched_getaffinity(0)))
    rc = lib().orc_quire_gemm(fmt_bits, _p(A), _p(B), M, N, K, _p(sa_), _p(sb_), group,
                              _p(out), _p(q), nlimbs, nthreads)
    if rc != 0:
        raise ValueError("oracle quire_gemm: bad arguments")
    return (out, q) if nlimbs else out


def bp32_to_double(codes: np.ndarray) -> np.ndarray:
    """bposit32 -> float64 (decode_bposit32 + decoded_to_fraction_32,
    reference/bposit_ref.py:43-94); NaR -> NaN."""
    c = np.ascontiguousarray(codes, dtype=np.uint32)
    out = np.empty(c.shape, np.float64)
    lib().orc_bp32_to_double_batch(_p(c), c.size, _p(out))
    return out


def encode_bp8_exact(x: float) -> int:
    """encode_bposit8 on the exact value of x (reference/bposit_ref.py:216-270
    without the float entry's limit_denominator)."""
    return int(lib().orc_encode_bp8_exact(float(x)))


# ---- python-int helpers for quires ------------------------------------------
def int_to_limbs(q: int, nlimbs: int) -> np.ndarray:
    v = q & ((1 << (32 * nlimbs)) - 1)
    return np.array([(v >> (32 * i)) & 0xFFFFFFFF for i in range(nlimbs)], dtype=np.uint32)


def limbs_to_int(limbs) -> int:
    nl = len(limbs)
    v = 0
    for i in range(nl - 1, -1, -1):
        v = (v << 32) | int(limbs[i])
    if v >> (32 * nl - 1):
        v -= 1 << (32 * nl)
    return v
