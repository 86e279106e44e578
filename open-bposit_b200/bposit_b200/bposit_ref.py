"""The hot-path subset of the reference's format module (reference/bposit_ref.py)
as vectorised device calls: code values, the bp16 encoder and the single
quire -> bposit32 round.  Scalar inputs return scalars, arrays return arrays.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from .bposit_quantize import _LIMIT_ZERO

QUIRE_FRAC_BITS = 96   # reference/bposit_ref.py:541
QUIRE_BITS = 256


def _device():
    return torch.device("cuda", torch.cuda.current_device())


_RUNG_BITS = {"bp4": 4, "aip5": 5, "bp8": 8, "bp16": 16}


def _codes_dev(code, nb: int) -> torch.Tensor:
    """Code(s) masked to nb bits on the device, widened to bp8 for bp4 / aip5."""
    a = np.asarray(np.asarray(code, dtype=np.int64) & ((1 << nb) - 1))
    t = torch.from_numpy(np.ascontiguousarray(a.astype(np.uint8 if nb <= 8 else np.uint16)).reshape(a.shape))
    t = t.to(_device())
    return ops.transcode(t, nb, 8) if nb < 8 else t


def code_value(code, fmt: str):
    """Exact value of bp4 / aip5 / bp8 / bp16 code(s), 0 for zero and NaR
    (reference/bposit_ref.py:1022-1025), as float (exact)."""
    nb = _RUNG_BITS.get(fmt)
    if nb is None:
        raise KeyError(fmt)
    v = ops.decode(_codes_dev(code, nb), 8 if nb <= 8 else 16).cpu().numpy().astype(np.float64)
    return float(v) if v.ndim == 0 else v


def quantize_vec(vals, fmt: str) -> list:
    """Truncating encode of float values to bp4 / aip5 / bp8 codes
    (reference/bposit_ref.py:1017-1019, the encoders' float entries)."""
    x = torch.from_numpy(np.ascontiguousarray(np.asarray(vals, dtype=np.float64).ravel())).to(_device())
    if fmt in ("bp4", "aip5"):
        c = ops.quantize_small(x, fmt)
    elif fmt == "bp8":
        c = ops.quantize_bp8(x, nearest=False)
        c = torch.where(x.abs() <= _LIMIT_ZERO, torch.zeros_like(c), c)   # limit_denominator(10**8)
    else:
        raise KeyError(fmt)
    return [int(v) for v in c.cpu().numpy()]


def _round_out(q_bp32: torch.Tensor, out_fmt: str):
    if out_fmt == "bp32":
        return q_bp32
    if out_fmt == "bp16":
        return ops.bp32_to_bp16(q_bp32)
    raise KeyError(out_fmt)


def dot_at_precision(a_codes, b_codes, fmt: str, out_fmt: str = "bp32") -> int:
    """Exact dot of two code vectors of bp4 / aip5 / bp8, one quire, rounded once
    to out_fmt (reference/bposit_ref.py:1028-1035)."""
    nb = {"bp4": 4, "aip5": 5, "bp8": 8}.get(fmt)
    if nb is None:
        raise KeyError(fmt)
    a = _codes_dev(list(a_codes), nb).reshape(1, -1)
    b = _codes_dev(list(b_codes), nb).reshape(1, -1)
    n = min(a.shape[1], b.shape[1])                     # zip() semantics
    out, _ = ops.quire_gemm(a[:, :n].contiguous(), b[:, :n].contiguous(), 8)
    return int(ops.to_host(_round_out(out, out_fmt))[0, 0])


def mixed_precision_sum(items, out_fmt: str) -> int:
    """Exact sum of [(code, fmt), ...] over bp4 / aip5 / bp8 / bp16 in one quire,
    rounded once to out_fmt (reference/bposit_ref.py:995-1002): every item is
    widened to bp16 and the row is one bp16 quire dot against 1.0."""
    items = list(items)
    if not items:
        return 0
    dev = _device()
    fmts = [f for _, f in items]
    for f in set(fmts):
        if f not in _RUNG_BITS:
            raise KeyError(f)
    row = np.zeros(len(items), np.uint16)
    for f in set(fmts):
        nb = _RUNG_BITS[f]
        idx = np.array([i for i, g in enumerate(fmts) if g == f])
        c = np.array([int(items[i][0]) & ((1 << nb) - 1) for i in idx], np.int64)
        if nb == 16:
            row[idx] = c.astype(np.uint16)
        else:
            t = torch.from_numpy(c.astype(np.uint8)).to(dev)
            row[idx] = ops.transcode(t, nb, 16).cpu().numpy()
    ones = torch.full((1, len(items)), 0x4000, dtype=torch.uint16, device=dev)   # bp16 1.0
    out, _ = ops.quire_gemm(torch.from_numpy(row).to(dev).reshape(1, -1), ones, 16)
    return int(ops.to_host(_round_out(out, out_fmt))[0, 0])


def encode_bposit16(value, mode: str = "truncate"):
    """encode_bposit16 on the exact value of fp32 input(s) (reference/bposit_ref.py:489-507
    with Fraction(x)); mode "truncate" or "rtne"."""
    if mode not in ("truncate", "rtne"):
        raise ValueError(f"unknown rounding mode: {mode!r}")
    a = np.asarray(value, dtype=np.float32)
    t = torch.from_numpy(np.ascontiguousarray(a).reshape(a.shape)).to(_device())
    c = ops.encode_bp16(t, rtne=(mode == "rtne")).cpu().numpy()
    return int(c) if c.ndim == 0 else c


# |q| >= 2^(96 + 241) rounds to +-maxpos in both bposit32 and bposit16 (total
# exponent above 240, resp. 112: reference/bposit_ref.py:104-105, 416-419), so
# larger Python ints are clamped there before they are cut into 16 limbs.
_QUIRE_SAT = 1 << (96 + 241)


def _ints_to_limbs(qs, nl: int = 16) -> np.ndarray:
    out = np.empty((len(qs), nl), dtype=np.uint32)
    for i, q in enumerate(qs):
        q = int(q)
        if abs(q) >= _QUIRE_SAT:
            q = _QUIRE_SAT if q > 0 else -_QUIRE_SAT
        out[i] = np.frombuffer((q & ((1 << (32 * nl)) - 1)).to_bytes(4 * nl, "little"), dtype=np.uint32)
    return out


def quire256_to_bposit32(q):
    """Single round of exact quire(s) (Python ints, 96 fraction bits) to
    bposit32 (reference/bposit_ref.py:703-722)."""
    scalar = np.ndim(q) == 0
    qs = [q] if scalar else list(np.asarray(q, dtype=object).ravel())
    limbs = torch.from_numpy(_ints_to_limbs(qs)).to(_device())
    out = ops.quire_to_bp32(limbs).cpu().numpy()
    return int(out[0]) if scalar else out.reshape(np.shape(q))


def quire256_to_bposit16(q):
    """Single round of exact quire(s) (Python ints, 96 fraction bits) to
    bposit16, truncating (reference/bposit_ref.py:620-635)."""
    scalar = np.ndim(q) == 0
    qs = [q] if scalar else list(np.asarray(q, dtype=object).ravel())
    limbs = torch.from_numpy(_ints_to_limbs(qs)).to(_device())
    out = ops.quire_to_bp16(limbs).cpu().numpy()
    return int(out[0]) if scalar else out.reshape(np.shape(q))
