"""The hot-path subset of the reference's format module (reference/bposit_ref.py)
as vectorised device calls: code values, the bp16 encoder and the single
quire -> bposit32 round.  Scalar inputs return scalars, arrays return arrays.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops

QUIRE_FRAC_BITS = 96   # reference/bposit_ref.py:541
QUIRE_BITS = 256


def _device():
    return torch.device("cuda", torch.cuda.current_device())


def code_value(code, fmt: str):
    """Exact value of bp8 / bp16 code(s), 0 for zero and NaR
    (reference/bposit_ref.py:1022-1025), as float (exact)."""
    nb = {"bp8": 8, "bp16": 16}.get(fmt)
    if nb is None:
        raise KeyError(fmt)
    a = np.asarray(np.asarray(code, dtype=np.int64) & ((1 << nb) - 1))
    t = torch.from_numpy(np.ascontiguousarray(a.astype(np.uint8 if nb == 8 else np.uint16)).reshape(a.shape)).to(_device())
    v = ops.decode(t, nb).cpu().numpy().astype(np.float64)
    return float(v) if v.ndim == 0 else v


def encode_bposit16(value, mode: str = "truncate"):
    """encode_bposit16 on the exact value of fp32 input(s) (reference/bposit_ref.py:489-507
    with Fraction(x)); mode "truncate" or "rtne"."""
    if mode not in ("truncate", "rtne"):
        raise ValueError(f"unknown rounding mode: {mode!r}")
    a = np.asarray(value, dtype=np.float32)
    t = torch.from_numpy(np.ascontiguousarray(a).reshape(a.shape)).to(_device())
    c = ops.encode_bp16(t, rtne=(mode == "rtne")).cpu().numpy()
    return int(c) if c.ndim == 0 else c


def _ints_to_limbs(qs, nl: int = 16) -> np.ndarray:
    out = np.empty((len(qs), nl), dtype=np.uint32)
    for i, q in enumerate(qs):
        out[i] = np.frombuffer((int(q) & ((1 << (32 * nl)) - 1)).to_bytes(4 * nl, "little"), dtype=np.uint32)
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
