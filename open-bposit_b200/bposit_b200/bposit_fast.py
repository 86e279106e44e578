"""Drop-in for the reference's numpy fast path (reference/bposit_fast.py) on a
B200: the same function names, argument meaning, return types and errors,
computed by the library's sm_100a kernels.

    import bposit_fast as bf                      # reference
    from bposit_b200 import bposit_fast as bf     # this library

Inputs may be numpy arrays / lists (copied to the current CUDA device, results
returned as numpy / Python ints like the reference) or CUDA tensors (kept on
the device, except where the reference returns Python ints).  Formats: the
reference's "bp4", "aip5" and "bp8", plus "bp16".  Every bp4 / AI-posit5 value
is a bp8 value, so those codes are widened to bp8 on the device (exactly) and
go through the bp8 quire GEMM; the quires are the same numbers.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops

QUIRE_FRAC_BITS = 96
_NBITS = {"bp4": 4, "aip5": 5, "bp8": 8, "bp16": 16}


def _nbits(fmt: str) -> int:
    try:
        return _NBITS[fmt]
    except KeyError:
        raise KeyError(fmt) from None


def _device():
    return torch.device("cuda", torch.cuda.current_device())


def _gemm_bits(nb: int) -> int:
    """The quire-GEMM format that carries codes of nb bits (bp4 / aip5 -> bp8)."""
    return 8 if nb <= 8 else 16


def _codes_to_dev(c, nb: int) -> torch.Tensor:
    """Codes (any integer array-like or CUDA tensor) masked to nb bits, on the
    device in the GEMM format (_gemm_bits)."""
    dt = torch.uint8 if nb <= 8 else torch.uint16
    if isinstance(c, torch.Tensor) and c.is_cuda:
        t = c.contiguous() if c.dtype == dt and nb in (8, 16) else (c.to(torch.int64) & ((1 << nb) - 1)).to(dt)
    else:
        a = np.asarray(c, dtype=np.int64) & ((1 << nb) - 1)      # the reference's `& mask`
        a = a.astype(np.uint8 if nb <= 8 else np.uint16)
        t = torch.from_numpy(np.ascontiguousarray(a)).to(_device())
    return ops.transcode(t, nb, 8) if nb < 8 else t


def _limbs_to_ints(q: np.ndarray) -> np.ndarray:
    """[..., nl] uint32 two's complement limbs -> object array of Python ints."""
    shape = q.shape[:-1]
    flat = np.ascontiguousarray(q).reshape(-1, q.shape[-1])
    out = np.empty(flat.shape[0], dtype=object)
    for i in range(flat.shape[0]):
        out[i] = int.from_bytes(flat[i].tobytes(), "little", signed=True)
    return out.reshape(shape)


def _broadcast(a: torch.Tensor, b: torch.Tensor):
    """numpy broadcasting of the reference's elementwise `mant[a] * mant[b]`."""
    ka, kb = a.shape[1], b.shape[1]
    if ka == kb:
        return a, b
    if ka == 1:
        return a.expand(1, kb).contiguous(), b
    if kb == 1:
        return a, b.expand(1, ka).contiguous()
    raise ValueError(f"operands could not be broadcast together with shapes ({ka},) ({kb},)")


def quantize_bp8(x, *, nearest: bool = False):
    """bposit8 quantize -> dequantize of every element of x (reference/bposit_fast.py:69-99):
    nearest=False keeps the largest grid magnitude <= |x| (bit-identical to the
    reference's truncating encode for |x| >= minpos), nearest=True rounds to the
    nearest grid value with ties to the smaller magnitude; nonzero values below
    minpos go to +-minpos.  Returns float64 values (numpy for array input, a
    CUDA tensor for CUDA tensor input)."""
    if isinstance(x, torch.Tensor) and x.is_cuda:
        xx = x if x.dtype in (torch.float32, torch.float64) else x.to(torch.float64)
        _, v = ops.quantize_bp8(xx, nearest=nearest, return_values=True)
        return v.to(torch.float64)
    xa = np.asarray(x, dtype=np.float64)
    xt = torch.from_numpy(np.ascontiguousarray(xa)).to(_device())
    _, v = ops.quantize_bp8(xt, nearest=nearest, return_values=True)
    return v.cpu().numpy().reshape(xa.shape)


def quantize_bp8_codes(x, *, nearest: bool = True):
    """The bp8 codes of quantize_bp8(x, nearest=...) (the value->code map of
    examples/w8a8_rounding_demo.py:30-31, 47-49): uint8, same shape."""
    if isinstance(x, torch.Tensor) and x.is_cuda:
        return ops.quantize_bp8(x if x.dtype in (torch.float32, torch.float64) else x.to(torch.float64),
                                nearest=nearest)
    xa = np.asarray(x, dtype=np.float64)
    xt = torch.from_numpy(np.ascontiguousarray(xa)).to(_device())
    return ops.quantize_bp8(xt, nearest=nearest).cpu().numpy().reshape(xa.shape)


def dot_quire(a_codes, b_codes, fmt: str) -> int:
    """Exact quire (integer, 96 fraction bits) of the dot of two code vectors
    (reference/bposit_fast.py:102-128)."""
    nb = _nbits(fmt)
    a = _codes_to_dev(a_codes, nb).reshape(1, -1)
    b = _codes_to_dev(b_codes, nb).reshape(1, -1)
    a, b = _broadcast(a, b)
    _, q = ops.quire_gemm(a, b, _gemm_bits(nb), quire_limbs=16)
    return int(_limbs_to_ints(ops.to_host(q))[0, 0])


_OUT_FMTS = ("bp16", "bp32")   # reference/bposit_ref.py:989-992


def dot(a_codes, b_codes, fmt: str, out_fmt: str = "bp32") -> int:
    """Exact dot rounded once to out_fmt, "bp32" or "bp16"
    (reference/bposit_fast.py:131-133)."""
    if out_fmt not in _OUT_FMTS:
        raise KeyError(out_fmt)
    nb = _nbits(fmt)
    a = _codes_to_dev(a_codes, nb).reshape(1, -1)
    b = _codes_to_dev(b_codes, nb).reshape(1, -1)
    a, b = _broadcast(a, b)
    out, _ = ops.quire_gemm(a, b, _gemm_bits(nb))
    if out_fmt == "bp16":
        out = ops.bp32_to_bp16(out)
    return int(ops.to_host(out)[0, 0])


def matmul_quire(A_codes, B_codes, fmt: str):
    """Exact quire of every output of A[T,K] @ B[N,K]^T as a [T,N] object
    array of Python ints (reference/bposit_fast.py:136-176)."""
    nb = _nbits(fmt)
    if np.ndim(A_codes) != 2 or np.ndim(B_codes) != 2:
        raise ValueError("matmul_quire expects A[T,K] and B[N,K]")
    A = _codes_to_dev(A_codes, nb)
    B = _codes_to_dev(B_codes, nb)
    _, q = ops.quire_gemm(A, B, _gemm_bits(nb), quire_limbs=16)
    return _limbs_to_ints(ops.to_host(q))


def matmul_bp16(A_codes, B_codes, fmt: str = "bp8", *, a_exps=None, b_exps=None, group: int = 128,
                algo: int = 0):
    """As matmul_bp32, every output rounded once to bposit16 instead
    (quire256_to_bposit16, reference/bposit_ref.py:620-635).  uint16 codes."""
    out = matmul_bp32(A_codes, B_codes, fmt, a_exps=a_exps, b_exps=b_exps, group=group, algo=algo)
    on_dev = isinstance(out, torch.Tensor)
    r = ops.bp32_to_bp16(out if on_dev else torch.from_numpy(out).to(_device()))
    return r if on_dev else ops.to_host(r)


def matmul_bp32(A_codes, B_codes, fmt: str = "bp8", *, a_exps=None, b_exps=None, group: int = 128,
                algo: int = 0):
    """A[T,K] @ B[N,K]^T with every output rounded once to bposit32 (the
    reference's matmul_quire followed by quire256_to_bposit32 per element), with
    optional per-(row, group) power-of-two exponents.  Returns uint32 codes
    (numpy for host input, a CUDA tensor for CUDA input)."""
    nb = _nbits(fmt)
    on_dev = isinstance(A_codes, torch.Tensor) and A_codes.is_cuda
    A = _codes_to_dev(A_codes, nb)
    B = _codes_to_dev(B_codes, nb)
    sa = None if a_exps is None else torch.as_tensor(a_exps, dtype=torch.int32).to(A.device).contiguous()
    sb = None if b_exps is None else torch.as_tensor(b_exps, dtype=torch.int32).to(A.device).contiguous()
    out, _ = ops.quire_gemm(A, B, _gemm_bits(nb), sa=sa, sb=sb, group=group, algo=algo)
    return out if on_dev else ops.to_host(out)
