"""Device-level API: torch CUDA tensors in, torch CUDA tensors out, zero copy.

Each op launches the library's sm_100a kernels through the C ABI on the
current torch stream.  Codes are uint8 (bp8), uint16 (bp16) and uint32
(bposit32) tensors; quires are [..., nlimbs] uint32 two's-complement limbs with
96 fraction bits.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_FMT = {"bp8": 8, "bp16": 16, 8: 8, 16: 16}
_CODE_DTYPE = {8: torch.uint8, 16: torch.uint16}


def device_error() -> int:
    """Read and clear the current device's kernel error word (synchronizes with
    the device): nonzero when a bounded wait inside a tensor-core GEMM gave up.
    While the word is set, every bposit32 output of the tensor-core path is NaR
    (0x80000000), a code no quire round produces."""
    v = ctypes.c_int(0)
    _lib.check(_lib.lib().bp_device_error(ctypes.byref(v)))
    return int(v.value)


def check_device_error() -> None:
    """Raise BpositError if a tensor-core GEMM gave up on a bounded wait since
    the last check (the word is cleared by the check)."""
    v = device_error()
    if v:
        raise _lib.BpositError(_lib.BP_ECUDA, f"a tensor-core GEMM gave up on a bounded wait (error word {v:#x}); "
                                              "its bposit32 outputs were set to NaR")


def to_host(t: torch.Tensor):
    """t as a numpy array, once the device work behind it is done and no GEMM
    reported a timed-out wait (check_device_error)."""
    a = t.cpu().numpy()
    check_device_error()
    return a


def fmt_bits(fmt) -> int:
    try:
        return _FMT[fmt]
    except KeyError:
        raise KeyError(fmt) from None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dev(t: torch.Tensor, name: str, dtype=None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    return t.contiguous()


def decode(codes: torch.Tensor, fmt=None) -> torch.Tensor:
    """code -> exact fp32 value (zero and NaR -> 0)."""
    f = fmt_bits(fmt) if fmt is not None else (8 if codes.dtype == torch.uint8 else 16)
    c = _dev(codes, "codes", _CODE_DTYPE[f])
    out = torch.empty(c.shape, dtype=torch.float32, device=c.device)
    _lib.check(_lib.lib().bp_decode(f, _p(c), c.numel(), _p(out), _stream()))
    return out


def quantize_bp8(x: torch.Tensor, nearest: bool = True, return_values: bool = False, out=None):
    """fp32 (or float64) -> bp8 codes; with return_values also the exact values
    (fp32 for fp32 input, float64 for float64 input)."""
    if x.dtype == torch.float64:
        xx = _dev(x, "x")
        codes = out if out is not None else torch.empty(xx.shape, dtype=torch.uint8, device=xx.device)
        vals = torch.empty(xx.shape, dtype=torch.float64, device=xx.device) if return_values else None
        _lib.check(_lib.lib().bp_quantize_bp8_f64(_p(xx), xx.numel(), int(nearest), _p(codes), _p(vals),
                                                  _stream()))
        return (codes, vals) if return_values else codes
    xx = _dev(x, "x", torch.float32)
    codes = out if out is not None else torch.empty(xx.shape, dtype=torch.uint8, device=xx.device)
    vals = torch.empty(xx.shape, dtype=torch.float32, device=xx.device) if return_values else None
    _lib.check(_lib.lib().bp_quantize_bp8(_p(xx), xx.numel(), int(nearest), _p(codes), _p(vals), _stream()))
    return (codes, vals) if return_values else codes


def quantize_bp8_grouped(x: torch.Tensor, group: int = 128, nearest: bool = True, exps=None,
                         maxpos_log2: int = 24, out=None):
    """Row-wise grouped quantization of x[rows, K]: returns (codes[rows, K],
    exps[rows, ceil(K/group)] int32).  When exps is None the power-of-two
    exponents ceil(log2(absmax / 2^maxpos_log2)) are computed."""
    xx = _dev(x, "x", torch.float32)
    if xx.dim() != 2:
        raise ValueError("x must be 2-D [rows, K]")
    rows, K = xx.shape
    G = (K + group - 1) // group
    compute = exps is None
    e = torch.empty((rows, G), dtype=torch.int32, device=xx.device) if compute else _dev(exps, "exps", torch.int32)
    codes = out if out is not None else torch.empty((rows, K), dtype=torch.uint8, device=xx.device)
    _lib.check(_lib.lib().bp_quantize_bp8_grouped(_p(xx), rows, K, group, int(nearest), int(compute),
                                                  maxpos_log2, _p(e), _p(codes), _stream()))
    return codes, e


def encode_bp16(x: torch.Tensor, rtne: bool = True, out=None) -> torch.Tensor:
    xx = _dev(x, "x", torch.float32)
    codes = out if out is not None else torch.empty(xx.shape, dtype=torch.uint16, device=xx.device)
    _lib.check(_lib.lib().bp_encode_bp16(_p(xx), xx.numel(), int(rtne), _p(codes), _stream()))
    return codes


def quire_to_bp32(limbs: torch.Tensor) -> torch.Tensor:
    """[..., nlimbs] uint32 quires (nlimbs 8, 12 or 16) -> [...] bp32 codes."""
    q = _dev(limbs, "limbs", torch.uint32)
    nl = q.shape[-1]
    out = torch.empty(q.shape[:-1], dtype=torch.uint32, device=q.device)
    _lib.check(_lib.lib().bp_quire_to_bp32(_p(q), nl, out.numel(), _p(out), _stream()))
    return out


def w8a8_encode_rows(x: torch.Tensor):
    """The reference W8A8 recipe's activation side for x[rows, K] (fp32): per-row
    exponents (recommended_exponents, float64 on the device) and the truncating
    bp8 codes of x / 2^e.  Returns (codes [rows, K] uint8, exps [rows] int32)."""
    xx = _dev(x, "x", torch.float32)
    if xx.dim() != 2:
        raise ValueError("x must be 2-D [rows, K]")
    rows, K = xx.shape
    codes = torch.empty((rows, K), dtype=torch.uint8, device=xx.device)
    exps = torch.empty(rows, dtype=torch.int32, device=xx.device)
    _lib.check(_lib.lib().bp_w8a8_encode_rows(_p(xx), rows, K, _p(exps), _p(codes), _stream()))
    return codes, exps


def quantize_small(x: torch.Tensor, fmt) -> torch.Tensor:
    """Truncating float64 -> bposit4 ("bp4"/4) or AI-posit5 ("aip5"/5) codes, uint8."""
    f = {"bp4": 4, "aip5": 5, 4: 4, 5: 5}.get(fmt)
    if f is None:
        raise KeyError(fmt)
    xx = _dev(x, "x", torch.float64)
    codes = torch.empty(xx.shape, dtype=torch.uint8, device=xx.device)
    _lib.check(_lib.lib().bp_quantize_small(f, _p(xx), xx.numel(), _p(codes), _stream()))
    return codes


def transcode(codes: torch.Tensor, fmt_in, fmt_out) -> torch.Tensor:
    """Exact widening of codes: bp4 / aip5 (uint8, one code per byte) or bp8 to
    bp8 (uint8) or bp16 (uint16); NaR -> NaR."""
    fi = {"bp4": 4, "aip5": 5, "bp8": 8, 4: 4, 5: 5, 8: 8}.get(fmt_in)
    fo = {"bp8": 8, "bp16": 16, 8: 8, 16: 16}.get(fmt_out)
    if fi is None or fo is None or fo <= fi:
        raise KeyError(f"{fmt_in} -> {fmt_out}")
    c = _dev(codes, "codes", torch.uint8)
    out = torch.empty(c.shape, dtype=torch.uint8 if fo == 8 else torch.uint16, device=c.device)
    _lib.check(_lib.lib().bp_transcode(fi, fo, _p(c), c.numel(), _p(out), _stream()))
    return out


def quire_to_bp16(limbs: torch.Tensor) -> torch.Tensor:
    """[..., nlimbs] quire limbs -> bposit16 codes (quire256_to_bposit16)."""
    q = _dev(limbs, "limbs", torch.uint32)
    nl = q.shape[-1]
    out = torch.empty(q.shape[:-1], dtype=torch.uint16, device=q.device)
    _lib.check(_lib.lib().bp_quire_to_bp16(_p(q), nl, out.numel(), _p(out), _stream()))
    return out


def bp32_to_bp16(codes: torch.Tensor) -> torch.Tensor:
    """bposit32 codes of quire rounds -> the bposit16 rounds of the same quires."""
    c = _dev(codes, "codes", torch.uint32)
    out = torch.empty(c.shape, dtype=torch.uint16, device=c.device)
    _lib.check(_lib.lib().bp_bp32_to_bp16(_p(c), c.numel(), _p(out), _stream()))
    return out


def gemm_workspace_size(fmt, M: int, N: int, K: int, algo: int = 0) -> int:
    return int(_lib.lib().bp_quire_gemm_workspace_size(fmt_bits(fmt), M, N, K, algo))


def quire_gemm(A: torch.Tensor, B: torch.Tensor, fmt=None, sa=None, sb=None, group: int = 128,
               out=None, quire_limbs: int = 0, algo: int = 0, workspace=None):
    """Exact quire GEMM A[M,K] @ B[N,K]^T -> (bp32 codes [M,N], raw quires
    [M,N,quire_limbs] or None).  `out` may be a [M, ldo >= N] uint32 view (a
    column block of a wider matrix is allowed: its row stride is used)."""
    f = fmt_bits(fmt) if fmt is not None else (8 if A.dtype == torch.uint8 else 16)
    a = _dev(A, "A", _CODE_DTYPE[f])
    b = _dev(B, "B", _CODE_DTYPE[f])
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("quire_gemm expects A[M,K] and B[N,K]")
    M, K = a.shape
    N, K2 = b.shape
    if K2 != K:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    sa_ = None if sa is None else _dev(sa, "sa", torch.int32)
    sb_ = None if sb is None else _dev(sb, "sb", torch.int32)
    if out is None:
        out = torch.empty((M, N), dtype=torch.uint32, device=a.device)
        ldo = N
    else:
        if out.dtype != torch.uint32 or out.shape != (M, N) or out.stride(1) != 1:
            raise ValueError("out must be a [M, N] uint32 view with unit column stride")
        ldo = out.stride(0)
    q = torch.empty((M, N, quire_limbs), dtype=torch.uint32, device=a.device) if quire_limbs else None
    need = gemm_workspace_size(f, M, N, K, algo)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=a.device)
    _lib.check(_lib.lib().bp_quire_gemm(f, _p(a), _p(b), M, N, K, _p(sa_), _p(sb_), group, _p(out), ldo,
                                        _p(q), quire_limbs, algo, _p(workspace), workspace.numel(),
                                        _stream()))
    return out, q


def quire_gemm_f32(A: torch.Tensor, B: torch.Tensor, fmt=None, sa=None, sb=None, group: int = 128,
                   row_exp=None, col_exp=None, bias=None, out=None, out_bp32=None, algo: int = 0,
                   workspace=None) -> torch.Tensor:
    """Exact quire GEMM A[M,K] @ B[N,K]^T whose output stage writes the fp32
    hand-off directly: value(bposit32) * 2^(row_exp[m] + col_exp[n]) + bias[n],
    rounded once to fp32 -- the numbers of quire_gemm followed by bp32_to_f32.
    `out` (optional) is a [M, N] float32 view with unit column stride;
    `out_bp32` (optional) also receives the bposit32 codes."""
    f = fmt_bits(fmt) if fmt is not None else (8 if A.dtype == torch.uint8 else 16)
    a = _dev(A, "A", _CODE_DTYPE[f])
    b = _dev(B, "B", _CODE_DTYPE[f])
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("quire_gemm_f32 expects A[M,K] and B[N,K]")
    M, K = a.shape
    N = b.shape[0]
    sa_ = None if sa is None else _dev(sa, "sa", torch.int32)
    sb_ = None if sb is None else _dev(sb, "sb", torch.int32)
    re = None if row_exp is None else _dev(row_exp, "row_exp", torch.int32)
    ce = None if col_exp is None else _dev(col_exp, "col_exp", torch.int32)
    bs = None if bias is None else _dev(bias, "bias", torch.float32)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    elif out.dtype != torch.float32 or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out must be a [M, N] float32 view with unit column stride")
    ldo = 0
    if out_bp32 is not None:
        if out_bp32.dtype != torch.uint32 or out_bp32.shape != (M, N) or out_bp32.stride(1) != 1:
            raise ValueError("out_bp32 must be a [M, N] uint32 view with unit column stride")
        ldo = out_bp32.stride(0)
    need = gemm_workspace_size(f, M, N, K, algo)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=a.device)
    _lib.check(_lib.lib().bp_quire_gemm_f32(f, _p(a), _p(b), M, N, K, _p(sa_), _p(sb_), group, _p(re), _p(ce),
                                            _p(bs), _p(out), out.stride(0), _p(out_bp32), ldo, algo,
                                            _p(workspace), workspace.numel(), _stream()))
    return out


def quire_gemm_host(A, B, fmt=None, sa=None, sb=None, group: int = 128, out=None, algo: int = 0):
    """Exact quire GEMM on host arrays (CPU tensors or numpy; page-locked CPU
    tensors copy fastest): the library sends one operand whole and streams the
    other in row chunks (A when M >= N, so that each chunk's results leave in
    one contiguous copy; else B), overlapping the copies with the tensor-core
    work.  Returns the [M, N] uint32 bposit32 codes as a CPU tensor (`out`, if
    given; its rows may be strided), complete once the current CUDA stream is
    synchronized."""
    def host(x, dtype):
        t = torch.as_tensor(x)
        if t.is_cuda:
            raise ValueError("quire_gemm_host takes host arrays")
        return t.contiguous() if t.dtype == dtype else t.to(dtype).contiguous()
    f = fmt_bits(fmt) if fmt is not None else (8 if torch.as_tensor(A).dtype == torch.uint8 else 16)
    a = host(A, _CODE_DTYPE[f])
    b = host(B, _CODE_DTYPE[f])
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("quire_gemm_host expects A[M,K] and B[N,K]")
    M, K = a.shape
    N = b.shape[0]
    sa_ = None if sa is None else host(sa, torch.int32)
    sb_ = None if sb is None else host(sb, torch.int32)
    if out is None:
        out = torch.empty((M, N), dtype=torch.uint32, pin_memory=True)
    elif out.is_cuda or out.dtype != torch.uint32 or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out must be a host [M, N] uint32 tensor with unit column stride")
    _lib.check(_lib.lib().bp_quire_gemm_host(f, a.data_ptr(), b.data_ptr(), M, N, K,
                                             None if sa_ is None else sa_.data_ptr(),
                                             None if sb_ is None else sb_.data_ptr(), group,
                                             out.data_ptr(), out.stride(0), algo, _stream()))
    return out


def quire_gemm_multi(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor, peer_ptrs, peer_col0: int,
                     fmt=None, sa=None, sb=None, group: int = 128, algo: int = 0, workspace=None):
    """quire_gemm whose bp32 results are also stored into every matrix in
    `peer_ptrs` (device addresses of [M, ldo] uint32 matrices, normally other
    GPUs' result buffers) at column `peer_col0`, by the GEMM's finish kernel itself.
    `out` is this rank's [M, N] column block (row stride ldo)."""
    f = fmt_bits(fmt) if fmt is not None else (8 if A.dtype == torch.uint8 else 16)
    a = _dev(A, "A", _CODE_DTYPE[f])
    b = _dev(B, "B", _CODE_DTYPE[f])
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("quire_gemm_multi expects A[M,K] and B[N,K]")
    M, K = a.shape
    N = b.shape[0]
    if out.dtype != torch.uint32 or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out must be a [M, N] uint32 view with unit column stride")
    sa_ = None if sa is None else _dev(sa, "sa", torch.int32)
    sb_ = None if sb is None else _dev(sb, "sb", torch.int32)
    ptrs = (ctypes.c_void_p * max(1, len(peer_ptrs)))(*[int(x) for x in peer_ptrs])
    need = gemm_workspace_size(f, M, N, K, algo)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=a.device)
    _lib.check(_lib.lib().bp_quire_gemm_multi(f, _p(a), _p(b), M, N, K, _p(sa_), _p(sb_), group, _p(out),
                                              out.stride(0), ptrs, len(peer_ptrs), peer_col0, algo,
                                              _p(workspace), workspace.numel(), _stream()))
    return out


def enable_peer_access(peer_device: int) -> None:
    """Let the current device read and write `peer_device`'s memory directly."""
    _lib.check(_lib.lib().bp_enable_peer_access(int(peer_device)))


IPC_HANDLE_BYTES = 64


class _DeviceBuffer:
    """__cuda_array_interface__ view of memory the library allocated (no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 2, "strides": None}


def ipc_alloc(shape, device) -> tuple[torch.Tensor, bytes, int]:
    """Zeroed uint32 tensor in memory that other processes can map (CUDA IPC):
    (tensor, handle, device address).  The tensor does not own the memory;
    release it with ipc_free(address) once no process uses it."""
    numel = 1
    for d in shape:
        numel *= int(d)
    with torch.cuda.device(device):
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _lib.check(_lib.lib().bp_ipc_alloc(max(4, numel * 4), ctypes.byref(ptr), handle))
        t = torch.as_tensor(_DeviceBuffer(ptr.value, shape, "<i4"), device=device).view(torch.uint32)
    return t, handle.raw, int(ptr.value)


def ipc_free(ptr: int) -> None:
    _lib.check(_lib.lib().bp_ipc_free(ctypes.c_void_p(ptr)))


def ipc_open(handle: bytes) -> int:
    """Map another process's ipc_alloc memory into the current device's
    context; returns its device address here."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("bad IPC handle")
    ptr = ctypes.c_void_p()
    _lib.check(_lib.lib().bp_ipc_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr)))
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _lib.check(_lib.lib().bp_ipc_close(ctypes.c_void_p(ptr)))


def bp32_to_f32(codes: torch.Tensor, row_exp=None, col_exp=None, bias=None, out=None) -> torch.Tensor:
    """[M,N] bp32 codes -> fp32 of value * 2^(row_exp[m] + col_exp[n]) + bias[n],
    rounded once (nearest-even) from the exact value."""
    c = _dev(codes, "codes", torch.uint32)
    if c.dim() != 2:
        raise ValueError("codes must be [M, N]")
    M, N = c.shape
    re = None if row_exp is None else _dev(row_exp, "row_exp", torch.int32)
    ce = None if col_exp is None else _dev(col_exp, "col_exp", torch.int32)
    b = None if bias is None else _dev(bias, "bias", torch.float32)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=c.device)
    elif out.dtype != torch.float32 or out.shape != (M, N) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [M, N] float32 tensor")
    _lib.check(_lib.lib().bp_bp32_to_f32(_p(c), M, N, _p(re), _p(ce), _p(b), _p(out), _stream()))
    return out


def bp32_to_f64(codes: torch.Tensor, row_exp=None, col_exp=None) -> torch.Tensor:
    """[M, N] bp32 codes -> float64 values * 2^(row_exp[m] + col_exp[n])."""
    c = _dev(codes, "codes", torch.uint32)
    if c.dim() == 1:
        c = c.view(1, -1)
    M, N = c.shape
    re = None if row_exp is None else _dev(row_exp, "row_exp", torch.int32)
    ce = None if col_exp is None else _dev(col_exp, "col_exp", torch.int32)
    out = torch.empty((M, N), dtype=torch.float64, device=c.device)
    _lib.check(_lib.lib().bp_bp32_to_f64(_p(c), M, N, _p(re), _p(ce), _p(out), _stream()))
    return out
