"""ctypes binding of libbposit_b200.so (the C ABI in include/bposit_b200.h).

The library is built in-tree (open-bposit_b200/Makefile) next to this file.
There is no fallback: if the library is missing or no sm_100 device is
present, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.path.join(_HERE, "libbposit_b200.so")
_PKG_ROOT = os.path.dirname(_HERE)

BP_OK = 0
BP_EINVAL = -1
BP_EFMT = -2
BP_EALIGN = -3
BP_ECUDA = -4
BP_ERANGE = -5
BP_ENODEV = -6
BP_EWORKSPACE = -7

_lock = threading.Lock()
_lib = None


class BpositError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (status {code})")
        self.code = code


def build(verbose: bool = False) -> str:
    """Compile the CUDA library with nvcc for sm_100a (make, in-tree)."""
    out = None if verbose else subprocess.DEVNULL
    subprocess.run(["make", "-s", "-j8", "-C", _PKG_ROOT], check=True, stdout=out)
    return SO_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(SO_PATH):
            raise RuntimeError(
                f"{SO_PATH} is missing: build it with `make -C {_PKG_ROOT}` "
                "(the b-posit ops have no CPU fallback)")
        L = ctypes.CDLL(SO_PATH)
        vp, sz, i32, i64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64
        sig = {
            "bp_version": ([], i32),
            "bp_last_error": ([], ctypes.c_char_p),
            "bp_launch_count": ([], ctypes.c_ulonglong),
            "bp_device_error": ([vp], i32),
            "bp_decode": ([i32, vp, sz, vp, vp], i32),
            "bp_quantize_bp8": ([vp, sz, i32, vp, vp, vp], i32),
            "bp_quantize_bp8_f64": ([vp, sz, i32, vp, vp, vp], i32),
            "bp_quantize_bp8_grouped": ([vp, i32, i32, i32, i32, i32, i32, vp, vp, vp], i32),
            "bp_encode_bp16": ([vp, sz, i32, vp, vp], i32),
            "bp_quire_to_bp32": ([vp, i32, sz, vp, vp], i32),
            "bp_quire_gemm": ([i32, vp, vp, i32, i32, i32, vp, vp, i32, vp, i64, vp, i32, i32,
                               vp, sz, vp], i32),
            "bp_quire_gemm_workspace_size": ([i32, i32, i32, i32, i32], sz),
            "bp_quire_gemm_f32": ([i32, vp, vp, i32, i32, i32, vp, vp, i32, vp, vp, vp, vp, i64, vp, i64, i32,
                                   vp, sz, vp], i32),
            "bp_quire_gemm_multi": ([i32, vp, vp, i32, i32, i32, vp, vp, i32, vp, i64, vp, i32, i64, i32,
                                     vp, sz, vp], i32),
            "bp_enable_peer_access": ([i32], i32),
            "bp_quire_to_bp16": ([vp, i32, sz, vp, vp], i32),
            "bp_quantize_small": ([i32, vp, sz, vp, vp], i32),
            "bp_bp32_to_f32": ([vp, i32, i32, vp, vp, vp, vp, vp], i32),
            "bp_quire_gemm_host": ([i32, vp, vp, i32, i32, i32, vp, vp, i32, vp, i64, i32, vp], i32),
            "bp_w8a8_encode_rows": ([vp, i32, i32, vp, vp, vp], i32),
            "bp_transcode": ([i32, i32, vp, sz, vp, vp], i32),
            "bp_bp32_to_bp16": ([vp, sz, vp, vp], i32),
            "bp_ipc_alloc": ([sz, vp, vp], i32),
            "bp_ipc_free": ([vp], i32),
            "bp_ipc_open": ([vp, vp], i32),
            "bp_ipc_close": ([vp], i32),
            "bp_quire_gemm_noalloc": ([i32, vp, vp, i32, i32, i32, vp, vp, i32, vp, i64, vp, i32, vp], i32),
            "bp_bp32_to_f64": ([vp, i32, i32, vp, vp, vp, vp], i32),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


EXPORTED = (
    "bp_version", "bp_last_error", "bp_launch_count", "bp_device_error", "bp_decode", "bp_quantize_bp8", "bp_quantize_bp8_f64",
    "bp_quantize_bp8_grouped", "bp_encode_bp16", "bp_quire_to_bp32", "bp_quire_to_bp16", "bp_bp32_to_bp16",
    "bp_quantize_small", "bp_transcode", "bp_bp32_to_f32", "bp_quire_gemm_host",
    "bp_w8a8_encode_rows",
    "bp_quire_gemm", "bp_quire_gemm_f32",
    "bp_quire_gemm_workspace_size", "bp_quire_gemm_multi", "bp_enable_peer_access",
    "bp_ipc_alloc", "bp_ipc_free", "bp_ipc_open", "bp_ipc_close", "bp_quire_gemm_noalloc",
    "bp_bp32_to_f64",
)


def check(rc: int) -> None:
    """Raise for a negative status, mapping to the reference's exception types
    where one exists (bad format -> KeyError as the reference's dict lookups,
    bad argument -> ValueError)."""
    if rc == BP_OK:
        return
    msg = lib().bp_last_error().decode(errors="replace")
    if rc == BP_EFMT:
        raise KeyError(msg)
    if rc in (BP_EINVAL, BP_ERANGE, BP_EALIGN, BP_EWORKSPACE):
        raise ValueError(msg)
    raise BpositError(rc, msg)
