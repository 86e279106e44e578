"""bp_quire_gemm_noalloc: the quire GEMM for callers that cannot allocate
device memory (a plugin whose host framework owns the device-memory budget, or
a latency-critical loop that cannot afford cudaMalloc's device
synchronization).  Checked through the C ABI against the allocating entry
point bp_quire_gemm (algo 1, the same CUDA-core GEMM) and against the oracle,
on two calls in a row with different inputs, so a stale scratch array from the
first call would show up in the second; then on bp16 codes, unscaled bp8 codes
(the GEMM's fast window) and a call with M + N exactly at the scratch limit, so
the last scratch record is written and read.  Kept in its own file, collected
last; it needs nothing from the other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT_ROWS = 65536   # (1 MiB scratch) / (16-byte record per row of A and of B)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(seed, M, N, K, group, fmt=8, scaled=True):
    rng = np.random.default_rng(seed)
    hi = 256 if fmt == 8 else 65536
    dt = np.uint8 if fmt == 8 else np.uint16
    A = rng.integers(0, hi, (M, K)).astype(dt)
    B = rng.integers(0, hi, (N, K)).astype(dt)
    if not scaled:
        return A, B, None, None
    G = (K + group - 1) // group
    sa = rng.integers(-20, 6, (M, G)).astype(np.int32)
    sb = rng.integers(-20, 6, (N, G)).astype(np.int32)
    return A, B, sa, sb


def _dev(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _both(L, stream, fmt, A, B, sa, sb, group, limbs):
    """(allocating entry point, no-alloc entry point) results: bp32 and quires."""
    M, K = A.shape
    N = B.shape[0]
    dA, dB, dsa, dsb = _dev(A), _dev(B), _dev(sa), _dev(sb)
    ref = torch.empty((M, N), dtype=torch.uint32, device="cuda")
    refq = torch.empty((M, N, limbs), dtype=torch.uint32, device="cuda") if limbs else None
    rc = L.bp_quire_gemm(fmt, _p(dA), _p(dB), M, N, K, _p(dsa), _p(dsb), group, _p(ref), N, _p(refq), limbs,
                         1, None, 0, stream)
    assert rc == 0, L.bp_last_error()
    out = torch.full((M, N), 0xDEAD, dtype=torch.int32, device="cuda").view(torch.uint32)
    outq = torch.zeros((M, N, limbs), dtype=torch.uint32, device="cuda") if limbs else None
    rc = L.bp_quire_gemm_noalloc(fmt, _p(dA), _p(dB), M, N, K, _p(dsa), _p(dsb), group, _p(out), N, _p(outq),
                                 limbs, stream)
    assert rc == 0, L.bp_last_error()
    assert L.bp_last_error() == b""
    torch.cuda.synchronize()
    return ref, refq, out, outq


def test_noalloc_matches_allocating_entry_point_twice(orc):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from bposit_b200 import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, (M, N, K, group) in ((1, (70, 130, 700, 128)), (2, (33, 257, 300, 64))):
        A, B, sa, sb = _inputs(seed, M, N, K, group)
        ref, refq, out, outq = _both(L, stream, 8, A, B, sa, sb, group, 16)
        assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        assert torch.equal(outq.view(torch.int32), refq.view(torch.int32))
        exp = orc.quire_gemm(A, B, 8, sa=sa, sb=sb, group=group)
        assert np.array_equal(out.cpu().numpy(), exp)


@pytest.mark.parametrize("case", ["bp16", "bp8_unscaled", "limit_rows"])
def test_noalloc_formats_and_limit(orc, case):
    from bposit_b200 import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if case == "bp16":
        A, B, sa, sb = _inputs(7, 40, 90, 333, 128, fmt=16, scaled=False)
        fmt = 16
    elif case == "bp8_unscaled":
        A, B, sa, sb = _inputs(8, 64, 100, 1000, 128, scaled=False)
        fmt = 8
    else:   # M + N == LIMIT_ROWS, small K: the last statistics record (row N-1 of B) is used
        A, B, sa, sb = _inputs(9, 16, LIMIT_ROWS - 16, 8, 128, scaled=False)
        fmt = 8
    for _ in range(2):   # two calls in a row on the shared scratch
        ref, _, out, _ = _both(L, stream, fmt, A, B, sa, sb, 128, 0)
        assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
    if case == "limit_rows":
        # the oracle on a column sample that includes the last rows of B
        cols = np.r_[0:64, LIMIT_ROWS - 16 - 64:LIMIT_ROWS - 16]
        exp = orc.quire_gemm(A, B[cols], fmt)
        assert np.array_equal(out.cpu().numpy()[:, cols], exp)
    else:
        assert np.array_equal(out.cpu().numpy(), orc.quire_gemm(A, B, fmt))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from bposit_b200 import _lib
    L = _lib.lib()
    vp = ctypes.c_void_p
    rc = L.bp_quire_gemm_noalloc(8, vp(256), vp(256), 40000, 30000, 16, None, None, 128, vp(256), 30000, None, 0,
                                 None)
    assert rc == _lib.BP_ERANGE
    assert b"scratch" in L.bp_last_error()
    rc = L.bp_quire_gemm_noalloc(8, vp(256), vp(256), 1, LIMIT_ROWS, 16, None, None, 128, vp(256), LIMIT_ROWS, None,
                                 0, None)
    assert rc == _lib.BP_ERANGE
