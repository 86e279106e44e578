"""bp_quire_gemm_noalloc: the quire GEMM for callers that cannot allocate
device memory (a plugin whose host framework owns the device-memory budget, or
a latency-critical loop that cannot afford cudaMalloc's device
synchronization).  Checked through the C ABI against the allocating entry
point bp_quire_gemm on two calls in a row with different inputs, so a stale
scratch array from the first call would show up in the second.  Kept in its own
file, collected last; it needs nothing from the other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(seed, M, N, K, group):
    rng = np.random.default_rng(seed)
    A = torch.from_numpy(rng.integers(0, 256, (M, K), dtype=np.uint8)).cuda()
    B = torch.from_numpy(rng.integers(0, 256, (N, K), dtype=np.uint8)).cuda()
    G = (K + group - 1) // group
    sa = torch.from_numpy(rng.integers(-20, 6, (M, G)).astype(np.int32)).cuda()
    sb = torch.from_numpy(rng.integers(-20, 6, (N, G)).astype(np.int32)).cuda()
    return A, B, sa, sb


def test_noalloc_matches_allocating_entry_point_twice():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from bposit_b200 import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, (M, N, K, group) in ((1, (70, 130, 700, 128)), (2, (33, 257, 300, 64))):
        A, B, sa, sb = _inputs(seed, M, N, K, group)
        ref = torch.empty((M, N), dtype=torch.uint32, device="cuda")
        refq = torch.empty((M, N, 16), dtype=torch.uint32, device="cuda")
        rc = L.bp_quire_gemm(8, _p(A), _p(B), M, N, K, _p(sa), _p(sb), group, _p(ref), N, _p(refq), 16,
                             0, None, 0, stream)
        assert rc == 0, L.bp_last_error()
        out = torch.full((M, N), 0xDEAD, dtype=torch.int32, device="cuda").view(torch.uint32)
        outq = torch.zeros((M, N, 16), dtype=torch.uint32, device="cuda")
        rc = L.bp_quire_gemm_noalloc(8, _p(A), _p(B), M, N, K, _p(sa), _p(sb), group, _p(out), N, _p(outq), 16,
                                     stream)
        assert rc == 0, L.bp_last_error()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        assert torch.equal(outq.view(torch.int32), refq.view(torch.int32))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from bposit_b200 import _lib
    L = _lib.lib()
    vp = ctypes.c_void_p
    rc = L.bp_quire_gemm_noalloc(8, vp(256), vp(256), 40000, 30000, 16, None, None, 128, vp(256), 30000, None, 0,
                                 None)
    assert rc == _lib.BP_ERANGE
    assert b"scratch" in L.bp_last_error()
