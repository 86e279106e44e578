"""CPU-only checks of the product library: it is built, loads, exports every
symbol include/bposit_b200.h declares, and validates arguments on the host;
plus an exhaustive host-compiled check of the format logic the kernels use."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "bposit_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?(?:unsigned\s+)?[a-z_0-9 ]+?\s*\*?\s*(bp_[a-z0-9_]+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from bposit_b200 import _lib
    L = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 10
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    assert set(syms) == set(_lib.EXPORTED)


def test_version_and_error_string():
    from bposit_b200 import _lib
    L = _lib.lib()
    assert L.bp_version() >= 100
    assert isinstance(L.bp_last_error(), bytes)


def test_host_argument_validation():
    """Invalid arguments are rejected before any device work."""
    from bposit_b200 import _lib
    L = _lib.lib()
    vp = ctypes.c_void_p
    rc = L.bp_quire_gemm(7, None, None, 1, 1, 1, None, None, 128, vp(16), 1, None, 0, 0, None, 0, None)
    assert rc == _lib.BP_EFMT
    rc = L.bp_quire_gemm(8, None, None, -1, 1, 1, None, None, 128, vp(16), 1, None, 0, 0, None, 0, None)
    assert rc == _lib.BP_EINVAL
    rc = L.bp_quire_gemm(8, vp(16), vp(16), 2, 4, 8, None, None, 128, vp(16), 3, None, 0, 0, None, 0, None)
    assert rc == _lib.BP_EINVAL and b"ldo" in L.bp_last_error()
    rc = L.bp_quire_gemm(8, vp(16), vp(16), 2, 4, 8, vp(16), None, 0, vp(16), 4, None, 0, 0, None, 0, None)
    assert rc == _lib.BP_EINVAL
    rc = L.bp_quire_gemm(8, vp(16), vp(16), 2, 4, 8, None, None, 128, vp(16), 4, vp(16), 5, 0, None, 0, None)
    assert rc == _lib.BP_EINVAL
    rc = L.bp_quire_gemm(8, vp(16), vp(16), 2, 4, 8, None, None, 128, vp(16), 4, None, 0, 6, None, 0, None)
    assert rc == _lib.BP_EINVAL   # algo 0..5
    rc = L.bp_quire_gemm(8, vp(16), vp(16), 2, 4, 8, None, None, 128, vp(16), 4, None, 0, 0, vp(17), 1 << 20, None)
    assert rc == _lib.BP_EALIGN
    assert L.bp_decode(9, vp(16), 4, vp(16), None) == _lib.BP_EFMT
    assert L.bp_decode(8, None, 4, vp(16), None) == _lib.BP_EINVAL
    assert L.bp_quire_to_bp32(vp(16), 9, 1, vp(16), None) == _lib.BP_EINVAL
    assert L.bp_quantize_bp8_grouped(vp(16), 2, 8, 0, 1, 1, 24, vp(16), vp(16), None) == _lib.BP_EINVAL
    # zero-size calls are no-ops that succeed without touching a device
    assert L.bp_quire_gemm(8, None, None, 0, 5, 3, None, None, 128, None, 5, None, 0, 0, None, 0, None) == 0
    assert L.bp_quire_gemm_workspace_size(8, 16, 16, 16, 1) >= 16 * 2 * 16


def test_plane_form_workspace():
    """The narrow bp8 form (algo 4, or auto for K >= 16384) holds K-major copies
    of both operands' codes beside its two digit planes; the wide form (algo 5)
    does not.  Auto sizes for whichever form the call may take."""
    from bposit_b200 import _lib
    L = _lib.lib()
    M, N, K = 256, 512, 4096
    narrow = L.bp_quire_gemm_workspace_size(8, M, N, K, 4)
    wide = L.bp_quire_gemm_workspace_size(8, M, N, K, 5)
    assert narrow >= 3 * (M + N) * K and wide >= 3 * (M + N) * K   # 2 planes + copies / 3 planes
    assert L.bp_quire_gemm_workspace_size(8, M, N, K, 0) == wide
    K = 65536
    assert L.bp_quire_gemm_workspace_size(8, M, N, K, 0) >= L.bp_quire_gemm_workspace_size(8, M, N, K, 4)
    assert L.bp_quire_gemm_workspace_size(8, M, N, K, 0) >= L.bp_quire_gemm_workspace_size(8, M, N, K, 5)
    assert L.bp_quire_gemm_workspace_size(16, M, N, K, 4) == L.bp_quire_gemm_workspace_size(16, M, N, K, 5)


def test_python_errors_match_reference_types():
    """Unknown formats raise KeyError (the reference's dict lookups); non-2-D
    GEMM operands raise ValueError (reference/bposit_fast.py:147-148)."""
    from bposit_b200 import bposit_fast, ops
    with pytest.raises(KeyError):
        ops.fmt_bits("bp5")
    with pytest.raises(KeyError):
        bposit_fast.dot_quire([1], [1], "bp6")
    with pytest.raises(ValueError):
        bposit_fast.matmul_quire([1, 2], [[1, 2]], "bp8")


@pytest.fixture(scope="module")
def host_check():
    build = os.path.join(REPO, "tests", "_build")
    os.makedirs(build, exist_ok=True)
    obj = os.path.join(build, "orc.o")
    exe = os.path.join(build, "host_format_check")
    subprocess.run(["gcc", "-O2", "-fPIC", "-c", "-o", obj, os.path.join(REPO, "oracle", "bposit_oracle.c")],
                   check=True)
    subprocess.run(["g++", "-O2", "-std=c++17", "-pthread", "-o", exe,
                    os.path.join(REPO, "tests", "host_format_check.cpp"), obj, "-lm"], check=True)
    return exe


@pytest.mark.parametrize("what", ["dec", "bp32", "q8", "e16", "e16t", "signed", "small"])
def test_format_logic_matches_oracle_exhaustively(host_check, what):
    """The kernels' format logic (bp_format.cuh) compiled for the host vs the
    oracle: all bp8/bp16 codes; 2M random quires; every non-negative fp32
    pattern for the bp8 quantize table (both modes); a strided full sweep of
    fp32 patterns plus every binade edge for the bp16 encoder (both modes); a
    strided fp32 sweep and 2M random doubles for the bposit4 / AI-posit5 encoders;
    the streaming kernels' table bp16 encoder on every fp32 pattern (both modes)
    and their closed-form bp16 decode on every code; the signed bp8 / bp16 tables
    on every fp32 pattern (both modes)."""
    nt = max(1, min(8, len(os.sched_getaffinity(0))))
    r = subprocess.run([host_check, what, str(nt)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "mismatches: 0" in r.stdout


def test_recommended_exponents_nan_row_raises_like_reference():
    """A NaN row passes the reference's `rms <= 0` guard and fails in
    int(np.round(np.log2(nan))) (reference/bposit_quantize.py:56-62)."""
    import numpy as np
    from bposit_b200.bposit_quantize import recommended_exponents
    with pytest.raises(ValueError):
        recommended_exponents(np.array([[np.nan, 1.0, 2.0]]))
    assert list(recommended_exponents(np.array([[0.0, 0.0], [4.0, 4.0]]))) == [0, 2]


def test_huge_quires_clamp_to_saturation():
    """Python-int quires beyond 16 limbs are clamped to 2^(96+241), which both
    the bposit32 and bposit16 rounds saturate at, instead of wrapping."""
    from bposit_b200.bposit_ref import _QUIRE_SAT, _ints_to_limbs
    from oracle import oracle as orc
    limbs = _ints_to_limbs([1 << 700, -(1 << 700), 5])
    assert orc.limbs_to_int(limbs[0]) == _QUIRE_SAT and orc.limbs_to_int(limbs[1]) == -_QUIRE_SAT
    assert orc.limbs_to_int(limbs[2]) == 5
    b32 = orc.quire_to_bp32(limbs)
    assert list(b32) == [0x7FFFFFFF, 0x80000001, orc.quire_to_bp32(limbs[2:3])[0]]
