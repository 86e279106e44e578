"""The reference-facing mirrors (bposit_fast / bposit_quantize / bposit_ref
names and return types) on the GPU, checked like the reference's own
self-tests (reference/bposit_fast.py:179-251, examples/smoke_test.sh:24-38)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from bposit_b200 import bposit_fast, bposit_quantize, bposit_ref
    return bposit_fast, bposit_quantize, bposit_ref


def test_quantize_bp8_values_match_reference(api, orc):
    bf, _, _ = api
    g = golden("fast_selftest")
    xs = g["xs"]
    got = bf.quantize_bp8(xs)                    # float64 in, float64 out, truncating
    assert got.dtype == np.float64 and got.shape == xs.shape
    exp = orc.decode_f32(g["enc_codes"], 8).astype(np.float64)
    assert np.array_equal(got, exp)
    q = golden("quantize_bp8")
    x = q["x"].astype(np.float64)
    vn = bf.quantize_bp8(x, nearest=True)
    dec = orc.decode_f32(q["codes_nearest"], 8).astype(np.float64)
    exp = np.where(q["codes_nearest"] == 0, np.copysign(0.0, x), dec)     # np.sign(-0.0) * 0 = -0.0
    assert np.array_equal(vn.view(np.uint64), exp.view(np.uint64))
    assert np.array_equal(bf.quantize_bp8_codes(x, nearest=True), q["codes_nearest"])


def test_device_error_word_clear_and_nar_handoff():
    """After ordinary tensor-core GEMMs the device error word reads 0 (a
    nonzero word makes the Python API raise and marks every tensor-core output
    NaR); NaR, which no quire round produces, reaches a model as NaN through the
    fp32 hand-off, while the reference's float64 rescale keeps NaR -> 0.0."""
    from bposit_b200 import ops
    rng = np.random.default_rng(5)
    A = torch.from_numpy(rng.integers(0, 256, (256, 256), dtype=np.uint8)).cuda()
    out, _ = ops.quire_gemm(A, A, 8, algo=2)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert not bool((out == 0x80000000).any())
    codes = torch.tensor([[0x80000000, 0x40000000, 0]], dtype=torch.int64).to(torch.uint32).cuda()
    f32 = ops.bp32_to_f32(codes).cpu().numpy()
    assert np.isnan(f32[0, 0]) and f32[0, 1] == 1.0 and f32[0, 2] == 0.0
    f64 = ops.bp32_to_f64(codes).cpu().numpy()
    assert f64[0, 0] == 0.0 and f64[0, 1] == 1.0


@pytest.mark.parametrize("algo,M,N,K,fmt,opts", [
    (1, 37, 50, 300, 8, "exps+bias"), (0, 512, 1152, 896, 8, "exps+bias"), (2, 256, 300, 2000, 8, "none"),
    (0, 300, 1024, 1000, 16, "col+bias"), (0, 64, 96, 640, 8, "groups"), (2, 1024, 768, 4096, 8, "groups")])
def test_quire_gemm_f32_equals_gemm_then_handoff(algo, M, N, K, fmt, opts):
    """bp_quire_gemm_f32 (the fp32 hand-off written by the GEMM's output stage)
    gives the same fp32 words as bp_quire_gemm followed by bp_bp32_to_f32, on
    the CUDA-core and tensor-core paths, and the same bposit32 codes when asked."""
    from bposit_b200 import ops
    rng = np.random.default_rng(M + N + K)
    dt = np.uint8 if fmt == 8 else np.uint16
    A = torch.from_numpy(rng.integers(0, 1 << fmt, (M, K)).astype(dt)).cuda()
    B = torch.from_numpy(rng.integers(0, 1 << fmt, (N, K)).astype(dt)).cuda()
    sa = sb = re = ce = bias = None
    if opts == "groups":
        G = (K + 127) // 128
        sa = torch.from_numpy(rng.integers(-10, 5, (M, G)).astype(np.int32)).cuda()
        sb = torch.from_numpy(rng.integers(-10, 5, (N, G)).astype(np.int32)).cuda()
    if opts in ("exps+bias",):
        re = torch.from_numpy(rng.integers(-6, 6, M).astype(np.int32)).cuda()
    if opts in ("exps+bias", "col+bias"):
        ce = torch.from_numpy(rng.integers(-6, 6, N).astype(np.int32)).cuda()
        bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).cuda()
    codes, _ = ops.quire_gemm(A, B, fmt, sa=sa, sb=sb, algo=algo)
    ref = ops.bp32_to_f32(codes, row_exp=re, col_exp=ce, bias=bias)
    out_bp32 = torch.empty((M, N), dtype=torch.uint32, device="cuda")
    got = ops.quire_gemm_f32(A, B, fmt, sa=sa, sb=sb, row_exp=re, col_exp=ce, bias=bias, out_bp32=out_bp32,
                             algo=algo)
    got2 = ops.quire_gemm_f32(A, B, fmt, sa=sa, sb=sb, row_exp=re, col_exp=ce, bias=bias, algo=algo)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), ref.view(torch.int32))
    assert torch.equal(got2.view(torch.int32), ref.view(torch.int32))
    assert torch.equal(out_bp32.view(torch.int32), codes.view(torch.int32))
    assert ops.device_error() == 0


def test_quire256_clamps_huge_python_ints(api):
    """quires far beyond 512 bits round to +-maxpos exactly as the reference's
    unbounded Python ints do (bposit32 saturates above total exponent 240,
    bposit16 above 112), instead of wrapping in the 16-limb buffer."""
    _, _, br = api
    for q in (1 << 600, -(1 << 600), (1 << 511) + 12345, (1 << (96 + 241)) - 1):
        s = -1 if q < 0 else 1
        assert br.quire256_to_bposit32(q) == (0x7FFFFFFF if s > 0 else 0x80000001)
        assert br.quire256_to_bposit16(q) == (0x7FFF if s > 0 else 0x8001)


def test_dot_and_dot_quire_selftest(api):
    bf, _, _ = api
    g = golden("fast_selftest")
    off = g["off"]
    for i in range(0, len(off) - 1, 7):
        a = g["a"][off[i]:off[i + 1]].astype(np.int64)
        b = g["b"][off[i]:off[i + 1]].astype(np.int64)
        assert bf.dot(a, b, "bp8", "bp32") == int(g["bp32"][i])


def test_dot_quire_rtl_vectors(api, orc):
    bf, _, _ = api
    g = golden("rtl_bp8")
    for i in range(g["a"].shape[0]):
        q = bf.dot_quire(g["a"][i].tolist(), g["b"][i].tolist(), "bp8")
        assert q & ((1 << 256) - 1) == orc.limbs_to_int(g["quire"][i]) & ((1 << 256) - 1)


def test_matmul_quire_vs_per_dot(api):
    """reference/bposit_fast.py:228-238: matmul_quire == per-dot quire."""
    bf, _, _ = api
    rng = np.random.default_rng(0)
    A = rng.integers(0, 256, size=(3, 200), dtype=np.int64)
    B = rng.integers(0, 256, size=(5, 200), dtype=np.int64)
    M = bf.matmul_quire(A, B, "bp8")
    assert M.shape == (3, 5) and M.dtype == object
    for i in range(3):
        for j in range(5):
            assert int(M[i, j]) == bf.dot_quire(A[i], B[j], "bp8")


def test_quire256_to_bposit32(api):
    _, _, br = api
    g = golden("encoder_vectors")
    qs = [int.from_bytes(g["quire"][i].tobytes(), "little", signed=True) for i in range(0, 132811, 97)]
    got = br.quire256_to_bposit32(np.array(qs, dtype=object))
    assert np.array_equal(got, g["bp32"][::97])
    assert br.quire256_to_bposit32(0) == 0


def test_code_value_and_encode_bposit16(api):
    _, _, br = api
    g = golden("bp16")
    assert np.array_equal(br.encode_bposit16(g["x"], "rtne"), g["rtne"])
    with pytest.raises(ValueError):
        br.encode_bposit16(1.0, "nearest")
    assert br.code_value(0x40, "bp8") == 1.0 and br.code_value(0x80, "bp8") == 0.0


def test_quantize_w8a8_matches_reference(api):
    """examples/smoke_test.sh:24-38 inputs: Y identical to the reference's
    quantize_w8a8 output, and deterministic across calls."""
    _, bq, _ = api
    g = golden("quantize_w8a8")
    assert np.array_equal(bq.recommended_exponents(g["W"]), g["w_exp"])
    assert np.array_equal(bq.recommended_exponents(g["X"]), g["x_exp"])
    y1 = bq.quantize_w8a8(g["W"], g["X"])
    y2 = bq.quantize_w8a8(g["W"], g["X"])
    assert np.array_equal(y1, g["Y"])
    assert np.array_equal(y1, y2)


def test_shuffled_tiling_reproducible(api):
    """examples/w8a8_rounding_demo.py:80-89: identical codes across a re-run and
    a shuffled tiling of the input."""
    bf, _, _ = api
    rng = np.random.default_rng(0)
    x0 = rng.standard_normal((16, 128)) * 0.5
    c1 = bf.quantize_bp8_codes(x0, nearest=True)
    flat = x0.ravel()
    idx = np.arange(flat.size)
    rng.shuffle(idx)
    out = np.empty(flat.size, np.uint8)
    for s in range(0, flat.size, 97):
        j = idx[s:s + 97]
        out[j] = bf.quantize_bp8_codes(flat[j], nearest=True)
    assert np.array_equal(c1, bf.quantize_bp8_codes(x0, nearest=True))
    assert np.array_equal(c1, out.reshape(x0.shape))


def test_small_rungs_against_reference_vectors():
    """bposit4 / AI-posit5 through the reference-named API: code_value,
    quantize_vec, dot_at_precision (bp32 and bp16 out), mixed_precision_sum
    over bp4/aip5/bp8/bp16, and bposit_fast.matmul_quire / dot for bp4 and aip5."""
    from bposit_b200 import bposit_fast as bf
    from bposit_b200 import bposit_ref as br
    g = golden("rungs")
    for fmt, nb in (("bp4", 4), ("aip5", 5)):
        assert np.array_equal(br.code_value(np.arange(1 << nb), fmt), g[f"{fmt}_values"])
    x = g["q_in"]
    for fmt in ("bp4", "aip5", "bp8"):
        assert br.quantize_vec(x, fmt) == [int(v) for v in g[f"q_{fmt}"]], fmt
    for fmt in ("bp4", "aip5", "bp8"):
        lens = g[f"dot_{fmt}_len"]
        off = np.concatenate([[0], np.cumsum(lens)])
        for i in range(0, len(lens), 3):
            a = g[f"dot_{fmt}_a"][off[i]:off[i + 1]]
            b = g[f"dot_{fmt}_b"][off[i]:off[i + 1]]
            assert br.dot_at_precision(a, b, fmt, "bp32") == int(g[f"dot_{fmt}_bp32"][i])
            assert br.dot_at_precision(a, b, fmt, "bp16") == int(g[f"dot_{fmt}_bp16"][i])
            if fmt != "bp8":
                assert bf.dot(a, b, fmt) == int(g[f"dot_{fmt}_bp32"][i])
    fm = ("bp4", "aip5", "bp8", "bp16")
    lens = g["mix_len"]
    off = np.concatenate([[0], np.cumsum(lens)])
    for i in range(0, len(lens), 2):
        items = [(int(c), fm[f]) for c, f in zip(g["mix_code"][off[i]:off[i + 1]], g["mix_fmt"][off[i]:off[i + 1]])]
        assert br.mixed_precision_sum(items, "bp32") == int(g["mix_bp32"][i]), i
        assert br.mixed_precision_sum(items, "bp16") == int(g["mix_bp16"][i]), i
    # matmul_quire on bp4 codes equals the bp8 GEMM of the widened codes
    rng = np.random.default_rng(3)
    A = rng.integers(0, 16, (5, 70))
    B = rng.integers(0, 16, (4, 70))
    q4 = bf.matmul_quire(A, B, "bp4")
    from oracle import oracle as orc
    _, q = orc.quire_gemm(orc.transcode(A.astype(np.uint8), 4, 8), orc.transcode(B.astype(np.uint8), 4, 8), 8,
                          nlimbs=16)
    assert all(int(q4[i, j]) == int.from_bytes(q[i, j].tobytes(), "little", signed=True)
               for i in range(5) for j in range(4))


@pytest.mark.parametrize("case", ["chunked", "chunked_groups", "bp16_small", "pageable", "rows", "rows_groups",
                                  "rows_strided_out", "rows_bp16_small"])
def test_quire_gemm_host_buffers(case):
    """bp_quire_gemm_host (host buffers; one operand prepared once, the other
    streamed in row chunks: B when M < N, A when M >= N) gives exactly the
    device GEMM's codes."""
    from bposit_b200 import ops
    rng = np.random.default_rng(7)
    group = 128
    if case in ("chunked", "chunked_groups", "pageable"):
        M, N, K, fmt = 2048, 3000, 16384, 8      # 82 MB of codes: B in 4 chunks of 768 rows, the last padded
    elif case == "rows_bp16_small":
        M, N, K, fmt = 300, 200, 1000, 16        # one chunk, CUDA-core GEMM (B's preparation step is a no-op)
    elif case.startswith("rows"):
        M, N, K, fmt = 3000, 2048, 16384, 8      # A in 4 chunks of 768 rows, the last padded
    else:
        M, N, K, fmt = 200, 300, 1000, 16
    dt = np.uint8 if fmt == 8 else np.uint16
    if case in ("chunked_groups", "rows_groups"):
        X = torch.randn(M, K, device="cuda")
        W = torch.randn(N, K, device="cuda") * 0.02
        A, sa = ops.quantize_bp8_grouped(X, group=group)
        B, sb = ops.quantize_bp8_grouped(W, group=group)
    else:
        A = torch.from_numpy(rng.integers(0, 1 << fmt, (M, K)).astype(dt)).cuda()
        B = torch.from_numpy(rng.integers(0, 1 << fmt, (N, K)).astype(dt)).cuda()
        sa = sb = None
    ref, _ = ops.quire_gemm(A, B, fmt, sa=sa, sb=sb, group=group)
    if case == "pageable":
        hA, hB = A.cpu().numpy(), B.cpu().numpy()
        out = ops.quire_gemm_host(hA, hB, fmt)
    else:
        hA, hB = A.cpu().pin_memory(), B.cpu().pin_memory()
        hsa = None if sa is None else sa.cpu().pin_memory()
        hsb = None if sb is None else sb.cpu().pin_memory()
        wide = None
        if case == "rows_strided_out":          # the result lands in a column block of a wider matrix
            wide = torch.zeros((M, N + 40), dtype=torch.uint32).pin_memory()
        out = ops.quire_gemm_host(hA, hB, fmt, sa=hsa, sb=hsb, group=group,
                                  out=None if wide is None else wide[:, 16:16 + N])
        if wide is not None:
            torch.cuda.current_stream().synchronize()
            assert not wide[:, :16].view(torch.int32).any() and not wide[:, 16 + N:].view(torch.int32).any()
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out.view(torch.int32), ref.cpu().view(torch.int32))
