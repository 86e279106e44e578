"""GPU parity of the exact quire GEMM (both the CUDA-core and the tensor-core
paths, through the C ABI) against the reference's golden vectors and the
oracle: every bposit32 output word and every raw quire bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

# 1 = CUDA cores, 2 = tensor cores (paired SMs when M > 128), 3 = tensor cores, one SM per
# tile, 4 / 5 = tensor cores with the narrow (2 base-256 planes) / wide (3 base-128) bp8 form
ALGOS = [1, 2, 3, 4, 5]
ALGOS16 = [1, 2, 3]


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from bposit_b200 import ops as o
    return o


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def tc_ok(ops, fmt, M, N, K):
    from bposit_b200 import _lib
    L = _lib.lib()
    return L.bp_quire_gemm_workspace_size(fmt, M, N, K, 2) > L.bp_quire_gemm_workspace_size(fmt, M, N, K, 1)


def run(ops, A, B, fmt, algo, sa=None, sb=None, group=128, quire_limbs=0):
    out, q = ops.quire_gemm(dev(A), dev(B), fmt, sa=None if sa is None else dev(sa),
                            sb=None if sb is None else dev(sb), group=group, quire_limbs=quire_limbs,
                            algo=algo)
    return out.cpu().numpy(), (None if q is None else q.cpu().numpy())


def test_bp8_exhaustive_products(ops):
    """reference/gen_bp8_exhaustive.py: all 65,536 bp8 x bp8 products."""
    g = golden("bp8_exhaustive")
    A = np.arange(256, dtype=np.uint8).reshape(256, 1)
    out, _ = run(ops, A, A, 8, 1)
    assert np.array_equal(out.ravel(), g["bp32"])


def test_rtl_bp8_dots(ops):
    """reference/gen_rtl_vectors.py: 22 bp8 dots of K=32 (quires and bp32)."""
    g = golden("rtl_bp8")
    for i in range(g["a"].shape[0]):
        out, q = run(ops, g["a"][i:i + 1], g["b"][i:i + 1], 8, 1, quire_limbs=8)
        assert np.array_equal(q[0, 0], g["quire"][i]), i
        assert int(out[0, 0]) == int(g["bp32"][i]), i


def test_fast_selftest_dots(ops):
    """reference/bposit_fast.py:181-197: 300 seeded bp8 dots, K in [1, 400)."""
    g = golden("fast_selftest")
    off = g["off"]
    for i in range(len(off) - 1):
        out, _ = run(ops, g["a"][off[i]:off[i + 1]][None], g["b"][off[i]:off[i + 1]][None], 8, 1)
        assert int(out[0, 0]) == int(g["bp32"][i]), i


@pytest.mark.parametrize("algo", ALGOS)
def test_w8a8_linear_golden(ops, algo):
    """16x576x576 group-scaled W8A8 linear: every quire and bp32 word."""
    g = golden("w8a8_linear")
    if algo >= 2 and not tc_ok(ops, 8, 16, 576, 576):
        pytest.skip("tensor-core path not available for this shape")
    out, q = run(ops, g["xc"], g["wc"], 8, algo, sa=g["sx"], sb=g["sw"], quire_limbs=8)
    assert np.array_equal(q, g["quire"])
    assert np.array_equal(out, g["bp32"])


def rand_codes(rng, shape, fmt, zero_frac=0.05):
    n = 1 << fmt
    c = rng.integers(0, n, size=shape, dtype=np.int64)
    c[rng.random(shape) < zero_frac] = 0
    return c.astype(np.uint8 if fmt == 8 else np.uint16)


SHAPES = [(1, 1, 1), (1, 1, 0), (3, 5, 7), (17, 33, 65), (64, 48, 130), (129, 131, 257), (200, 256, 512)]


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_bp8_random_vs_oracle(ops, orc, algo, M, N, K):
    if algo >= 2 and not tc_ok(ops, 8, M, N, K):
        pytest.skip("tensor-core path not available for this shape")
    rng = np.random.default_rng(M * 1000 + N * 10 + K)
    A, B = rand_codes(rng, (M, K), 8), rand_codes(rng, (N, K), 8)
    out, q = run(ops, A, B, 8, algo, quire_limbs=8)
    rb, rq = orc.quire_gemm(A, B, 8, nlimbs=8)
    assert np.array_equal(q, rq)
    assert np.array_equal(out, rb)


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("M,N,K,group", [(5, 7, 300, 128), (40, 70, 576, 128), (130, 66, 1000, 64)])
def test_bp8_group_scaled_vs_oracle(ops, orc, algo, M, N, K, group):
    if algo >= 2 and not tc_ok(ops, 8, M, N, K):
        pytest.skip("tensor-core path not available for this shape")
    rng = np.random.default_rng(K + group)
    X = (rng.standard_normal((M, K)) * np.exp2(rng.integers(-6, 6, (M, 1)))).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    sx, sw = orc.group_scales(X, group), orc.group_scales(W, group)
    xc, wc = orc.quantize_bp8_grouped(X, sx, group), orc.quantize_bp8_grouped(W, sw, group)
    out, q = run(ops, xc, wc, 8, algo, sa=sx, sb=sw, group=group, quire_limbs=16)
    rb, rq = orc.quire_gemm(xc, wc, 8, sa=sx, sb=sw, group=group, nlimbs=16)
    assert np.array_equal(q, rq)
    assert np.array_equal(out, rb)


def test_bp8_truncating_terms(ops, orc):
    """Scales that push products below 2^-96: per-term truncation toward zero
    (the reference's int() / bposit_fast.py:125-127 branch)."""
    rng = np.random.default_rng(11)
    M, N, K, group = 6, 9, 200, 32
    A, B = rand_codes(rng, (M, K), 8), rand_codes(rng, (N, K), 8)
    G = (K + group - 1) // group
    sa = rng.integers(-40, 5, (M, G)).astype(np.int32)
    sb = rng.integers(-40, 5, (N, G)).astype(np.int32)
    out, q = run(ops, A, B, 8, 1, sa=sa, sb=sb, group=group, quire_limbs=16)
    rb, rq = orc.quire_gemm(A, B, 8, sa=sa, sb=sb, group=group, nlimbs=16)
    assert np.array_equal(q, rq)
    assert np.array_equal(out, rb)


@pytest.mark.parametrize("algo", ALGOS16)
@pytest.mark.parametrize("M,N,K", [(2, 3, 5), (33, 17, 100), (128, 64, 256)])
def test_bp16_random_vs_oracle(ops, orc, algo, M, N, K):
    """bp16 quire GEMM on uniformly random codes (exponents up to +-112, so
    products span 2^-224..2^224 and many terms truncate per term)."""
    if algo >= 2 and not tc_ok(ops, 16, M, N, K):
        pytest.skip("tensor-core path not available for this shape")
    rng = np.random.default_rng(M + N + K)
    A, B = rand_codes(rng, (M, K), 16), rand_codes(rng, (N, K), 16)
    out, q = run(ops, A, B, 16, algo, quire_limbs=16)
    rb, rq = orc.quire_gemm(A, B, 16, nlimbs=16)
    assert np.array_equal(q, rq)
    assert np.array_equal(out, rb)


@pytest.mark.parametrize("algo", ALGOS16)
def test_bp16_normal_range_vs_oracle(ops, orc, algo):
    """bp16 operands ~ N(0,1) * 2^U{-8..8} per row (the large-GEMM distribution)."""
    from bposit_b200 import workloads
    M, N, K = 96, 160, 1024
    if algo >= 2 and not tc_ok(ops, 16, M, N, K):
        pytest.skip("tensor-core path not available for this shape")
    A = orc.encode_bp16(workloads.per_row_po2(M, K, 1), True)
    B = orc.encode_bp16(workloads.per_row_po2(N, K, 2), True)
    out, _ = run(ops, A, B, 16, algo)
    assert np.array_equal(out, orc.quire_gemm(A, B, 16))


@pytest.mark.parametrize("algo", [2, 3])
@pytest.mark.parametrize("K", [8192, 150000])
def test_bp16_sums_beyond_64_bits(ops, orc, algo, K):
    """bp16 rows whose main digits span the full 27 bits (values near 2^10,
    one tiny element per row sets the base and becomes a listed tail), all of
    one sign: the exact main sums pass 2^64, so every word of the tensor-core
    path's sums (and, at K = 150000, its split-K chunks) is exercised."""
    rng = np.random.default_rng(K + algo)
    M, N = 200, 192
    if not tc_ok(ops, 16, M, N, K):
        pytest.skip("tensor-core path not available for this shape")

    def operand(rows):
        x = (1024.0 * (1.0 + rng.random((rows, K)))).astype(np.float32)
        x[:, 0] = np.float32(2.0 ** -16)
        x[1::7] *= -1.0
        return orc.encode_bp16(x, True)

    A, B = operand(M), operand(N)
    out, _ = run(ops, A, B, 16, algo)
    rows = np.arange(M) if K <= 8192 else np.array([0, 1, 129, 199])
    assert np.array_equal(out[rows], orc.quire_gemm(A[rows], B, 16))
    assert _device_error() == 0


def test_column_block_output(ops, orc):
    """ldo > N: an output shard written into its column block of a wider matrix."""
    rng = np.random.default_rng(5)
    A, B = rand_codes(rng, (20, 64), 8), rand_codes(rng, (30, 64), 8)
    full = torch.zeros((20, 100), dtype=torch.uint32, device="cuda")
    ops.quire_gemm(dev(A), dev(B), 8, out=full[:, 40:70])
    got = full.cpu().numpy()
    assert np.array_equal(got[:, 40:70], orc.quire_gemm(A, B, 8))
    assert not got[:, :40].any() and not got[:, 70:].any()


def test_zero_and_nar_only(ops):
    A = np.array([[0, 0x80, 0], [0x80, 0x80, 0x80]], np.uint8)
    B = np.array([[0x40, 0x7F, 0x01]], np.uint8)
    out, q = run(ops, A, B, 8, 1, quire_limbs=8)
    assert not out.any() and not q.any()


@pytest.mark.parametrize("algo", [0, 4, 5])
def test_tc_nar_codes_count_as_zero(ops, orc, algo):
    """NaR codes inside tensor-core rows decode to 0, as code_value does
    (reference/bposit_ref.py:1022-1025): rows with scattered NaRs, a row of NaR
    and zero only, a row whose one nonzero code sits among NaRs.  K = 16384
    takes the narrow form under auto, whose row statistics treat a span that
    holds a NaR apart."""
    rng = np.random.default_rng(11)
    M, N, K = 384, 352, 16384     # M x N large enough for the tensor cores under auto

    def codes(rows):   # magnitudes 0x28 .. 0x57 (values near 1), random signs
        mag = rng.integers(0x28, 0x58, (rows, K))
        return np.where(rng.random((rows, K)) < 0.5, mag, 256 - mag).astype(np.uint8)

    A, B = codes(M), codes(N)
    A[rng.random((M, K)) < 0.01] = 0x80
    B[rng.random((N, K)) < 0.01] = 0x80
    A[3] = np.where(rng.random(K) < 0.5, 0x80, 0).astype(np.uint8)
    A[5] = 0x80
    A[5, 777] = 0x41
    B[7, :4096] = 0x80
    out, _ = run(ops, A, B, 8, algo)
    assert np.array_equal(out, orc.quire_gemm(A, B, 8))
    assert not out[3].any()


def test_smollm_layer_shapes_row_subsample(ops, orc):
    """The SmolLM2-135M-shaped projections at M=2048 (group-scaled RTN codes):
    all outputs computed on the device, 16 rows checked against the oracle."""
    from bposit_b200 import workloads
    rng = np.random.default_rng(0)
    M = 2048
    for name, N, K in workloads.SMOLLM_SHAPES:
        X = rng.standard_normal((M, K)).astype(np.float32)
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        xc, sx = ops.quantize_bp8_grouped(dev(X))
        wc, sw = ops.quantize_bp8_grouped(dev(W))
        out, _ = ops.quire_gemm(xc, wc, 8, sa=sx, sb=sw)
        rows = np.sort(rng.choice(M, 16, replace=False))
        ref = orc.quire_gemm(xc.cpu().numpy()[rows], wc.cpu().numpy(), 8, sa=sx.cpu().numpy()[rows],
                             sb=sw.cpu().numpy())
        assert np.array_equal(out.cpu().numpy()[rows], ref), name


@pytest.mark.parametrize("algo", [0, 5])
def test_large_bp8_k65536_row_subsample(ops, orc, algo):
    """bp8 4096 x 4096 x 65536 (operands N(0,1) * 2^U{-8..8} per row): every
    output on the device, 3 full rows and a 64-column block checked against
    the oracle; auto (the narrow form, tens of tail elements per row) and the
    wide form."""
    from bposit_b200 import workloads
    M = N = 4096
    K = 65536
    torch.manual_seed(0)
    gen = torch.Generator(device="cuda").manual_seed(1)

    def operand(rows):
        x = torch.randn((rows, K), device="cuda", generator=gen)
        e = torch.randint(-8, 9, (rows, 1), device="cuda", generator=gen).float()
        return ops.quantize_bp8(x * torch.exp2(e), nearest=True)

    A, B = operand(M), operand(N)
    out, _ = ops.quire_gemm(A, B, 8, algo=algo)
    o = out.cpu().numpy()
    An, Bn = A.cpu().numpy(), B.cpu().numpy()
    rows = np.array([0, 3900, 4095])   # the last tiles (last M block, both halves) run K-split
    assert np.array_equal(o[rows], orc.quire_gemm(An[rows], Bn, 8))
    cols = np.arange(1000, 1064)
    assert np.array_equal(o[:64, cols], orc.quire_gemm(An[:64], Bn[cols], 8))
    assert _device_error() == 0
    del A, B, out
    torch.cuda.empty_cache()


def test_large_bp16_8192_row_subsample(ops, orc):
    """bp16 8192 x 8192 x 8192 (operands N(0,1) * 2^U{-8..8} per row,
    encode_bposit16 RTNE): every output on the device; four full rows and a
    64 x 64 block checked against the oracle.  With 256 x 64 tile pairs the
    8192^3 grid is 4096 pairs, 55 full waves of 74 and a last partial wave that
    runs split along K; in the grouped tile order those last tiles are tile
    rows 24..31 x tile columns 124..127, so rows 6200 and 8191 cross them
    (columns 7936..8191) and row 0 / the block cross whole-K tiles."""
    M = N = K = 8192
    gen = torch.Generator(device="cuda").manual_seed(2)

    def operand(rows):
        x = torch.randn((rows, K), device="cuda", generator=gen)
        e = torch.randint(-8, 9, (rows, 1), device="cuda", generator=gen).float()
        return ops.encode_bp16(x * torch.exp2(e), rtne=True)

    A, B = operand(M), operand(N)
    out, _ = ops.quire_gemm(A, B, 16)
    o = out.cpu().numpy()
    An, Bn = A.cpu().numpy(), B.cpu().numpy()
    rows = np.array([0, 4321, 6200, 8191])
    assert np.array_equal(o[rows], orc.quire_gemm(An[rows], Bn, 16))
    blk_r, blk_c = np.arange(1000, 1064), np.arange(3000, 3064)
    assert np.array_equal(o[np.ix_(blk_r, blk_c)], orc.quire_gemm(An[blk_r], Bn[blk_c], 16))
    assert _device_error() == 0
    del A, B, out
    torch.cuda.empty_cache()


@pytest.mark.parametrize("algo", [2, 3, 4])
def test_balanced_last_wave(ops, orc, algo):
    """96 paired (192 single) tiles: one full wave runs whole, the remaining tiles
    run split along K with 128-bit partials; rows in whole and split tiles."""
    M, N, K = 2048, 1152, 4096
    rng = np.random.default_rng(11)
    A = rand_codes(rng, (M, K), 8)
    B = rand_codes(rng, (N, K), 8)
    out, _ = run(ops, A, B, 8, algo)
    rows = np.array([0, 1000, 1600, 1800, 2000, 2047])
    assert np.array_equal(out[rows], orc.quire_gemm(A[rows], B, 8))


def _device_error():
    import ctypes
    from bposit_b200 import _lib
    v = ctypes.c_int(0)
    assert _lib.lib().bp_device_error(ctypes.byref(v)) == 0
    return v.value


@pytest.mark.parametrize("fmt,algo", [(8, 2), (8, 4), (16, 2)])
def test_tc_listed_tails(ops, orc, fmt, algo):
    """Rows whose values span more than the tensor-core digit window: a few
    tiny elements per row become listed tails, corrected exactly on CUDA cores."""
    rng = np.random.default_rng(40 + fmt)
    M, N, K = 150, 170, 1000
    X = rng.standard_normal((M, K)).astype(np.float32)
    Y = rng.standard_normal((N, K)).astype(np.float32)
    for Z in (X, Y):
        rows = np.repeat(np.arange(Z.shape[0]), 3)
        cols = rng.integers(0, K, rows.size)
        Z[rows, cols] = (rng.standard_normal(rows.size) * (2.0 ** -22 if fmt == 8 else 2.0 ** -60)).astype(np.float32)
    if fmt == 8:
        A, B = orc.quantize_bp8(X)[0], orc.quantize_bp8(Y)[0]
    else:
        A, B = orc.encode_bp16(X, True), orc.encode_bp16(Y, True)
    out, q = run(ops, A, B, fmt, algo, quire_limbs=16)
    rb, rq = orc.quire_gemm(A, B, fmt, nlimbs=16)
    assert np.array_equal(q, rq)
    assert np.array_equal(out, rb)
    assert _device_error() == 0


def test_tc_narrow_correction_term_bounds(ops, orc):
    """Narrow-form tail corrections at the edges of their integer forms.  The
    other operand's rows span 29, 30 and 31 binades (largest binade minus
    smallest lsb) in its three 512-column passes; 31 leaves the int32
    multiply form.  The tail rows' largest tail exponent above the row minimum
    runs from about 21 to 30, so passes take the int32 multiply, the 64-bit
    shift and the 128-bit forms.  Raw quires and bposit32 words bit-exact."""
    rng = np.random.default_rng(77)
    M, N, K = 64, 1536, 512
    X = np.zeros((M, K), np.float32)
    for i in range(M):
        bx = 12 + i % 9                                   # largest binade 12 .. 20
        cols = rng.choice(K, 40, replace=False)
        X[i, cols[0]] = 2.0 ** bx
        X[i, cols[1]] = 2.0 ** -24                        # minpos: lsb -24
        X[i, cols[2:]] = (rng.standard_normal(38) * 2.0 ** rng.integers(-20, bx, 38)).astype(np.float32)
    Y = rng.standard_normal((N, K)).astype(np.float32)
    Y[:, 0] = 2.0 ** (5 + np.arange(N) // 512)            # largest binade 5, 6, 7 per pass
    Y[:, 1] = 2.0 ** -24
    A, B = orc.quantize_bp8(X)[0], orc.quantize_bp8(Y)[0]
    out, q = run(ops, A, B, 8, 4, quire_limbs=16)
    rb, rq = orc.quire_gemm(A, B, 8, nlimbs=16)
    assert np.array_equal(q, rq)
    assert np.array_equal(out, rb)
    out2, _ = run(ops, A, B, 8, 4)
    assert np.array_equal(out2, rb)
    assert _device_error() == 0


@pytest.mark.parametrize("algo", [2, 4])
def test_tc_tail_overflow_goes_to_fixup(ops, orc, algo):
    """More tail elements in a row than the tail list holds: that row's
    outputs are recomputed by the exact fixup kernel."""
    rng = np.random.default_rng(9)
    M, N, K = 40, 50, 3000
    A = orc.quantize_bp8(rng.standard_normal((M, K)).astype(np.float32))[0]
    B = orc.quantize_bp8(rng.standard_normal((N, K)).astype(np.float32))[0]
    A[3, :2000] = 0x01          # 2000 x minpos
    A[3, 2000] = 0x7F           # maxpos: the row's window cannot reach minpos
    B[7, ::2] = 0xFF            # -minpos
    B[7, 1] = 0x7E
    out, _ = run(ops, A, B, 8, algo)
    assert np.array_equal(out, orc.quire_gemm(A, B, 8))
    assert _device_error() == 0


@pytest.mark.parametrize("algo", [2, 5])
def test_tc_split_k(ops, orc, algo):
    """K beyond one exact int32 chunk: per-chunk 128-bit partial sums (auto
    takes the narrow form here, with its tail lists; 5 the wide one)."""
    rng = np.random.default_rng(10)
    M, N, K = 64, 96, 200000
    A = orc.quantize_bp8(rng.standard_normal((M, K)).astype(np.float32))[0]
    B = orc.quantize_bp8(rng.standard_normal((N, K)).astype(np.float32))[0]
    out, _ = run(ops, A, B, 8, algo)
    rows = np.array([0, 17, 63])
    assert np.array_equal(out[rows], orc.quire_gemm(A[rows], B, 8))
    assert _device_error() == 0
