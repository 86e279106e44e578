"""GPU parity of the elementwise codec kernels (through the C ABI) against the
oracle and the reference's golden outputs: bit-exact codes and values."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from bposit_b200 import ops as o
    return o


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_decode_all_codes(ops, orc):
    c8 = np.arange(256, dtype=np.uint8)
    c16 = np.arange(65536, dtype=np.uint16)
    assert np.array_equal(ops.decode(dev(c8)).cpu().numpy().view(np.uint32),
                          orc.decode_f32(c8, 8).view(np.uint32))
    assert np.array_equal(ops.decode(dev(c16)).cpu().numpy().view(np.uint32),
                          orc.decode_f32(c16, 16).view(np.uint32))
    g = golden("bp16")["decoded"]
    got = ops.decode(dev(c16)).cpu().numpy().astype(np.float64)
    assert np.array_equal(np.where(np.isnan(g), 0.0, g), got)


def test_decode_unaligned_and_ragged(ops, orc):
    rng = np.random.default_rng(3)
    base = rng.integers(0, 256, 4099, dtype=np.uint8)
    t = dev(base)
    for off in (0, 1, 3, 15):
        for n in (0, 1, 15, 16, 17, 4000):
            got = ops.decode(t[off:off + n]).cpu().numpy()
            assert np.array_equal(got.view(np.uint32), orc.decode_f32(base[off:off + n], 8).view(np.uint32))


@pytest.mark.parametrize("off", [0, 1, 2, 3, 4, 5, 8])
def test_codec_ragged_offsets_all_kernels(ops, orc, off):
    """Every codec kernel on views starting `off` elements into an aligned
    buffer (vector path when the view stays 4/8/16-byte aligned, scalar path
    otherwise) and on lengths around the tile sizes (partial tiles, the
    elements after the last whole four-element unit)."""
    from bposit_b200 import workloads
    big = workloads.codec_sweep(3 * 32768 + 64, "bp16", seed=off)
    xt = dev(big)
    c8 = np.random.default_rng(off).integers(0, 256, big.size, dtype=np.uint8)
    c16 = np.random.default_rng(off + 1).integers(0, 65536, big.size).astype(np.uint16)
    c8t, c16t = dev(c8), dev(c16)
    for n in (0, 1, 3, 4, 5, 4095, 4096, 4097, 8193, 3 * 32768 + 7):
        sl = slice(off, off + n)
        assert np.array_equal(ops.decode(c8t[sl]).cpu().numpy().view(np.uint32),
                              orc.decode_f32(c8[sl], 8).view(np.uint32))
        assert np.array_equal(ops.decode(c16t[sl]).cpu().numpy().view(np.uint32),
                              orc.decode_f32(c16[sl], 16).view(np.uint32))
        for rtne in (True, False):
            assert np.array_equal(ops.encode_bp16(xt[sl], rtne=rtne).cpu().numpy(), orc.encode_bp16(big[sl], rtne))
        got = ops.quantize_bp8(xt[sl], nearest=True).cpu().numpy()
        assert np.array_equal(got, orc.quantize_bp8(big[sl], nearest=True)[0])


def test_quantize_bp8_golden(ops):
    """bposit_fast.quantize_bp8 codes on every midpoint / grid point +-1 ulp,
    the specials and a seeded sample (both modes)."""
    g = golden("quantize_bp8")
    x = dev(g["x"])
    cn, vn = ops.quantize_bp8(x, nearest=True, return_values=True)
    ct = ops.quantize_bp8(x, nearest=False)
    assert np.array_equal(cn.cpu().numpy(), g["codes_nearest"])
    assert np.array_equal(ct.cpu().numpy(), g["codes_trunc"])
    assert np.array_equal(vn.cpu().numpy().view(np.uint32), ops.decode(cn).cpu().numpy().view(np.uint32))


def test_quantize_bp8_f64_golden(ops):
    """The float64 entry on the reference self-test sample (truncating mode,
    reference/bposit_fast.py:199-212) and on the golden float32 set."""
    g = golden("fast_selftest")
    assert np.array_equal(ops.quantize_bp8(dev(g["xs"]), nearest=False).cpu().numpy(), g["enc_codes"])
    q = golden("quantize_bp8")
    x64 = dev(q["x"].astype(np.float64))
    assert np.array_equal(ops.quantize_bp8(x64, nearest=True).cpu().numpy(), q["codes_nearest"])
    assert np.array_equal(ops.quantize_bp8(x64, nearest=False).cpu().numpy(), q["codes_trunc"])


def test_quantize_bp8_f64_between_fp32(ops, orc):
    """float64 values that are not fp32: one float64 ulp around every midpoint."""
    _, mids = orc.bp8_grid()
    x = np.concatenate([np.nextafter(mids, np.inf), np.nextafter(mids, -np.inf), mids])
    x = np.concatenate([x, -x])
    got = ops.quantize_bp8(dev(x), nearest=True).cpu().numpy()
    assert np.array_equal(got, orc.quantize_bp8_f64(x, nearest=True))


@pytest.mark.parametrize("n", [1, 15, 16, 17, 1000, 1 << 20])
def test_quantize_bp8_random_vs_oracle(ops, orc, n):
    from bposit_b200 import workloads
    x = workloads.codec_sweep(n, "bp8", seed=n)
    for nearest in (True, False):
        c, v = ops.quantize_bp8(dev(x), nearest=nearest, return_values=True)
        rc, rv = orc.quantize_bp8(x, nearest=nearest)
        assert np.array_equal(c.cpu().numpy(), rc)
        assert np.array_equal(v.cpu().numpy().view(np.uint32), rv.view(np.uint32))


def test_quantize_bp8_nan_and_unaligned(ops, orc):
    x = np.array([np.nan, -np.nan, 1.0, -2.0, np.inf, -np.inf, 0.0, -0.0], np.float32)
    big = np.tile(x, 9)
    t = dev(big)
    for off in (0, 1, 2, 3):
        got = ops.quantize_bp8(t[off:off + 33]).cpu().numpy()
        ref, _ = orc.quantize_bp8(big[off:off + 33])
        assert np.array_equal(got, ref)
    assert ops.quantize_bp8(dev(x[:1])).item() == 0x80


def test_encode_bp16_golden(ops):
    g = golden("bp16")
    assert np.array_equal(ops.encode_bp16(dev(g["x"]), rtne=True).cpu().numpy(), g["rtne"])
    assert np.array_equal(ops.encode_bp16(dev(g["x_trunc"]), rtne=False).cpu().numpy(), g["trunc"])


@pytest.mark.parametrize("n", [7, 1 << 20])
def test_encode_bp16_random_vs_oracle(ops, orc, n):
    from bposit_b200 import workloads
    x = workloads.codec_sweep(n, "bp16", seed=n + 1)
    for rtne in (True, False):
        assert np.array_equal(ops.encode_bp16(dev(x), rtne=rtne).cpu().numpy(), orc.encode_bp16(x, rtne))


def test_codec_roundtrip_every_code(ops):
    """encode(value(code)) == code for every finite nonzero code
    (reference/roundtrip_test.py), for bp8 (both modes) and bp16 (both modes)."""
    c8 = torch.arange(256, dtype=torch.int32).to(torch.uint8).cuda()
    v8 = ops.decode(c8)
    for nearest in (True, False):
        back = ops.quantize_bp8(v8, nearest=nearest).cpu().numpy()
        exp = np.arange(256, dtype=np.uint8)
        exp[0x80] = 0
        assert np.array_equal(back, exp)
    c16 = torch.arange(65536, dtype=torch.int32).to(torch.uint16).cuda()
    v16 = ops.decode(c16)
    for rtne in (True, False):
        back = ops.encode_bp16(v16, rtne=rtne).cpu().numpy()
        exp = np.arange(65536, dtype=np.uint16)
        exp[0x8000] = 0
        assert np.array_equal(back, exp)


def test_codec_sweep_full_size_properties(ops, orc):
    """The 2^28-element sweep (1 GiB of fp32): a seeded 2^22 subsample matches
    the oracle, decode(quantize(x)) is idempotent under re-quantization, and
    the code order follows the value order."""
    n = 1 << 28
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.empty(n, dtype=torch.float32, device="cuda")
    half = n // 2
    x[:half].normal_(generator=gen)
    e = torch.empty(n - half, dtype=torch.float32, device="cuda").uniform_(-26, 26, generator=gen)
    s = torch.where(torch.rand(n - half, device="cuda", generator=gen) < 0.5, -1.0, 1.0)
    x[half:] = torch.exp2(e) * s
    codes, vals = ops.quantize_bp8(x, nearest=True, return_values=True)
    idx = torch.randint(0, n, (1 << 22,), device="cuda", generator=gen)
    xs = x[idx].cpu().numpy()
    rc, _ = orc.quantize_bp8(xs, nearest=True)
    assert np.array_equal(codes[idx].cpu().numpy(), rc)
    again = ops.quantize_bp8(vals, nearest=True)
    assert torch.equal(again, codes)
    # monotone: sort by x, values must be non-decreasing
    sub = torch.sort(x[idx]).values
    sv = ops.quantize_bp8(sub, nearest=True, return_values=True)[1]
    assert bool((sv[1:] >= sv[:-1]).all())
    c16 = ops.encode_bp16(x, rtne=True)
    r16 = orc.encode_bp16(xs, True)
    assert np.array_equal(c16.view(torch.int16)[idx].cpu().numpy().view(np.uint16), r16)
    dv = ops.decode(c16)
    assert torch.equal(ops.encode_bp16(dv, rtne=True).view(torch.int16), c16.view(torch.int16))
    del x, codes, vals, c16, dv
    torch.cuda.empty_cache()


def test_group_quantize_w8a8_linear(ops):
    g = golden("w8a8_linear")
    for name, sname, cname in (("X", "sx", "xc"), ("W", "sw", "wc")):
        codes, e = ops.quantize_bp8_grouped(dev(g[name]), group=128, nearest=True)
        assert np.array_equal(e.cpu().numpy(), g[sname])
        assert np.array_equal(codes.cpu().numpy(), g[cname])
        codes2, _ = ops.quantize_bp8_grouped(dev(g[name]), group=128, nearest=True, exps=e)
        assert torch.equal(codes, codes2)


@pytest.mark.parametrize("shape,group", [((3, 5), 4), ((7, 129), 128), ((33, 1000), 64), ((2, 576), 128)])
def test_group_quantize_vs_oracle(ops, orc, shape, group):
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) * np.exp2(rng.integers(-30, 30, size=(shape[0], 1)))).astype(np.float32)
    x[0, :min(3, shape[1])] = 0.0
    if shape[1] > 4:
        x[1 % shape[0], 4] = 1e-42   # subnormal
    for nearest in (True, False):
        codes, e = ops.quantize_bp8_grouped(dev(x), group=group, nearest=nearest)
        re_ = orc.group_scales(x, group)
        assert np.array_equal(e.cpu().numpy(), re_)
        assert np.array_equal(codes.cpu().numpy(), orc.quantize_bp8_grouped(x, re_, group, nearest))


def test_quire_to_bp32_encoder_vectors(ops):
    """All 132,811 quire256 -> bposit32 vectors of reference/gen_encoder_vectors.py."""
    g = golden("encoder_vectors")
    q = dev(g["quire"])
    assert np.array_equal(ops.quire_to_bp32(q).cpu().numpy(), g["bp32"])
    # sign-extended to 12 and 16 limbs
    for nl in (12, 16):
        ext = np.where((g["quire"][:, 7:8] >> 31) == 1, np.uint32(0xFFFFFFFF), np.uint32(0))
        wide = np.concatenate([g["quire"]] + [ext] * (nl - 8), axis=1)
        assert np.array_equal(ops.quire_to_bp32(dev(wide)).cpu().numpy(), g["bp32"])


def test_quire_to_bp16_golden(ops):
    """quire256_to_bposit16 (reference/bposit_ref.py:620-635) on the encoder-vector
    quires and the extra saturation / power-of-two / seeded quires, directly from
    the limbs and through the bposit32 round."""
    g = golden("quire_bp16")
    ev = golden("encoder_vectors")
    assert np.array_equal(ops.quire_to_bp16(dev(ev["quire"])).cpu().numpy(), g["ev_bp16"])
    assert np.array_equal(ops.bp32_to_bp16(dev(ev["bp32"])).cpu().numpy(), g["ev_bp16"])
    assert np.array_equal(ops.quire_to_bp16(dev(g["quire"])).cpu().numpy(), g["bp16"])
    assert np.array_equal(ops.bp32_to_bp16(ops.quire_to_bp32(dev(g["quire"]))).cpu().numpy(), g["bp16"])


def test_dot_out_fmt_bp16(orc):
    """dot(..., out_fmt="bp16") and matmul_bp16 against the oracle's quires."""
    from bposit_b200 import bposit_fast as bf
    rng = np.random.default_rng(5)
    A = rng.integers(0, 256, (7, 300), dtype=np.uint8)
    B = rng.integers(0, 256, (5, 300), dtype=np.uint8)
    _, q = orc.quire_gemm(A, B, 8, nlimbs=16)
    ref = orc.quire_to_bp16(q.reshape(-1, 16)).reshape(7, 5)
    assert np.array_equal(bf.matmul_bp16(A, B, "bp8"), ref)
    assert bf.dot(A[2], B[3], "bp8", out_fmt="bp16") == int(ref[2, 3])
    with pytest.raises(KeyError):
        bf.dot(A[0], B[0], "bp8", out_fmt="bp8")


def test_bp32_to_f64(ops, orc):
    g = golden("bp32_decode")
    c = g["codes"]
    got = ops.bp32_to_f64(dev(c)).cpu().numpy().ravel()
    v = g["values"]
    assert np.array_equal(got, np.where(np.isnan(v), 0.0, v))
