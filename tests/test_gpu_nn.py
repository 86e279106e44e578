"""The torch.nn drop-in (BpositLinear) and the Qwen2.5-0.5B-shaped forward built
on it, against the oracle: every checked output equals the oracle's W8A8
quire GEMM (the reference's per-row recipe, or the per-group-128 one), one
bposit32 round, exact value * scale + bias rounded to the nearest fp32."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def oracle_linear(orc, X: np.ndarray, W: np.ndarray, bias, scales: str = "w8a8", group: int = 128,
                  act: str = "bp8") -> np.ndarray:
    """The oracle's output of BpositLinear for rows X[M, K] (fp32 values)."""
    if act == "bp16":
        from bposit_b200.bposit_quantize import recommended_exponents
        W64 = W.astype(np.float64)
        ew = recommended_exponents(W64)
        s = W64 / np.exp2(ew.astype(np.float64))[:, None]
        wc = np.where(np.abs(s) <= 4.999999999999999e-09, 0, orc.quantize_bp8_f64(s, nearest=False)).astype(np.uint8)
        xc = orc.encode_bp16(X.astype(np.float32), True)
        v = orc.bp32_to_double(orc.quire_gemm(xc, orc.transcode(wc, 8, 16), 16))
        v = v * np.exp2(ew[None, :].astype(np.float64))
    elif scales == "group128":
        xs = orc.group_scales(X, group)
        ws = orc.group_scales(W, group)
        xc = orc.quantize_bp8_grouped(X, xs, group, True)
        wc = orc.quantize_bp8_grouped(W, ws, group, True)
        v = orc.bp32_to_double(orc.quire_gemm(xc, wc, 8, sa=xs, sb=ws, group=group))
    else:
        from bposit_b200.bposit_quantize import recommended_exponents
        X64, W64 = X.astype(np.float64), W.astype(np.float64)
        ex, ew = recommended_exponents(X64), recommended_exponents(W64)

        def enc(M, e):
            s = M / np.exp2(e.astype(np.float64))[:, None]
            c = orc.quantize_bp8_f64(s, nearest=False)
            return np.where(np.abs(s) <= 4.999999999999999e-09, 0, c).astype(np.uint8)

        v = orc.bp32_to_double(orc.quire_gemm(enc(X64, ex), enc(W64, ew), 8))
        v = v * np.exp2((ex[:, None] + ew[None, :]).astype(np.float64))
    if bias is not None:
        v = v + np.asarray(bias, np.float64)[None, :]
    return v.astype(np.float32)


@pytest.mark.parametrize("scales", ["w8a8", "group128"])
@pytest.mark.parametrize("M,K,N,bias", [(37, 576, 200, True), (5, 1536, 576, False), (130, 896, 1152, True)])
def test_bposit_linear_matches_oracle(orc, M, K, N, bias, scales):
    from bposit_b200.bposit_quantize import recommended_exponents
    from bposit_b200.nn import BpositLinear, row_exponents
    torch.manual_seed(M)
    lin = torch.nn.Linear(K, N, bias=bias).cuda()
    x = torch.randn(M, K, device="cuda")
    x[torch.rand(M, K, device="cuda") < 0.01] *= 20.0
    y = BpositLinear.from_linear(lin, scales=scales)(x)
    xn = x.cpu().numpy()
    assert np.array_equal(row_exponents(x).cpu().numpy(), recommended_exponents(xn.astype(np.float64)))
    ref = oracle_linear(orc, xn, lin.weight.detach().cpu().numpy(),
                        None if not bias else lin.bias.detach().cpu().numpy(), scales)
    assert y.dtype == torch.float32
    assert np.array_equal(y.cpu().numpy(), ref)


def test_qwen_shaped_forward_linears_match_oracle(orc):
    from bposit_b200.forward import qwen05, synthetic_ids
    from bposit_b200.nn import BpositLinear
    model = qwen05(layers=2)
    ids = synthetic_ids(1, 48, seed=1)
    captured = []

    def hook(mod, inp, out):
        captured.append((mod, inp[0].detach().reshape(-1, mod.in_features).clone(),
                         out.detach().reshape(-1, mod.out_features).clone()))

    hs = [m.register_forward_hook(hook) for m in model.modules() if isinstance(m, BpositLinear)]
    h = model(ids)
    for x in hs:
        x.remove()
    assert torch.isfinite(h).all()
    assert len(captured) == 8            # qkv, o, gate_up, down per layer
    rng = np.random.default_rng(0)
    for mod, x, y in captured:
        rows = rng.choice(x.shape[0], 6, replace=False)
        ref = oracle_linear(orc, x[rows].cpu().numpy(), mod.weight.cpu().numpy(),
                            None if mod.bias is None else mod.bias.cpu().numpy(), mod.scales)
        assert np.array_equal(y[rows].cpu().numpy(), ref)
    # sanity against the fp32 model with the same weights (not a parity claim)
    ref_model = qwen05(layers=2, bposit=False)
    h32 = ref_model(ids)
    cos = torch.nn.functional.cosine_similarity(h.flatten(), h32.flatten(), dim=0).item()
    assert cos > 0.97


def test_qwen_full_size_forward_row_subsample(orc):
    """The whole Qwen2.5-0.5B-shaped forward of the benchmark (24 layers, batch
    8 x 1024 tokens): at 8192 tokens every linear takes the tensor-core path
    (qkv 8192x1152x896, o 8192x896x896, gate/up 8192x9728x896, down
    8192x896x4864, with K-split last waves and side-stream finishes).  For the
    first, a middle and the last layer, eight rows of every linear's captured
    input and output are checked against the oracle."""
    from bposit_b200.forward import qwen05, synthetic_ids
    from bposit_b200.nn import BpositLinear
    model = qwen05(layers=24)
    ids = synthetic_ids(8, 1024, seed=0)
    rng = np.random.default_rng(24)
    rows = np.sort(np.concatenate([[0, 8191], rng.choice(np.arange(1, 8191), 6, replace=False)]))
    rows_t = torch.from_numpy(rows).cuda()
    check = {0, 12, 23}
    captured = []

    def hook(mod, inp, out):
        x = inp[0].detach().reshape(-1, mod.in_features)
        y = out.detach().reshape(-1, mod.out_features)
        captured.append((mod, x.index_select(0, rows_t).cpu(), y.index_select(0, rows_t).cpu()))

    hs = []
    for li, layer in enumerate(model.layers):
        if li in check:
            hs += [m.register_forward_hook(hook) for m in layer.modules() if isinstance(m, BpositLinear)]
    h = model(ids)
    for x in hs:
        x.remove()
    assert torch.isfinite(h).all()
    assert len(captured) == 4 * len(check)
    for mod, x, y in captured:
        ref = oracle_linear(orc, x.numpy(), mod.weight.cpu().numpy(),
                            None if mod.bias is None else mod.bias.cpu().numpy(), mod.scales)
        assert np.array_equal(y.numpy(), ref), (mod.in_features, mod.out_features)
    from bposit_b200 import ops
    assert ops.device_error() == 0


@pytest.mark.parametrize("K", [1, 2, 3, 20, 21, 576, 896, 1536, 4864, 9216, 9217, 12292])
def test_w8a8_encode_rows_matches_reference_rule(orc, K):
    """ops.w8a8_encode_rows: per-row exponents equal recommended_exponents
    (reference/bposit_quantize.py:46-63, numpy on the host) and the codes equal
    the oracle's truncating encode of x / 2^e with the limit_denominator zero cut."""
    from bposit_b200 import ops
    from bposit_b200.bposit_quantize import recommended_exponents
    rng = np.random.default_rng(K)
    R = 64
    X = (rng.standard_normal((R, K)) * np.exp2(rng.integers(-20, 20, (R, 1)))).astype(np.float32)
    X[0] = 0.0                                            # all-zero row
    X[1, : max(1, K // 20)] *= 1000.0                     # outliers: the p95 branch
    X[2] = 3.0                                            # all equal (ties at every rank)
    X[3] = np.where(np.arange(K) % 2 == 0, 1.0, -2.0)     # two values
    X[4] = (rng.integers(-3, 4, K) * 2.0 ** -30).astype(np.float32)   # tiny: the zero cut after scaling
    X[5, :] = np.float32(2.0 ** 7)                        # power of two
    X[6, :] = 1.0                                         # exactly one element above 2 rms (when K allows):
    X[6, K // 2] = 10.0                                   # the 95th percentile's rank at the candidates' edge
    X[7] = (rng.standard_normal(K) * np.where(rng.random(K) < 0.08, 30.0, 1.0)).astype(np.float32)  # heavy tail
    xt = torch.from_numpy(X).cuda()
    codes, exps = ops.w8a8_encode_rows(xt)
    ex_ref = recommended_exponents(X.astype(np.float64))
    assert np.array_equal(exps.cpu().numpy(), ex_ref)
    s = X.astype(np.float64) / np.exp2(ex_ref.astype(np.float64))[:, None]
    c_ref = np.where(np.abs(s) <= 4.999999999999999e-09, 0, orc.quantize_bp8_f64(s, nearest=False))
    assert np.array_equal(codes.cpu().numpy(), c_ref.astype(np.uint8))


@pytest.mark.parametrize("M,K,N,bias", [(37, 576, 200, True), (130, 896, 1152, False)])
def test_bposit_linear_bp16_activations_match_oracle(orc, M, K, N, bias):
    """act="bp16": RTNE bp16 activations, bp8 weights widened to bp16, one exact
    bp16 quire GEMM -- equal to the oracle's composition of the same steps."""
    from bposit_b200.nn import BpositLinear
    torch.manual_seed(M + 1)
    lin = torch.nn.Linear(K, N, bias=bias).cuda()
    x = torch.randn(M, K, device="cuda")
    x[torch.rand(M, K, device="cuda") < 0.01] *= 300.0
    y = BpositLinear.from_linear(lin, act="bp16")(x)
    ref = oracle_linear(orc, x.cpu().numpy(), lin.weight.detach().cpu().numpy(),
                        None if not bias else lin.bias.detach().cpu().numpy(), act="bp16")
    assert np.array_equal(y.cpu().numpy(), ref)
