"""torch.nn drop-in: a Linear layer computed as a bp8 W8A8 exact-quire GEMM.

    lin = BpositLinear.from_linear(torch.nn.Linear(896, 4864).cuda())
    y = lin(x)                       # x [..., 896] float -> y [..., 4864] float32

Two scale recipes:

* ``scales="w8a8"`` (default) -- the reference's W8A8 recipe
  (reference/bposit_quantize.py:46-89): one power-of-two exponent per row of
  W and of X (round(log2(ref)), ref = RMS or the 95th percentile of |x| when
  that exceeds twice the RMS), truncating bp8 encode of the scaled rows, the
  exact quire GEMM, one bposit32 round per output, then value * 2^(e_x + e_w)
  (+ bias) rounded once to the nearest fp32.  The weight exponents come from
  the host numpy rule (``bposit_quantize.recommended_exponents``); the
  activations go through one kernel per forward (``ops.w8a8_encode_rows``:
  the same rule in float64 on the device, then the encode; numpy's summation
  order is not reproduced, so an exponent can differ only when ref lies within
  an ulp of 2^(k + 1/2), or the 95th percentile within an ulp of twice the
  RMS).
* ``scales="group128"`` -- the per-(row, 128-group) power-of-two scales of the
  benchmark's W8A8 linear: s = ceil(log2(absmax)) - 24, round-to-nearest
  encode, scales folded into the GEMM's element exponents.  This maps each
  group's largest value to bp8's maxpos, where the format has no fraction bits,
  so it is the benchmark's definition rather than an accurate recipe.

With ``act="bp16"`` (``scales="w8a8"`` only) the activations are not scaled
but encoded as bp16, round-to-nearest-even (``encode_bposit16(·, "rtne")``,
reference/bposit_ref.py:382-507), and the bp8 weight codes are widened exactly
to bp16 (every bp8 value is a bp16 value): the same exact quire GEMM then runs
in bp16, one bposit32 round, value * 2^e_w (+ bias) rounded once to fp32 --
the bp16 activation path of the mixed-rung quire.

The weight is encoded once, on first use or by ``quantize_weight()``.  The
reference itself has no module API; this wraps its recipe for torch models.

Multi-GPU (one process per GPU, ``torch.distributed`` initialised):
``shard_linears(model)`` makes every BpositLinear split its GEMM's output block
over the process group -- a pm x pn grid of (tokens, output features) blocks,
``dist.choose_grid`` -- each rank computing its block from its rows of the
activation codes and of the (replicated) weight codes, the GEMM's finish
kernel storing the bposit32 words into every rank's copy of the full output
over NVLink (``dist.FusedShardedQuireGemm``).  Outputs are column- and
row-independent and no partial sum crosses a rank, so the result is the same
words as on one GPU; everything outside the linears runs replicated.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from .bposit_quantize import _LIMIT_ZERO, _encode_rows, recommended_exponents


def row_exponents(x: torch.Tensor) -> torch.Tensor:
    """recommended_exponents (reference/bposit_quantize.py:46-63) of the rows of
    x [rows, K] on the device, float64: int32 [rows]."""
    v = x.double()
    K = v.shape[1]
    rms = torch.sqrt(torch.mean(v * v, dim=1))
    a = v.abs()
    # numpy percentile, 'linear': position 0.95 (K - 1) between sorted a[lo], a[lo + 1]
    pos = 0.95 * (K - 1)
    lo = int(np.floor(pos))
    t = pos - lo
    top = torch.topk(a, K - lo, dim=1, largest=True, sorted=True).values
    a_lo = top[:, -1]
    a_hi = top[:, -2] if K - lo >= 2 else a_lo
    d = a_hi - a_lo
    p95 = a_hi - d * (1.0 - t) if t >= 0.5 else a_lo + d * t
    ref = torch.where((p95 > 0) & (p95 > 2 * rms), p95, rms)
    ex = torch.round(torch.log2(torch.where(rms > 0, ref, torch.ones_like(ref))))
    return torch.where(rms > 0, ex, torch.zeros_like(ex)).to(torch.int32)


def _encode_scaled(x: torch.Tensor, ex: torch.Tensor) -> torch.Tensor:
    """Truncating bp8 encode of x / 2^ex[row] in float64, with the float entry's
    limit_denominator(10**8) zero cut (encode_bposit8, reference/bposit_ref.py:258-270)."""
    xs = x.double() / torch.exp2(ex.to(torch.float64))[:, None]   # exact: power-of-two scale
    c = ops.quantize_bp8(xs.contiguous(), nearest=False)
    return torch.where(xs.abs() <= _LIMIT_ZERO, torch.zeros_like(c), c)


class BpositLinear(torch.nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, group: int = 128,
                 scales: str = "w8a8", device=None, dtype=torch.float32, act: str = "bp8"):
        super().__init__()
        if scales not in ("w8a8", "group128"):
            raise ValueError(f"unknown scale recipe {scales!r}")
        if act not in ("bp8", "bp16") or (act == "bp16" and scales != "w8a8"):
            raise ValueError(f"unsupported activation format {act!r} with scales {scales!r}")
        self.in_features, self.out_features, self.group, self.scales = in_features, out_features, group, scales
        self.act = act
        self._wq16 = None        # bp8 weight codes widened to bp16 (act="bp16")
        self.weight = torch.nn.Parameter(torch.empty((out_features, in_features), device=device, dtype=dtype),
                                         requires_grad=False)
        self.bias = (torch.nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype), requires_grad=False)
                     if bias else None)
        self._wq = None          # (codes [N, K] uint8, exponents [N, G] int32)
        self._ws = None          # GEMM workspace, grown on demand
        self._ws_key = None
        self.sharded = False     # split the GEMM over the process group (shard_linears)
        self.algo = 0            # bp_quire_gemm algo of this layer's GEMM (0: the library's choice)

    @classmethod
    def from_linear(cls, lin: torch.nn.Linear, group: int = 128, scales: str = "w8a8",
                    act: str = "bp8") -> "BpositLinear":
        m = cls(lin.in_features, lin.out_features, bias=lin.bias is not None, group=group, scales=scales,
                device=lin.weight.device, dtype=torch.float32, act=act)
        with torch.no_grad():
            m.weight.copy_(lin.weight.float())
            if lin.bias is not None:
                m.bias.copy_(lin.bias.float())
        return m

    @torch.no_grad()
    def quantize_weight(self):
        """Encode the weight with the module's scale recipe; call again after
        changing ``weight``.  Returns (codes [N, K] uint8, exponents int32)."""
        W = self.weight.float().contiguous()
        if self.scales == "group128":
            self._wq = ops.quantize_bp8_grouped(W, group=self.group)
        else:
            Wn = W.double().cpu().numpy()
            ew = recommended_exponents(Wn)
            self._wq = (_encode_rows(Wn, ew, W.device), torch.from_numpy(ew.astype(np.int32)).to(W.device))
        self._wq16 = ops.transcode(self._wq[0], 8, 16) if self.act == "bp16" else None
        return self._wq

    def _workspace(self, M: int, device):
        fmt = 16 if self.act == "bp16" else 8
        key = (M, self.out_features, self.in_features, fmt, self.algo)
        if self._ws_key != key:
            need = ops.gemm_workspace_size(fmt, M, self.out_features, self.in_features, self.algo)
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
            self._ws_key = key
        return self._ws

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected last dimension {self.in_features}, got {x.shape[-1]}")
        if self._wq is None:
            self.quantize_weight()
        wc, ws = self._wq
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).float().contiguous()
        M = x2.shape[0]
        bias = None if self.bias is None else self.bias.float().contiguous()
        if self.scales == "group128":
            xc, xs = ops.quantize_bp8_grouped(x2, group=self.group)
            y = self._linear(xc, wc, 8, xs, ws, None, None, bias, M)
        elif self.act == "bp16":
            xc = ops.encode_bp16(x2, rtne=True)
            y = self._linear(xc, self._wq16, 16, None, None, None, ws, bias, M)
        else:
            xc, ex = ops.w8a8_encode_rows(x2)
            y = self._linear(xc, wc, 8, None, None, ex, ws, bias, M)
        return y.reshape(*lead, self.out_features)

    def _linear(self, xc, wc, fmt, sa, sb, row_exp, col_exp, bias, M):
        """fp32 [M, N] of xc @ wc^T: on this GPU one GEMM whose output stage
        writes the fp32 hand-off (value * 2^(row_exp + col_exp) + bias); sharded,
        this rank's block of bposit32 codes all-gathered into the full matrix,
        then the same hand-off."""
        if self.sharded and _world() > 1:
            g = _shared_gemm(M, self.out_features, self.in_features, fmt, xc.device)
            m0, m1, n0, n1 = g.block
            codes = g(xc[m0:m1], wc[n0:n1], sa=None if sa is None else sa[m0:m1],
                      sb=None if sb is None else sb[n0:n1])
            return ops.bp32_to_f32(codes, row_exp=row_exp, col_exp=col_exp, bias=bias)
        return ops.quire_gemm_f32(xc, wc, fmt, sa=sa, sb=sb, group=self.group, row_exp=row_exp, col_exp=col_exp,
                                  bias=bias, algo=self.algo, workspace=self._workspace(M, xc.device))

    def extra_repr(self) -> str:
        arith = "bp8 W8A8" if self.act == "bp8" else "bp8 weights, bp16 activations"
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, scales={self.scales}, arithmetic={arith} exact quire")


def bpositify(module: torch.nn.Module, group: int = 128, scales: str = "w8a8", act: str = "bp8") -> torch.nn.Module:
    """Replace every torch.nn.Linear inside `module` by a BpositLinear (in place)."""
    for name, child in list(module.named_children()):
        if isinstance(child, torch.nn.Linear):
            setattr(module, name, BpositLinear.from_linear(child, group=group, scales=scales, act=act))
        else:
            bpositify(child, group=group, scales=scales, act=act)
    return module


# ---- multi-GPU: N-sharded linears -------------------------------------------
_SHARED_GEMMS: dict = {}


def _world() -> int:
    import torch.distributed as dist
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _shared_gemm(M: int, N: int, K: int, fmt: int, device):
    """The fused sharded GEMM of one (M, N, K, fmt) shape, shared by every
    linear of that shape (its result buffer is consumed by the caller's
    bp32 -> fp32 hand-off before the next call's opening barrier).  Creating
    one is collective: every rank runs the same linears in the same order."""
    from .dist import FusedShardedQuireGemm
    key = (M, N, K, fmt, str(device))
    g = _SHARED_GEMMS.get(key)
    if g is None:
        g = FusedShardedQuireGemm(M, N, device, fmt=fmt, K=K)
        _SHARED_GEMMS[key] = g
    return g


def shard_linears(module: torch.nn.Module) -> torch.nn.Module:
    """Make every BpositLinear inside `module` split its GEMM over the default
    process group (see the module docstring).  In place; no-op on one rank."""
    for m in module.modules():
        if isinstance(m, BpositLinear):
            m.sharded = True
    return module


def close_sharded() -> None:
    """Release the shared sharded GEMMs' buffers.  Collective: call on every
    rank before destroying the process group."""
    for g in list(_SHARED_GEMMS.values()):
        g.close()
    _SHARED_GEMMS.clear()
