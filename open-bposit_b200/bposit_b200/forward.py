"""A model-shaped forward around the W8A8 linear (the callers either side of the
hot path): a Qwen2.5-0.5B-shaped decoder stack with random-init weights
(seeded; there is no checkpoint).

Everything except the linears -- embedding, RMSNorm, RoPE, causal grouped-query
attention, SiLU gating -- runs in fp32 torch; every linear is a torch.nn.Linear
that ``bpositify`` turns into a BpositLinear (bp8 W8A8, exact quire, one
bposit32 round, nearest fp32 out).  q/k/v and gate/up are fused along N, which
is exact because GEMM outputs are column-independent.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .nn import bpositify

QWEN05 = dict(hidden=896, inter=4864, heads=14, kv_heads=2, head_dim=64, layers=24, vocab=151936,
              rope_theta=1e6, eps=1e-6)


class RMSNorm(torch.nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


def _rope(x, cos, sin):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return x * cos + torch.cat((-x2, x1), dim=-1) * sin


class DecoderLayer(torch.nn.Module):
    def __init__(self, c):
        super().__init__()
        h, hd = c["hidden"], c["head_dim"]
        self.c = c
        self.ln1 = RMSNorm(h, c["eps"])
        self.qkv = torch.nn.Linear(h, (c["heads"] + 2 * c["kv_heads"]) * hd, bias=True)
        self.o = torch.nn.Linear(c["heads"] * hd, h, bias=False)
        self.ln2 = RMSNorm(h, c["eps"])
        self.gate_up = torch.nn.Linear(h, 2 * c["inter"], bias=False)
        self.down = torch.nn.Linear(c["inter"], h, bias=False)

    def forward(self, x, cos, sin):
        c = self.c
        B, S, _ = x.shape
        hd, nh, nkv = c["head_dim"], c["heads"], c["kv_heads"]
        qkv = self.qkv(self.ln1(x))
        q, k, v = qkv.split([nh * hd, nkv * hd, nkv * hd], dim=-1)
        q = _rope(q.view(B, S, nh, hd).transpose(1, 2), cos, sin)
        k = _rope(k.view(B, S, nkv, hd).transpose(1, 2), cos, sin)
        v = v.view(B, S, nkv, hd).transpose(1, 2)
        rep = nh // nkv
        a = F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1),
                                           is_causal=True)
        x = x + self.o(a.transpose(1, 2).reshape(B, S, nh * hd))
        g, u = self.gate_up(self.ln2(x)).chunk(2, dim=-1)
        return x + self.down(F.silu(g) * u)


class QwenShaped(torch.nn.Module):
    """Qwen2.5-0.5B-shaped decoder stack (no LM head): token ids -> final hidden."""

    def __init__(self, c=None, layers: int | None = None):
        super().__init__()
        c = dict(QWEN05 if c is None else c)
        if layers is not None:
            c["layers"] = layers
        self.c = c
        self.embed = torch.nn.Embedding(c["vocab"], c["hidden"])
        self.layers = torch.nn.ModuleList([DecoderLayer(c) for _ in range(c["layers"])])
        self.norm = RMSNorm(c["hidden"], c["eps"])

    @torch.no_grad()
    def init_weights(self, seed: int = 0):
        dev = self.embed.weight.device
        g = torch.Generator(device=dev).manual_seed(seed)
        for p in self.parameters():          # matrices N(0, 0.02^2); RMSNorm weights stay 1
            if p.dim() >= 2:
                p.copy_(torch.randn(p.shape, generator=g, device=dev) * 0.02)
        for layer in self.layers:
            layer.qkv.bias.copy_(torch.randn(layer.qkv.bias.shape, generator=g, device=dev) * 0.02)
        return self

    def linear_ops(self, tokens: int) -> float:
        """2 * tokens * sum(N * K) over the decoder linears."""
        n = 0
        for layer in self.layers:
            for lin in (layer.qkv, layer.o, layer.gate_up, layer.down):
                n += lin.in_features * lin.out_features
        return 2.0 * tokens * n

    @torch.no_grad()
    def forward(self, ids):
        c = self.c
        S = ids.shape[1]
        x = self.embed(ids)
        pos = torch.arange(S, device=ids.device, dtype=torch.float32)
        inv = 1.0 / (c["rope_theta"] ** (torch.arange(0, c["head_dim"], 2, device=ids.device,
                                                         dtype=torch.float32) / c["head_dim"]))
        ang = torch.outer(pos, inv)
        cos = torch.cat((ang.cos(), ang.cos()), -1)[None, None]
        sin = torch.cat((ang.sin(), ang.sin()), -1)[None, None]
        for layer in self.layers:
            x = layer(x, cos, sin)
        return self.norm(x)


def qwen05(layers: int = 24, device="cuda", seed: int = 0, bposit: bool = True) -> QwenShaped:
    m = QwenShaped(layers=layers).to(device).init_weights(seed)
    return bpositify(m) if bposit else m


def synthetic_ids(batch: int, seq: int, vocab: int = QWEN05["vocab"], seed: int = 0, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq), generator=g, device=device)
