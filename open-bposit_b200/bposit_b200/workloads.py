"""Seeded synthetic inputs with the shapes and value distributions of the five
benchmark workloads (no dataset or checkpoint is needed: every workload is
random-init by definition).

* ``w8a8_linear``  -- one bp8 W8A8 linear: X[16,576] ~ N(0,1) with 1% outliers
  ~ N(0,20^2), W[576,576] ~ N(0,0.02^2), per-group-128 power-of-two scales.
* ``codec_sweep``  -- fp32 values: half N(0,1), half log-uniform magnitudes over
  the bp8 (2^+-24) or bp16 (2^+-112) range, with +-0, saturation edges, exact
  midpoints (ties) and sub-minpos values mixed in.
* ``smollm_layers`` -- the q/k/v/o/gate/up/down projection shapes of a
  SmolLM2-135M-shaped Llama block (hidden 576, intermediate 1536, 9 Q / 3 KV
  heads, head_dim 64) at M=2048 tokens.
* ``large_gemm``   -- operands N(0,1) * 2^U{-8..8} per row (bp8
  4096x4096x65536, bp16 8192^3).
"""
from __future__ import annotations

import numpy as np

SMOLLM_SHAPES = (  # (name, N, K) for y = x @ W^T with W[N, K]
    ("q_proj", 576, 576),
    ("k_proj", 192, 576),
    ("v_proj", 192, 576),
    ("o_proj", 576, 576),
    ("gate_proj", 1536, 576),
    ("up_proj", 1536, 576),
    ("down_proj", 576, 1536),
)

QWEN05_SHAPES = (  # one Qwen2.5-0.5B-shaped layer, N-fused qkv and gate+up
    ("qkv_proj", 896 + 2 * 128, 896),
    ("o_proj", 896, 896),
    ("gate_up_proj", 2 * 4864, 896),
    ("down_proj", 896, 4864),
)


def w8a8_linear(seed: int = 0, M: int = 16, K: int = 576, N: int = 576):
    """(X[M,K], W[N,K]) float32."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, K))
    mask = rng.random((M, K)) < 0.01
    X[mask] = rng.standard_normal(int(mask.sum())) * 20.0
    W = rng.standard_normal((N, K)) * 0.02
    return X.astype(np.float32), W.astype(np.float32)


def codec_sweep(n: int, fmt: str = "bp8", seed: int = 0) -> np.ndarray:
    """n float32 values for the encode/decode sweep (see module docstring)."""
    rng = np.random.default_rng(seed)
    lim = 24 if fmt == "bp8" else 112
    half = n // 2
    a = rng.standard_normal(half).astype(np.float32)
    mag = np.exp2(rng.uniform(-lim - 2, lim + 2, n - half)).astype(np.float32)
    sgn = np.where(rng.random(n - half) < 0.5, -1.0, 1.0).astype(np.float32)
    b = mag * sgn
    x = np.concatenate([a, b])
    edges = np.array([0.0, -0.0, 2.0 ** lim, -(2.0 ** lim), 2.0 ** (lim + 1), -(2.0 ** (lim + 1)),
                      2.0 ** -lim, -(2.0 ** -lim), 2.0 ** (-lim - 2), -(2.0 ** (-lim - 2)),
                      1.0, -1.0, 1.5, 1.0625, 3.0 * 2.0 ** -lim], dtype=np.float32)
    m = min(len(edges), n)
    x[:m] = edges[:m]
    return x


def per_row_po2(rows: int, cols: int, seed: int, lo: int = -8, hi: int = 8) -> np.ndarray:
    """N(0,1) scaled by 2^U{lo..hi} per row, float32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    e = rng.integers(lo, hi + 1, size=(rows, 1))
    return (x * np.exp2(e).astype(np.float32)).astype(np.float32)
