"""bposit_b200 -- the b-posit W8A8 hot path (bp8 / bp16 encode and decode,
exact quire GEMM, single quire -> bposit32 round) as sm_100a CUDA kernels
behind a C ABI, with drop-in mirrors of the reference's Python API:

    from bposit_b200 import bposit_fast, bposit_quantize, bposit_ref, ops
"""
from __future__ import annotations

__all__ = ["bposit_fast", "bposit_quantize", "bposit_ref", "ops", "workloads", "dist"]
__version__ = "0.1.0"


def __getattr__(name):
    if name in __all__:
        import importlib
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
