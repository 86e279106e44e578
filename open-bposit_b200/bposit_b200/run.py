"""Run one workload of the library on the current GPU and print its timing.

    python -m bposit_b200.run gemm M N K [--fmt bp8|bp16] [--group 128] [--calls 3] [--algo 0] [--timeline]
    python -m bposit_b200.run codec N [--fmt bp8|bp16] [--calls 3]
    python -m bposit_b200.run qwen05 [--batch 8] [--seq 1024] [--layers 24] [--fp32]
    python -m bposit_b200.run linear M N K [--calls 3]

``gemm`` times bp_quire_gemm on operands N(0,1) * 2^U{-8..8} per row (the
large-GEMM workload's distribution), quantized on the device (``--timeline``
adds the start and end of every kernel of one more call); ``linear`` times
one BpositLinear (the W8A8 nn.Linear drop-in, fp32 out) of N x K random
weights on M rows of N(0,1) activations; ``codec`` times
the encode and decode kernels on the codec-sweep value mix; ``qwen05`` times
the Qwen2.5-0.5B-shaped decoder forward with every linear a BpositLinear.  Each runs
`--calls` untimed calls and then `--calls` calls timed with CUDA events, so a
profiler can capture a fixed, small number of launches (e.g. ``ncu -k
regex:k_quire_gemm_tc -c 1``).
"""
from __future__ import annotations

import argparse
import sys

import torch

from . import ops
from .workloads import codec_sweep


def _operand(rows: int, K: int, fmt: int, gen: torch.Generator, group: int):
    x = torch.randn((rows, K), device="cuda", generator=gen)
    e = torch.randint(-8, 9, (rows, 1), device="cuda", generator=gen).float()
    x = x * torch.exp2(e)
    if group:
        if fmt != 8:
            raise SystemExit("group scales are a bp8 feature")
        return ops.quantize_bp8_grouped(x, group=group)
    if fmt == 8:
        return ops.quantize_bp8(x, nearest=True), None
    return ops.encode_bp16(x), None


def _time(fn, calls: int) -> float:
    for _ in range(calls):
        fn()
    torch.cuda.synchronize()
    s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(calls):
        fn()
    t.record()
    torch.cuda.synchronize()
    return s.elapsed_time(t) / calls


def run_gemm(a) -> str:
    fmt = ops.fmt_bits(a.fmt)
    gen = torch.Generator(device="cuda").manual_seed(a.seed)
    A, sa = _operand(a.M, a.K, fmt, gen, a.group)
    B, sb = _operand(a.N, a.K, fmt, gen, a.group)
    ws = torch.empty(max(256, ops.gemm_workspace_size(fmt, a.M, a.N, a.K, a.algo)), dtype=torch.uint8,
                     device="cuda")
    out = torch.empty((a.M, a.N), dtype=torch.uint32, device="cuda")

    def call():
        ops.quire_gemm(A, B, fmt, sa=sa, sb=sb, group=a.group or 128, out=out, algo=a.algo, workspace=ws)

    ms = _time(call, a.calls)
    line = (f"gemm {a.fmt} M={a.M} N={a.N} K={a.K} group={a.group}: {ms:.3f} ms/call, "
            f"{2.0 * a.M * a.N * a.K / ms / 1e9:.1f} TOPS")
    return line + ("\n" + _timeline(call) if a.timeline else "")


def _timeline(fn) -> str:
    """Start and end (ms from the first launch) of every kernel and memset of
    one more call, from torch.profiler's CUDA activity trace: which kernels
    overlap and which one ends the call."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    evs = [e for e in prof.events() if str(getattr(e, "device_type", "")).split(".")[-1] == "CUDA"]
    if not evs:
        return "  (no CUDA activity recorded)"
    t0 = min(e.time_range.start for e in evs)
    rows = []
    for e in sorted(evs, key=lambda e: e.time_range.start):
        name = e.name.replace("(anonymous namespace)::", "").replace("void ", "").replace("bp::", "").split("(")[0]
        rows.append(f"  {name[:48]:48s} {(e.time_range.start - t0) / 1e3:8.3f} -> {(e.time_range.end - t0) / 1e3:8.3f}"
                    f" ms  ({(e.time_range.end - e.time_range.start) / 1e3:.3f})")
    return "\n".join(rows)


def run_codec(a) -> str:
    fmt = ops.fmt_bits(a.fmt)
    x = torch.from_numpy(codec_sweep(a.n, a.fmt, a.seed)).cuda()
    if fmt == 8:
        codes = torch.empty(a.n, dtype=torch.uint8, device="cuda")
        enc = _time(lambda: ops.quantize_bp8(x, nearest=True, out=codes), a.calls)
    else:
        codes = torch.empty(a.n, dtype=torch.uint16, device="cuda")
        enc = _time(lambda: ops.encode_bp16(x, out=codes), a.calls)
    dec = _time(lambda: ops.decode(codes, a.fmt), a.calls)
    b = fmt // 8 + 4
    return (f"codec {a.fmt} n={a.n}: encode {enc:.3f} ms ({a.n * b / enc / 1e6:.0f} GB/s), "
            f"decode {dec:.3f} ms ({a.n * b / dec / 1e6:.0f} GB/s)")


def run_linear(a) -> str:
    from .nn import BpositLinear
    gen = torch.Generator(device="cuda").manual_seed(a.seed)
    lin = BpositLinear(a.K, a.N, bias=True, device="cuda")
    with torch.no_grad():
        lin.weight.copy_(torch.randn((a.N, a.K), device="cuda", generator=gen) * a.K ** -0.5)
    x = torch.randn((a.M, a.K), device="cuda", generator=gen)
    ms = _time(lambda: lin(x), a.calls)
    return (f"linear (W8A8 BpositLinear, fp32 out) M={a.M} N={a.N} K={a.K}: {ms:.3f} ms/call, "
            f"{2.0 * a.M * a.N * a.K / ms / 1e9:.1f} TOPS")


def run_qwen05(a) -> str:
    from .forward import qwen05, synthetic_ids
    model = qwen05(layers=a.layers, bposit=not a.fp32)
    ids = synthetic_ids(a.batch, a.seq, seed=a.seed)
    ms = _time(lambda: model(ids), a.calls)
    tok = a.batch * a.seq
    return (f"qwen05-shaped forward ({'fp32 torch linears' if a.fp32 else 'bp8 W8A8 exact-quire linears'}) "
            f"batch={a.batch} seq={a.seq} layers={a.layers}: {ms:.2f} ms, {tok / ms * 1e3:.0f} tokens/s, "
            f"linears {model.linear_ops(tok) / ms / 1e9:.1f} TOPS over the whole forward")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m bposit_b200.run")
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("M", type=int)
    g.add_argument("N", type=int)
    g.add_argument("K", type=int)
    g.add_argument("--fmt", default="bp8", choices=["bp8", "bp16"])
    g.add_argument("--group", type=int, default=0, help="per-group power-of-two scales (bp8)")
    g.add_argument("--algo", type=int, default=0)
    g.add_argument("--timeline", action="store_true", help="print the kernel timeline of one more call")
    c = sub.add_parser("codec")
    c.add_argument("n", type=int)
    c.add_argument("--fmt", default="bp8", choices=["bp8", "bp16"])
    w = sub.add_parser("qwen05")
    w.add_argument("--batch", type=int, default=8)
    w.add_argument("--seq", type=int, default=1024)
    w.add_argument("--layers", type=int, default=24)
    w.add_argument("--fp32", action="store_true", help="plain torch fp32 linears, for comparison")
    li = sub.add_parser("linear")
    li.add_argument("M", type=int)
    li.add_argument("N", type=int)
    li.add_argument("K", type=int)
    for p in (g, c, w, li):
        p.add_argument("--calls", type=int, default=3)
        p.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("no CUDA device")
    fn = {"gemm": run_gemm, "codec": run_codec, "qwen05": run_qwen05, "linear": run_linear}[a.what]
    print(fn(a), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
