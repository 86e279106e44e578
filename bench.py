#!/usr/bin/env python3
"""Benchmark of the b-posit W8A8 hot path on B200.

Headline (one JSON line on rank 0): bit-exact bp8 quire-GEMM throughput in
TOPS (2*M*N*K / time) on the large bp8 GEMM M=4096, N=4096, K=65536 with
operands N(0,1) * 2^U{-8..8} per row (seeded, synthetic), the output split into
blocks over a pm x pn grid of ranks (chosen by dist.choose_grid) and the
bposit32 result all-gathered by the GEMM's finish kernel itself (NVLink peer
stores; --gather nccl for N shards and an NCCL all-gather).

The same line carries, under "configs", one sub-line per other benchmark
workload, each with its own metric, roofline, end-to-end figure and CPU
baseline:
  "1"     one bp8 W8A8 linear X[16,576] @ W[576,576]^T, per-group-128 scales (1 GPU)
  "2"     the encode/decode sweep, 2^28 fp32 per rank (weak scaling)
  "3"     the SmolLM2-135M-shaped projection set at M=2048 (1 GPU)
  "4"     the Qwen2.5-0.5B-shaped forward, batch 8 x 1024 tokens, every linear
          N-sharded over the ranks
  "5bp16" the bp16 8192^3 quire GEMM, output blocks over the ranks
--config X prints workload X alone as the line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config all|5bp8|1|2|3|4|5bp16]
                    [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the CPU oracle port (oracle/, all host threads) on a
bounded sample of the same workload: rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (REPO, os.path.join(REPO, "open-bposit_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

M_, N_, K_ = 4096, 4096, 65536
METRIC = "bit-exact bp8 W8A8 quire-GEMM TOPS (bp8 4096x4096x65536)"
WORKLOAD = ("bp8 exact quire GEMM M=4096 N=4096 K=65536, operands N(0,1)*2^U{-8..8} per row, "
            "RTN-quantized; one bposit32 round per output; output blocks sharded over ranks, result all-gathered")
L2_FLUSH_BYTES = 256 << 20   # > the 126 MB L2


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def host_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


class Clocks:
    """SM clock and throttle reasons sampled every 20 ms by an NVML thread
    during a timed region (nvidia-smi at 200 ms is the fallback)."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, cuda_index: int):
        import threading
        self.idx = cuda_index
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = self.idx
        if vis:
            parts = [v.strip() for v in vis.split(",") if v.strip()]
            if self.idx < len(parts) and parts[self.idx].isdigit():
                idx = int(parts[self.idx])
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(idx)

    def _run(self, nv, h):
        bits = [(name, getattr(nv, attr, 0)) for name, attr in self.REASONS]
        while not self._stop.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, b in bits:
                    if b and (r & b):
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.02)

    def prepare(self):
        """The slow part of start() (NVML initialisation, several ms): done
        before the ranks' barrier, so that start() at the timed region's
        opening costs only a thread start and no rank begins late (a rank's
        late start shows up on every other rank as time spent waiting in the
        step's collectives)."""
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._nv = (nv, h)
        except Exception:
            self._nv = None
            self._start_smi()   # the fallback samples from here on (every 200 ms)
        return self

    def start(self):
        import threading
        if not hasattr(self, "_nv"):
            self.prepare()
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, args=self._nv, daemon=True)
            self._thread.start()
        return self

    def _start_smi(self):
        try:
            self._path = os.path.join("/tmp", f"bposit_clocks_{os.getpid()}.csv")
            self._fh = open(self._path, "w")
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self._fh, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self._proc = None

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            self._fh.close()
            for line in open(self._path):
                f = [x.strip() for x in line.split(",")]
                try:
                    self.samples.append(float(f[0]))
                    self.max_mhz = float(f[1])
                except (ValueError, IndexError):
                    continue
                for (name, _), v in zip(self.REASONS, f[2:6]):
                    if v.lower() == "active":
                        self.reasons.add(name)
            os.unlink(self._path)
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


class Ctx:
    """Process-wide state of one bench run (one process per GPU)."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.args, self.torch, self.dist = args, torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.device)
        self.peaks, self.peak_src = load_peaks()
        self.int8_peak = 2.0 * self.peaks["bf16_tflops"]
        self._flush = None

    def sync_all(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()

    def max_ranks(self, vals):
        if self.world == 1:
            return [float(v) for v in vals]
        t = self.torch.tensor([float(v) for v in vals], device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def flush_l2(self):
        if self._flush is None:
            self._flush = self.torch.empty(L2_FLUSH_BYTES, dtype=self.torch.uint8, device=self.device)
        self._flush.fill_(0x5A)

    def stream(self):
        return self.torch.cuda.current_stream()

    def timed(self, fn, steps, warmup, flush=False):
        """Device time per step of fn (ms, max over ranks) over `steps` timed
        steps after `warmup` untimed ones, bracketed by a barrier and a
        synchronize; with flush=True the L2 is flushed before every step and
        only the step itself is timed.  Also returns the clock record of the
        timed region (local rank 0) and the library's kernel launches in it."""
        from bposit_b200 import _lib
        torch = self.torch
        for _ in range(warmup):
            if flush:
                self.flush_l2()
            fn()
        clocks = Clocks(self.local).prepare() if self.local == 0 else None
        self.sync_all()
        if clocks is not None:
            clocks.start()
        n0 = _lib.lib().bp_launch_count()
        st = self.stream()
        if flush:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for a, b in evs:
                self.flush_l2()
                a.record(st)
                fn()
                b.record(st)
            launches = _lib.lib().bp_launch_count() - n0
            self.sync_all()
            ms = sum(a.elapsed_time(b) for a, b in evs) / steps
        else:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            for _ in range(steps):
                fn()
            b.record(st)
            launches = _lib.lib().bp_launch_count() - n0
            self.sync_all()
            ms = a.elapsed_time(b) / steps
        clk = clocks.stop() if clocks else None
        (ms,) = self.max_ranks([ms])
        return ms, clk, int(launches)

    def check_device(self):
        from bposit_b200 import ops
        ops.check_device_error()


def kernel_breakdown(ctx, fn, steps=2):
    """Device time per step of every kernel fn launches (ms), from the CUDA
    activity trace of torch.profiler over `steps` extra untimed steps (never
    the timed ones); grouped by kernel family.  None when tracing is
    unavailable."""
    torch = ctx.torch
    try:
        from torch.profiler import ProfilerActivity, profile
        ctx.sync_all()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(steps):
                fn()
            torch.cuda.synchronize()
        ctx.sync_all()
        groups = {}
        for ev in prof.events():
            if str(getattr(ev, "device_type", "")).split(".")[-1] != "CUDA":
                continue
            name = ev.name
            key = next((g for g, pats in (
                ("prep", ("k_tc_prep",)), ("gemm", ("k_quire_gemm_tc", "k_quire_gemm_simt")),
                ("tail_corr", ("k_tc_corr",)), ("kmajor_copy", ("k_kmajor",)), ("finish", ("k_tc_finish",)),
                ("fixup", ("k_tc_fixup",)),
                ("row_stats", ("k_row_stats",)), ("nccl", ("nccl",)), ("memcpy", ("Memcpy", "memcpy")),
                ("memset", ("Memset", "memset"))) if any(p in name for p in pats)), "other")
            dt = ev.time_range.elapsed_us()          # a device-side event: the kernel's own duration
            groups[key] = groups.get(key, 0.0) + dt / 1e3 / steps
        return {k: round(v, 4) for k, v in sorted(groups.items())}
    except Exception as e:   # tracing is a diagnostic: never fail the bench for it
        return {"unavailable": str(e)[:120]}


def as_graph(ctx, step, outputs):
    """(replay, info): `step` captured into a CUDA graph (after the eager
    warm-up that allocates every buffer), its replay checked against the eager
    step's outputs word for word; on any failure the eager step itself and the
    reason."""
    torch = ctx.torch
    try:
        step()
        torch.cuda.synchronize()
        ref = [o.clone() for o in outputs()]
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()                      # warm-up on the capture stream
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            step()
        for o in outputs():
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        same = all(torch.equal(a.view(torch.int32) if a.element_size() == 4 else a, b.view(torch.int32)
                               if b.element_size() == 4 else b) for a, b in zip(ref, outputs()))
        if not same:
            return step, {"cuda_graph": False, "why": "replay differs from the eager step"}, None
        return g.replay, {"cuda_graph": True, "replay_matches_eager": True}, g
    except Exception as e:   # capture is an optimisation: fall back to the eager step
        torch.cuda.synchronize()
        return step, {"cuda_graph": False, "why": f"{type(e).__name__}: {e}"[:200]}, None


def gather_obj(ctx, obj):
    if ctx.world == 1:
        return [obj]
    out = [None] * ctx.world
    ctx.dist.all_gather_object(out, obj)
    return out


def par_oracle(fn, chunks, threads):
    """fn over chunks on `threads` host threads (the oracle's ctypes calls
    release the GIL)."""
    if threads <= 1:
        return [fn(c) for c in chunks]
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(threads) as ex:
        return list(ex.map(fn, chunks))


def base_line(ctx, metric, unit, value, ms, steps, warmup, config, scaling, dtype="u8"):
    return {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": ctx.world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config}


def tensor_roofline(ctx, achieved_tops, kernel, note, slice_pairs=None, traffic=None, traffic_note=None):
    r = {"bound": "tensor", "achieved": round(achieved_tops, 3), "peak": round(ctx.int8_peak, 1), "unit": "TOPS",
         "frac": round(achieved_tops / ctx.int8_peak, 5), "traffic": traffic,
         "peak_source": f"int8 dense = 2 x {ctx.peak_src} bf16 {ctx.peaks['bf16_tflops']} TF/s",
         "kernel": kernel, "note": note}
    if slice_pairs:
        r.update({"slice_pairs_per_useful_mac": slice_pairs,
                  "issued_int8_TOPS": round(achieved_tops * slice_pairs, 1),
                  "issued_frac": round(achieved_tops * slice_pairs / ctx.int8_peak, 4)})
    if traffic_note:
        r["traffic_note"] = traffic_note
    return r


# ============================================================ workloads ===
def make_operand(ops, torch, rows, K, gen, device, fmt=8):
    """bp8 RTN / bp16 RTNE codes of N(0,1) * 2^U{-8..8} per row (in chunks)."""
    out = torch.empty((rows, K), dtype=torch.uint8 if fmt == 8 else torch.uint16, device=device)
    step = max(1, (1 << 27) // K)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        x = torch.randn((r1 - r0, K), device=device, generator=gen)
        e = torch.randint(-8, 9, (r1 - r0, 1), device=device, generator=gen).float()
        if fmt == 8:
            ops.quantize_bp8(x * torch.exp2(e), nearest=True, out=out[r0:r1])
        else:
            ops.encode_bp16(x * torch.exp2(e), rtne=True, out=out[r0:r1])
    return out


def host_operand(rows, K, seed, fmt=8):
    """The same distribution generated on the host (oracle samples)."""
    import numpy as np
    from oracle import oracle as orc
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, K)) * np.exp2(rng.integers(-8, 9, (rows, 1)))).astype(np.float32)
    return orc.quantize_bp8(x)[0] if fmt == 8 else orc.encode_bp16(x, True)


def cpu_gemm_rate(A, B, fmt, target_s, threads):
    """Oracle quire GEMM (threads over rows) on growing row samples of A until
    about target_s seconds: (TOPS, rows, seconds)."""
    from oracle import oracle as orc
    n = min(max(1, threads), A.shape[0])
    t0 = time.perf_counter()
    orc.quire_gemm(A[:n], B, fmt, nthreads=threads)
    dt = time.perf_counter() - t0
    rows = n
    reps = int(round(target_s / max(dt, 1e-6)))
    if reps > 1:
        rows = min(A.shape[0], n * reps)
        t0 = time.perf_counter()
        orc.quire_gemm(A[:rows], B, fmt, nthreads=threads)
        dt = time.perf_counter() - t0
    return 2.0 * rows * B.shape[0] * B.shape[1] / dt / 1e12, rows, dt


def gemm_cpu_baseline(A, B, fmt, M, N, K, all_s=10.0, one_s=4.0):
    threads = host_threads()
    v, rows, dt = cpu_gemm_rate(A, B, fmt, all_s, threads)
    v1, rows1, dt1 = cpu_gemm_rate(A, B, fmt, one_s, 1)
    return {"value": v, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{rows} of {M} rows x N={N} x K={K} ({dt:.1f} s, oracle port, {threads} threads)",
            "one_core": {"value": v1, "unit": "TOPS", "cores": 1,
                         "sample": f"{rows1} rows ({dt1:.1f} s)"}}


# ---------------------------------------------------- 5bp8: the headline ---
def run_headline(ctx, fmt=8, M=M_, N=N_, K=K_):
    """The large quire GEMM (bp8 4096x4096x65536, or bp16 8192^3 with fmt=16),
    output blocks over the ranks, all-gathered."""
    import numpy as np  # noqa: F401
    torch, args = ctx.torch, ctx.args
    from bposit_b200 import ops
    from bposit_b200.dist import FusedShardedQuireGemm, ShardedQuireGemm, assemble

    gen = torch.Generator(device=ctx.device).manual_seed(0 if fmt == 8 else 2)
    A = make_operand(ops, torch, M, K, gen, ctx.device, fmt)
    B = make_operand(ops, torch, N, K, gen, ctx.device, fmt)
    fused = args.gather == "fused"
    if fused:
        g = FusedShardedQuireGemm(M, N, ctx.device, algo=args.algo, K=K, fmt=fmt)
        m0, m1, n0, n1 = g.block
        grid = g.grid
    else:
        g = ShardedQuireGemm(M, N, ctx.device, algo=args.algo, fmt=fmt)
        (n0, n1), (m0, m1), grid = g.plan.bounds, (0, M), (1, ctx.world)
    A_full, B_full = A, B
    A = A_full[m0:m1].contiguous()
    Bs = B[n0:n1].contiguous()
    del B
    ws = torch.empty(max(256, ops.gemm_workspace_size(fmt, m1 - m0, n1 - n0, K, args.algo)), dtype=torch.uint8,
                     device=ctx.device)
    peers = [p + 4 * m0 * N for p in g.peer_ptrs] if fused else []
    kev = []

    def shard_step(A_, B_, rec=False):
        if fused and ctx.world > 1:
            ctx.dist.all_reduce(g.flag)
        if rec:
            kev.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
            kev[-1][0].record(ctx.stream())
        if fused:
            ops.quire_gemm_multi(A_, B_, g.result[m0:m1, n0:n1], peers, n0, fmt=fmt, algo=args.algo, workspace=ws)
        else:
            ops.quire_gemm(A_, B_, fmt, out=g.local[:, :n1 - n0] if ctx.world > 1 else g.result, algo=args.algo,
                           workspace=ws)
        if rec:
            kev[-1][1].record(ctx.stream())
        if ctx.world > 1:
            if fused:
                ctx.dist.all_reduce(g.flag)
            else:
                ctx.dist.all_gather_into_tensor(g.gathered.view(-1).view(torch.int32),
                                                g.local.view(-1).view(torch.int32))
                assemble(g.gathered, g.plan, g.result)
        return g.result

    steps = args.steps
    ms, clk, launches = ctx.timed(lambda: shard_step(A, Bs, rec=True), steps, args.warmup)
    kev = kev[-steps:]
    (kms,) = ctx.max_ranks([statistics.mean(a.elapsed_time(b) for a, b in kev)])
    ctx.check_device()
    tops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    k_tops = 2.0 * (m1 - m0) * (n1 - n0) * K / (kms * 1e-3) / 1e12
    # int8 MMAs per useful MAC: 4 in the narrow bp8 form (unscaled, K >= 16384 or
    # algo 4), 9 in the wide bp8 form, 16 for bp16
    narrow = fmt == 8 and args.algo in (0, 2, 3, 4) and (K >= 16384 or args.algo == 4)
    slice_pairs = (16 if fmt == 16 else (4 if narrow else 9)) \
        if ops.gemm_workspace_size(fmt, m1 - m0, n1 - n0, K, 2) and args.algo != 1 else None
    breakdown = kernel_breakdown(ctx, lambda: shard_step(A, Bs))
    per_rank = gather_obj(ctx, breakdown)
    nccl_variant = None
    if ctx.world > 1 and fused:
        # the same workload with N shards and one NCCL all-gather (+ local transpose)
        g2 = ShardedQuireGemm(M, N, ctx.device, algo=args.algo, fmt=fmt)
        a0, a1 = g2.plan.bounds
        Bn = B_full[a0:a1].contiguous()
        ws2 = torch.empty(max(256, ops.gemm_workspace_size(fmt, M, a1 - a0, K, args.algo)), dtype=torch.uint8,
                          device=ctx.device)
        ms2, _, _ = ctx.timed(lambda: g2(A_full, Bn), max(3, steps // 2), args.warmup)
        nccl_variant = {"value": round(2.0 * M * N * K / (ms2 * 1e-3) / 1e12, 3), "unit": "TOPS",
                        "ms_per_step": round(ms2, 3), "layout": f"1x{ctx.world} N shards + NCCL all_gather_into_tensor"}
        del g2, Bn, ws2
    del B_full
    torch.cuda.empty_cache()

    # end to end with host buffers (pinned): one GPU through bp_quire_gemm_host;
    # several through H2D of each rank's blocks, the sharded step and a D2H of the result
    hA = A.cpu().pin_memory()
    hB = Bs.cpu().pin_memory()
    hOut = torch.empty((M, N), dtype=torch.uint32).pin_memory()
    dA = torch.empty_like(A)
    dB = torch.empty_like(Bs)

    def e2e_step():
        if ctx.world == 1:
            ops.quire_gemm_host(hA, hB, fmt, out=hOut, algo=args.algo)
            return
        dA.copy_(hA, non_blocking=True)
        dB.copy_(hB, non_blocking=True)
        shard_step(dA, dB)
        hOut.copy_(g.result, non_blocking=True)

    ems, _, _ = ctx.timed(e2e_step, max(1, min(steps, 5)), 1)
    ctx.check_device()
    e2e_ok = bool(torch.equal(hOut.view(torch.int32), g.result.cpu().view(torch.int32))) if ctx.world == 1 else None
    e2e_tops = 2.0 * M * N * K / (ems * 1e-3) / 1e12
    hs, ht = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hs.record(ctx.stream())
    dA.copy_(hA, non_blocking=True)
    ht.record(ctx.stream())
    torch.cuda.synchronize()
    h2d_gbs = A.numel() * A.element_size() / (hs.elapsed_time(ht) * 1e-3) / 1e9
    del hA, hB, dA, dB

    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        An = A_full[:min(M, 512)].cpu().numpy()
        Bn = Bs.cpu().numpy()
        cpu = gemm_cpu_baseline(An, Bn, fmt, M, N, K, all_s=12.0 if fmt == 8 else 6.0,
                                one_s=4.0 if fmt == 8 else 3.0)

    traffic, traffic_note = None, "no capture at this shape"
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            tj = json.load(f)
        # the bp8 tensor-core call takes the narrow two-plane form for K >= 16384
        # (algo 0, 2, 3, 4), else the wide one; each has its own capture
        narrow = fmt == 8 and args.algo in (0, 2, 3, 4) and (K >= 16384 or args.algo == 4)
        ent = tj.get(f"quire_gemm_{'tc' if args.algo != 1 else 'simt'}" + ("" if fmt == 8 else "_bp16") +
                     ("_narrow" if narrow and args.algo != 1 else ""))
        if ent and ent.get("shape") == [m1 - m0, n1 - n0, K]:
            traffic = ent["dram_bytes_per_call"]
            traffic_note = ent.get("note", "DRAM bytes read+written by one call (ncu)")
    fname = "bp8" if fmt == 8 else "bp16"
    workload = WORKLOAD if fmt == 8 else ("bp16 exact quire GEMM M=N=K=8192, operands N(0,1)*2^U{-8..8} per row, "
                                          "RTNE-encoded; one bposit32 round per output; output blocks sharded "
                                          "over ranks, result all-gathered")
    metric = METRIC if fmt == 8 else "bit-exact bp16 quire-GEMM TOPS (bp16 8192^3)"
    config = {"workload": workload, "M": M, "N": N, "K": K, "fmt": fname,
              "l2": f"inputs {(M + N) * K * fmt // 8 >> 20} MiB > L2 (no flush needed)", "ranks": ctx.world}
    line = base_line(ctx, metric, "TOPS", tops, ms, steps, args.warmup, config, "strong")
    line.update({
        "layout": (f"{grid[0]}x{grid[1]} (M x N) block grid over {ctx.world} ranks + " +
                   ("all-gather fused into the GEMM's finish kernel (NVLink peer stores)" if fused
                    else "NCCL all-gather") + f"; algo {args.algo}"),
        "roofline": tensor_roofline(ctx, k_tops, "quire GEMM (all launches of one bp_quire_gemm call)",
                                    "achieved = useful 2MNK of this rank's block / device time of its GEMM call",
                                    slice_pairs, traffic, traffic_note),
        "e2e": {"value": round(e2e_tops, 3), "unit": "TOPS", "ms_per_step": round(ems, 3),
                "h2d_bytes_per_step": int(((m1 - m0) + (n1 - n0)) * K * fmt // 8),
                "d2h_bytes_per_step": int(M * N * 4), "h2d_link_gbs": round(h2d_gbs, 1),
                "matches_device_result": e2e_ok},
        "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clk,
        "nccl_gather_variant": nccl_variant,
        "breakdown_ms_per_step": {"rank0": per_rank[0], "per_rank": per_rank if ctx.world > 1 else None,
                                  "how": "CUDA activity trace (torch.profiler) of 2 extra untimed steps"},
    })
    line["roofline"]["kernel_ms"] = round(kms, 3)
    if fused:
        g.close()
    del A, A_full, Bs, ws
    torch.cuda.empty_cache()
    return line


# ------------------------------------------------- config 1: W8A8 linear ---
def run_c1(ctx):
    torch, args = ctx.torch, ctx.args
    import numpy as np
    from bposit_b200 import ops, workloads
    X, W = workloads.w8a8_linear(seed=0)
    M, K = X.shape
    N = W.shape[0]
    dX, dW = torch.from_numpy(X).to(ctx.device), torch.from_numpy(W).to(ctx.device)
    G = (K + 127) // 128
    xc = torch.empty((M, K), dtype=torch.uint8, device=ctx.device)
    wc = torch.empty((N, K), dtype=torch.uint8, device=ctx.device)
    out = torch.empty((M, N), dtype=torch.uint32, device=ctx.device)
    ws = torch.empty(max(256, ops.gemm_workspace_size(8, M, N, K)), dtype=torch.uint8, device=ctx.device)

    def step(x=dX, w=dW):
        _, sx = ops.quantize_bp8_grouped(x, group=128, out=xc)
        _, sw = ops.quantize_bp8_grouped(w, group=128, out=wc)
        ops.quire_gemm(xc, wc, 8, sa=sx, sb=sw, group=128, out=out, workspace=ws)

    steps = max(50, 10 * args.steps)
    run, ginfo, _graph = as_graph(ctx, step, lambda: [xc, wc, out])
    ms, clk, launches = ctx.timed(run, steps, max(args.warmup, 10), flush=True)
    ctx.check_device()
    ops_ = 2.0 * M * N * K
    hX, hW = torch.from_numpy(X).pin_memory(), torch.from_numpy(W).pin_memory()
    hOut = torch.empty((M, N), dtype=torch.uint32).pin_memory()
    eX, eW = torch.empty_like(dX), torch.empty_like(dW)

    def e2e():
        eX.copy_(hX, non_blocking=True)
        eW.copy_(hW, non_blocking=True)
        step(eX, eW)
        hOut.copy_(out, non_blocking=True)

    ems, _, _ = ctx.timed(e2e, steps, 10, flush=True)
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        from oracle import oracle as orc

        def oracle_step(threads):
            sx, sw = orc.group_scales(X), orc.group_scales(W)
            a, b = orc.quantize_bp8_grouped(X, sx), orc.quantize_bp8_grouped(W, sw)
            return orc.quire_gemm(a, b, 8, sa=sx, sb=sw, nthreads=threads)

        res = {}
        for th in (host_threads(), 1):
            ref = oracle_step(th)
            n, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < 2.0:
                oracle_step(th)
                n += 1
            res[th] = (ops_ * n / (time.perf_counter() - t0) / 1e12, n)
        assert np.array_equal(ref, out.cpu().numpy()), "config 1: device result differs from the oracle"
        th = host_threads()
        cpu = {"value": res[th][0], "unit": "TOPS", "cores": th, "kind": "port",
               "sample": f"the whole 16x576x576 linear (scales, quantize, GEMM), {res[th][1]} runs",
               "one_core": {"value": res[1][0], "unit": "TOPS", "cores": 1, "sample": f"{res[1][1]} runs"},
               "bit_exact_vs_device": True}
    config = {"workload": "bp8 W8A8 linear X[16,576] (N(0,1), 1% N(0,20^2) outliers) @ W[576,576]^T (N(0,0.02^2)), "
                          "per-group-128 power-of-two scales, RTN, exact quire, one bposit32 round",
              "M": M, "N": N, "K": K, "fmt": "bp8", "l2": "L2 flushed (256 MiB write) before every timed step",
              "ranks": 1}
    line = base_line(ctx, "bp8 W8A8 linear TOPS (16x576x576, group-128 scales, quantize + GEMM)", "TOPS",
                     ops_ / (ms * 1e-3) / 1e12, ms, steps, max(args.warmup, 10), config, "strong")
    line.update({
        "graph": ginfo,
        "roofline": tensor_roofline(ctx, ops_ / (ms * 1e-3) / 1e12, "whole step (2 grouped quantizes + GEMM)",
                                    "latency-bound: 5 kernels for 5.3 M MACs"),
        "e2e": {"value": round(ops_ / (ems * 1e-3) / 1e12, 4), "unit": "TOPS", "ms_per_step": round(ems, 4),
                "h2d_bytes_per_step": int((M + N) * K * 4), "d2h_bytes_per_step": int(M * N * 4)},
        "cpu_baseline": cpu, "gpu_launches": launches if not ginfo["cuda_graph"] else 5 * steps, "clocks": clk})
    return line


# -------------------------------------------------- config 2: codec sweep ---
def codec_input(ctx, n, lim):
    """The sweep's values for a format whose range is 2^+-lim: half N(0,1), half
    log-uniform magnitudes over 2^+-(lim + 2) with random signs, and, at the
    start, +-0, the saturation edges (+-maxpos, twice it, +-minpos, a quarter of
    it), exact midpoints of the bp8 grid (ties) and powers of two."""
    torch = ctx.torch
    gen = torch.Generator(device=ctx.device).manual_seed(1234 + ctx.rank + lim)
    x = torch.empty(n, dtype=torch.float32, device=ctx.device)
    half = n // 2
    x[:half].normal_(generator=gen)
    e = torch.empty(n - half, dtype=torch.float32, device=ctx.device).uniform_(-lim - 2, lim + 2, generator=gen)
    x[half:] = torch.exp2(e) * torch.where(torch.rand(n - half, device=ctx.device, generator=gen) < 0.5, -1.0, 1.0)
    del e
    m = 2.0 ** lim
    edges = [0.0, -0.0, m, -m, 2 * m, -2 * m, 1 / m, -1 / m, 0.25 / m, -0.25 / m, 1.0, -1.0, 1.5, 1.0625, 1.03125,
             1.09375, 3 / m, 12.0, -12.0, 0.75]
    x[:len(edges)] = torch.tensor(edges, dtype=torch.float32, device=ctx.device)
    return x


def run_c2(ctx):
    """2^28 fp32 per rank: bp8 RTN encode, bp8 decode, bp16 RTNE encode, bp16
    decode; plus plain copy / fill / read kernels of torch on the same buffers
    as the attainable-bandwidth markers."""
    torch, args = ctx.torch, ctx.args
    import ctypes

    from bposit_b200 import _lib, ops
    n = 1 << 28
    x = codec_input(ctx, n, 24)       # bp8's range 2^+-24
    x16 = codec_input(ctx, n, 112)    # bp16's range 2^+-112
    c8 = torch.empty(n, dtype=torch.uint8, device=ctx.device)
    c16 = torch.empty(n, dtype=torch.uint16, device=ctx.device)
    y = torch.empty(n, dtype=torch.float32, device=ctx.device)
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731

    def dec(codes):
        f = 8 if codes.dtype == torch.uint8 else 16
        _lib.check(_lib.lib().bp_decode(f, ctypes.c_void_p(codes.data_ptr()), codes.numel(),
                                        ctypes.c_void_p(y.data_ptr()), st()))

    kernels = {
        "bp8_encode_rtn": (lambda: ops.quantize_bp8(x, nearest=True, out=c8), 5),
        "bp8_decode": (lambda: dec(c8), 5),
        "bp16_encode_rtne": (lambda: ops.encode_bp16(x16, rtne=True, out=c16), 6),
        "bp16_decode": (lambda: dec(c16), 6),
    }
    markers = {
        "torch_copy_f32": (lambda: y.copy_(x), 8),
        "torch_fill_f32": (lambda: y.fill_(1.0), 4),
        "torch_amax_f32": (lambda: torch.amax(x), 4),
    }
    steps = max(10, args.steps)
    res, tot_b, tot_ms, clk0, launches = {}, 0.0, 0.0, None, 0
    for name, (fn, bpe) in list(kernels.items()) + list(markers.items()):
        ms, clk, nl = ctx.timed(fn, steps, args.warmup)
        gbs = bpe * n * ctx.world / (ms * 1e-3) / 1e9
        res[name] = {"GB/s": round(gbs, 1), "ms": round(ms, 4), "bytes_per_elem": bpe,
                     "frac_of_measured_hbm_per_gpu": round(gbs / ctx.world / ctx.peaks["hbm_gbs"], 4)}
        if name in kernels:
            tot_b += bpe * n * ctx.world
            tot_ms += ms
            launches += nl
            clk0 = clk0 or clk
    value = tot_b / (tot_ms * 1e-3) / 1e9
    dom = max(kernels, key=lambda k: res[k]["ms"])
    # end to end: host fp32 in (pinned), bp8 RTN codes out, through the public API
    hx = x.cpu().pin_memory()
    hc = torch.empty(n, dtype=torch.uint8).pin_memory()
    dx = torch.empty_like(x)

    def e2e():
        dx.copy_(hx, non_blocking=True)
        ops.quantize_bp8(dx, nearest=True, out=c8)
        hc.copy_(c8, non_blocking=True)

    ems, _, _ = ctx.timed(e2e, 3, 1)
    del hx, hc, dx
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        cpu = codec_cpu_baseline(x[: 1 << 22].cpu().numpy(), x16[: 1 << 22].cpu().numpy())
    del x, x16, c8, c16, y
    torch.cuda.empty_cache()
    config = {"workload": "2^28 fp32 per rank and format: half N(0,1), half log-uniform magnitudes over the format's "
                          "range (bp8 2^+-26, bp16 2^+-114) with +-0, saturation edges and exact ties; bp8 RTN "
                          "encode, bp8 decode, bp16 RTNE encode, bp16 decode (of the codes just encoded)",
              "elements_per_rank": n, "fmt": "bp8+bp16", "l2": "1 GiB input > L2", "ranks": ctx.world}
    line = base_line(ctx, "bp8/bp16 encode+decode GB/s (algorithmic bytes, 4 kernels)", "GB/s", value,
                     tot_ms, steps, args.warmup, config, "weak", dtype="f32/u8/u16")
    d = res[dom]
    line.update({
        "roofline": {"bound": "hbm", "achieved": d["GB/s"] / ctx.world, "peak": ctx.peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": d["frac_of_measured_hbm_per_gpu"], "traffic": None, "kernel": dom,
                     "peak_source": f"{ctx.peak_src} HBM copy bandwidth",
                     "note": "the kernel with the longest time; every kernel's figure under 'kernels'"},
        "kernels": {k: res[k] for k in kernels}, "attainable_markers": {k: res[k] for k in markers},
        "e2e": {"value": round(5 * n * ctx.world / (ems * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(ems, 3), "what": "bp8 RTN encode: pinned fp32 in, codes out",
                "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": n},
        "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clk0})
    return line


def codec_cpu_baseline(xs, xs16):
    """The oracle port's quantize_bp8(nearest=True) and bp16 RTNE encode on
    seeded 2^22-element samples of the sweep, all host threads and one."""
    import numpy as np
    from oracle import oracle as orc
    th = host_threads()
    out = {}
    for name, fn, bpe, src in (("bp8_encode_rtn", lambda c: orc.quantize_bp8(c, True), 5, xs),
                               ("bp16_encode_rtne", lambda c: orc.encode_bp16(c, True), 6, xs16)):
        chunks = np.array_split(src, max(1, th * 4))
        for t in (th, 1):
            t0 = time.perf_counter()
            reps = 0
            while True:
                par_oracle(fn, chunks, t)
                reps += 1
                if time.perf_counter() - t0 > 2.0:
                    break
            out[(name, t)] = bpe * xs.size * reps / (time.perf_counter() - t0) / 1e9
    v = 11 * xs.size / (5 * xs.size / out[("bp8_encode_rtn", th)] + 6 * xs.size / out[("bp16_encode_rtne", th)])
    v1 = 11 * xs.size / (5 * xs.size / out[("bp8_encode_rtn", 1)] + 6 * xs.size / out[("bp16_encode_rtne", 1)])
    return {"value": v, "unit": "GB/s", "cores": th, "kind": "port",
            "sample": f"{xs.size} elements of the sweep: bp8 RTN and bp16 RTNE encodes (the oracle port has no "
                      "separate decode cost worth timing: a table read)",
            "per_kernel_GBps": {k[0]: round(v_, 3) for k, v_ in out.items() if k[1] == th},
            "one_core": {"value": v1, "unit": "GB/s", "cores": 1,
                         "per_kernel_GBps": {k[0]: round(v_, 3) for k, v_ in out.items() if k[1] == 1}}}


# -------------------------------------------- config 3: SmolLM layer set ---
def run_c3(ctx):
    torch, args = ctx.torch, ctx.args
    from bposit_b200 import ops, workloads
    M = 2048
    gen = torch.Generator(device=ctx.device).manual_seed(3)
    layers = []
    for name, N, K in workloads.SMOLLM_SHAPES:
        X = torch.randn((M, K), device=ctx.device, generator=gen)
        W = torch.randn((N, K), device=ctx.device, generator=gen) * 0.02
        wc, sw = ops.quantize_bp8_grouped(W, group=128)
        layers.append({"name": name, "N": N, "K": K, "X": X, "wc": wc, "sw": sw,
                       "xc": torch.empty((M, K), dtype=torch.uint8, device=ctx.device),
                       "out": torch.empty((M, N), dtype=torch.uint32, device=ctx.device),
                       "ws": torch.empty(max(256, ops.gemm_workspace_size(8, M, N, K)), dtype=torch.uint8,
                                         device=ctx.device)})
    total_ops = sum(2.0 * M * L["N"] * L["K"] for L in layers)

    def step(xs=None):
        for i, L in enumerate(layers):
            _, sx = ops.quantize_bp8_grouped(L["X"] if xs is None else xs[i], group=128, out=L["xc"])
            ops.quire_gemm(L["xc"], L["wc"], 8, sa=sx, sb=L["sw"], group=128, out=L["out"], workspace=L["ws"])

    steps = max(10, args.steps)
    eager_launches = None
    n0 = None
    try:
        from bposit_b200 import _lib
        n0 = _lib.lib().bp_launch_count()
        step()
        torch.cuda.synchronize()
        eager_launches = _lib.lib().bp_launch_count() - n0
    except Exception:
        pass
    run, ginfo, _graph = as_graph(ctx, step, lambda: [L["out"] for L in layers])
    ms, clk, launches = ctx.timed(run, steps, args.warmup, flush=True)
    if ginfo["cuda_graph"] and eager_launches is not None:
        launches = eager_launches * steps
    ctx.check_device()
    hx = [L["X"].cpu().pin_memory() for L in layers]
    ho = [torch.empty(L["out"].shape, dtype=torch.uint32).pin_memory() for L in layers]
    dx = [torch.empty_like(L["X"]) for L in layers]

    def e2e():
        for h, d in zip(hx, dx):
            d.copy_(h, non_blocking=True)
        step(dx)
        for h, L in zip(ho, layers):
            h.copy_(L["out"], non_blocking=True)

    ems, _, _ = ctx.timed(e2e, steps, args.warmup, flush=True)
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        from oracle import oracle as orc
        th = host_threads()
        res = {}
        for t, rows in ((th, 16), (1, 4)):
            t0, macs = time.perf_counter(), 0.0
            for L in layers:
                xc = L["xc"][:rows].cpu().numpy()
                sx = ops.quantize_bp8_grouped(L["X"][:rows], group=128)[1].cpu().numpy()
                orc.quire_gemm(xc, L["wc"].cpu().numpy(), 8, sa=sx, sb=L["sw"].cpu().numpy(), nthreads=t)
                macs += rows * L["N"] * L["K"]
            res[t] = (2.0 * macs / (time.perf_counter() - t0) / 1e12, rows)
        cpu = {"value": res[th][0], "unit": "TOPS", "cores": th, "kind": "port",
               "sample": f"{res[th][1]} of {M} rows of each of the 7 projections (GEMM only)",
               "one_core": {"value": res[1][0], "unit": "TOPS", "cores": 1,
                            "sample": f"{res[1][1]} rows of each projection"}}
    config = {"workload": "SmolLM2-135M-shaped q/k/v/o/gate/up/down projections at M=2048, activations N(0,1), "
                          "weights N(0,0.02^2), per-group-128 scales; activation quantize + exact GEMM per step "
                          "(weights quantized once)",
              "M": M, "shapes_NK": [[L["N"], L["K"]] for L in layers], "fmt": "bp8",
              "l2": "L2 flushed (256 MiB write) before every timed step", "ranks": 1}
    line = base_line(ctx, "bp8 W8A8 projection-set TOPS (SmolLM2-135M shapes, M=2048)", "TOPS",
                     total_ops / (ms * 1e-3) / 1e12, ms, steps, args.warmup, config, "strong")
    line.update({
        "graph": ginfo,
        "roofline": tensor_roofline(ctx, total_ops / (ms * 1e-3) / 1e12, "whole step (7 x (quantize + GEMM))",
                                    "short K (576 / 1536) and small N: launch- and finish-bound"),
        "e2e": {"value": round(total_ops / (ems * 1e-3) / 1e12, 3), "unit": "TOPS", "ms_per_step": round(ems, 4),
                "h2d_bytes_per_step": int(sum(M * L["K"] * 4 for L in layers)),
                "d2h_bytes_per_step": int(sum(M * L["N"] * 4 for L in layers))},
        "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clk})
    return line


# ----------------------------------------- config 4: Qwen-shaped forward ---
def run_c4(ctx):
    torch, args = ctx.torch, ctx.args
    from bposit_b200.forward import qwen05, synthetic_ids
    batch, seq = 8, 1024
    model = qwen05(layers=24, device=ctx.device, seed=0)
    sharded = ctx.world > 1
    if sharded:
        from bposit_b200.nn import shard_linears
        shard_linears(model)
    ids = synthetic_ids(batch, seq, seed=0, device=ctx.device)
    tokens = batch * seq
    lin_ops = model.linear_ops(tokens)
    with torch.no_grad():
        model(ids)                    # weights are encoded on first use
    steps = max(3, args.steps // 4)
    holder = {}

    def fwd():
        holder["h"] = model(ids)

    ginfo = {"cuda_graph": False, "why": "sharded linears run eager (NCCL barriers and peer stores)"}
    run = fwd
    if not sharded:
        run, ginfo, _graph = as_graph(ctx, fwd, lambda: [holder["h"]])
    from bposit_b200 import _lib
    n0 = _lib.lib().bp_launch_count()
    fwd()
    torch.cuda.synchronize()
    per_fwd = _lib.lib().bp_launch_count() - n0
    ms, clk, launches = ctx.timed(run, steps, args.warmup)
    launches = per_fwd * steps
    ctx.check_device()
    hid = ids.cpu().pin_memory()
    hout = torch.empty((batch, seq, model.c["hidden"]), dtype=torch.float32).pin_memory()
    did = torch.empty_like(ids)

    def e2e():
        did.copy_(hid, non_blocking=True)
        hout.copy_(model(did), non_blocking=True)

    ems, _, _ = ctx.timed(e2e, steps, 1)
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu:
        import numpy as np
        from oracle import oracle as orc
        rng = np.random.default_rng(4)
        th = host_threads()
        shapes = [(lin.out_features, lin.in_features) for lin in (model.layers[0].qkv, model.layers[0].o,
                                                                     model.layers[0].gate_up, model.layers[0].down)]
        res = {}
        for t, rows in ((th, 16), (1, 2)):
            t0, macs = time.perf_counter(), 0.0
            for N, K in shapes:
                a = rng.integers(0, 256, (rows, K)).astype(np.uint8)
                b = rng.integers(0, 256, (N, K)).astype(np.uint8)
                orc.quire_gemm(a, b, 8, nthreads=t)
                macs += rows * N * K
            rate = macs / (time.perf_counter() - t0)            # MAC/s
            res[t] = (rate / (lin_ops / 2.0 / tokens), rows)     # tokens/s of the linears
        cpu = {"value": res[th][0], "unit": "tokens/s", "cores": th, "kind": "port",
               "sample": f"{res[th][1]} rows through each of the 4 linear shapes (linears only; the fp32 parts of "
                         "the forward are not included), scaled to tokens of the 24-layer stack",
               "one_core": {"value": res[1][0], "unit": "tokens/s", "cores": 1,
                            "sample": f"{res[1][1]} rows per linear shape"}}
    config = {"workload": "Qwen2.5-0.5B-shaped forward, random init: 24 layers, hidden 896, intermediate 4864, "
                          "14/2 heads, RMSNorm+RoPE fp32; batch 8 x seq 1024 uniform token ids; every linear a bp8 "
                          "W8A8 exact-quire GEMM (per-row recipe), qkv and gate/up fused along N",
              "batch": batch, "seq_len": seq, "fmt": "bp8", "ranks": ctx.world,
              "l2": "weights 358 MB of codes per forward > L2"}
    line = base_line(ctx, "Qwen2.5-0.5B-shaped W8A8 forward tokens/s (8 x 1024)", "tokens/s",
                     tokens / (ms * 1e-3), ms, steps, args.warmup, config, "strong", dtype="u8 (linears), f32")
    line.update({
        "graph": ginfo,
        "layout": ("every linear's N (output features) sharded over the ranks, bposit32 blocks all-gathered by the "
                   "GEMM's finish kernel; non-linear parts replicated" if sharded else "1 GPU"),
        "linear_TOPS": round(lin_ops / (ms * 1e-3) / 1e12, 3),
        "roofline": tensor_roofline(ctx, lin_ops / (ms * 1e-3) / 1e12, "whole forward",
                                    "achieved = decoder-linear useful ops / whole forward time (conservative)"),
        "e2e": {"value": round(tokens / (ems * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ems, 3),
                "h2d_bytes_per_step": int(tokens * 8), "d2h_bytes_per_step": int(tokens * model.c["hidden"] * 4)},
        "cpu_baseline": cpu, "gpu_launches": launches, "clocks": clk})
    del model
    if sharded:
        from bposit_b200.nn import close_sharded
        close_sharded()
    torch.cuda.empty_cache()
    return line


def run_c5bp16(ctx):
    return run_headline(ctx, fmt=16, M=8192, N=8192, K=8192)


RUNNERS = {"5bp8": run_headline, "1": run_c1, "2": run_c2, "3": run_c3, "4": run_c4, "5bp16": run_c5bp16}
SINGLE_GPU = ("1", "3")


def run_ours(args):
    ctx = Ctx(args)
    if args.config == "all":
        line = run_headline(ctx)
        subs = {}
        for c in ("1", "2", "3", "4", "5bp16"):
            if c in SINGLE_GPU and ctx.world > 1:
                continue
            try:
                subs[c] = RUNNERS[c](ctx)
            except Exception as e:   # a failing sub-workload is reported, not hidden, and the headline kept
                if ctx.world > 1:
                    raise
                subs[c] = {"error": f"{type(e).__name__}: {e}"[:300]}
        line["configs"] = subs
    else:
        line = RUNNERS[args.config](ctx)
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    if ctx.world > 1:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()
    return 0


def run_reference(args):
    """The CPU oracle port on the host cores, rank 0 only, on the headline's
    config (or --config's), each step a bounded sample."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    threads = host_threads()
    if args.config in ("all", "5bp8", "5bp16"):
        fmt, M, N, K = (8, M_, N_, K_) if args.config != "5bp16" else (16, 8192, 8192, 8192)
        rows_needed = max(64, 4 * threads)
        A = host_operand(rows_needed, K, 0, fmt)
        B = host_operand(N, K, 1, fmt)
        per_step = max(2.0, 60.0 / max(1, args.steps + args.warmup))
        from oracle import oracle as orc
        for _ in range(args.warmup):
            orc.quire_gemm(A[:1], B[:256], fmt, nthreads=threads)
        vals, rows_used, secs = [], 0, 0.0
        for _ in range(args.steps):
            v, rows_used, dt = cpu_gemm_rate(A, B, fmt, per_step, threads)
            vals.append(v)
            secs += dt
        value = statistics.median(vals)
        if fmt == 8:
            metric, workload = METRIC, WORKLOAD
        else:
            metric = "bit-exact bp16 quire-GEMM TOPS (bp16 8192^3)"
            workload = ("bp16 exact quire GEMM M=N=K=8192, operands N(0,1)*2^U{-8..8} per row, RTNE-encoded; one "
                        "bposit32 round per output; output blocks sharded over ranks, result all-gathered")
        config = {"workload": workload, "M": M, "N": N, "K": K, "fmt": "bp8" if fmt == 8 else "bp16",
                  "l2": f"inputs {(M + N) * K * fmt // 8 >> 20} MiB > L2 (no flush needed)", "ranks": world}
        sample = f"{rows_used} of {M} rows x N={N} x K={K} per step (oracle port, {threads} threads)"
        unit = "TOPS"
        ms = 1e3 * secs / max(1, args.steps)
    else:
        raise SystemExit(f"--impl reference supports the large-GEMM configs (5bp8, 5bp16), not {args.config}")
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u8" if fmt == 8 else "u16", "data": "synthetic",
        "config": config, "layout": f"host threads ({threads})",
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["all"] + list(RUNNERS), default="all",
                    help="all = the headline line (5bp8) carrying every other workload under 'configs'")
    ap.add_argument("--algo", type=int, default=0, help="0 auto, 1 CUDA cores, 2 tensor cores")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline legs")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="all-gather of the output blocks: in the GEMM's finish kernel (peer stores, M x N rank grid) "
                         "or NCCL (N shards)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
