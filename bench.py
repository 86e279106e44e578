#!/usr/bin/env python3
"""Benchmark of the b-posit W8A8 hot path on B200.

Headline (one JSON line on rank 0): bit-exact bp8 quire-GEMM throughput in
TOPS (2*M*N*K / time) on the large bp8 GEMM M=4096, N=4096, K=65536 with
operands N(0,1) * 2^U{-8..8} per row (seeded, synthetic), the output split into
blocks over a pm x pn grid of ranks (chosen by dist.choose_grid) and the
bposit32 result all-gathered by the GEMM's finish kernel itself (NVLink peer stores;
--gather nccl for N shards and an NCCL all-gather).
The same line carries the encode/decode sweep (2^28 fp32 per rank) in GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the CPU oracle port (oracle/, all host threads) on a
bounded row sample of the same GEMM: rank 0 only.
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
            "RTN-quantized; one bposit32 round per output; output blocks sharded over ranks (pm x pn grid), "
            "result all-gathered")


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled every 20 ms by an NVML thread
    during the timed region (nvidia-smi at 200 ms is the fallback)."""

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

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._run, args=(nv, h), daemon=True)
            self._thread.start()
        except Exception:
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


def make_operand(ops, torch, rows, K, gen, device):
    """bp8 RTN codes of N(0,1) * 2^U{-8..8} per row (generated in chunks)."""
    out = torch.empty((rows, K), dtype=torch.uint8, device=device)
    step = 512
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        x = torch.randn((r1 - r0, K), device=device, generator=gen)
        e = torch.randint(-8, 9, (r1 - r0, 1), device=device, generator=gen).float()
        ops.quantize_bp8(x * torch.exp2(e), nearest=True, out=out[r0:r1])
    return out


def cpu_reference(A_rows, B, target_s: float, threads: int):
    """Time the oracle port's quire GEMM (one row per host thread) on a row
    sample sized to about target_s seconds; returns (TOPS, rows, seconds)."""
    from oracle import oracle
    n = min(threads, A_rows.shape[0])
    t0 = time.perf_counter()
    oracle.quire_gemm(A_rows[:n], B, 8, nthreads=threads)
    t1 = time.perf_counter() - t0
    rows, dt = n, t1
    reps = int(round(target_s / max(t1, 1e-6)))
    if reps > 1:
        rows = min(A_rows.shape[0], n * reps)
        t0 = time.perf_counter()
        oracle.quire_gemm(A_rows[:rows], B, 8, nthreads=threads)
        dt = time.perf_counter() - t0
    tops = 2.0 * rows * B.shape[0] * B.shape[1] / dt / 1e12
    return tops, rows, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    import torch
    from oracle import oracle  # noqa: F401  (built by __graft_entry__.build)
    threads = max(1, len(os.sched_getaffinity(0)))
    # same operand distribution as the GPU arm, generated on the host
    rng = np.random.default_rng(0)
    rows_needed = max(64, 4 * threads)
    from oracle import oracle as orc
    A = orc.quantize_bp8((rng.standard_normal((rows_needed, K_)) *
                          np.exp2(rng.integers(-8, 9, (rows_needed, 1)))).astype(np.float32))[0]
    B = orc.quantize_bp8((rng.standard_normal((N_, K_)) *
                          np.exp2(rng.integers(-8, 9, (N_, 1)))).astype(np.float32))[0]
    per_step = max(2.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        orc.quire_gemm(A[:1], B[:256], 8, nthreads=threads)
    vals, rows_used, secs = [], 0, 0.0
    for _ in range(args.steps):
        v, rows_used, dt = cpu_reference(A, B, per_step, threads)
        vals.append(v)
        secs += dt
    value = statistics.median(vals)
    sample = f"{rows_used} of {M_} rows x N={N_} x K={K_} per step (oracle port, {threads} threads)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / max(1, args.steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic", "config": {"workload": WORKLOAD, "M": M_, "N": N_, "K": K_, "fmt": "bp8",
                                        "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def codec_sweep(ops, torch, device, world, steps, peaks):
    """2^28 fp32 per rank: bp8 RTN encode, bp8 decode, bp16 RTNE encode, bp16 decode."""
    import torch.distributed as dist
    n = 1 << 28
    gen = torch.Generator(device=device).manual_seed(1234 + (dist.get_rank() if world > 1 else 0))
    x = torch.empty(n, dtype=torch.float32, device=device)
    half = n // 2
    x[:half].normal_(generator=gen)
    e = torch.empty(n - half, dtype=torch.float32, device=device).uniform_(-26, 26, generator=gen)
    x[half:] = torch.exp2(e) * torch.where(torch.rand(n - half, device=device, generator=gen) < 0.5, -1.0, 1.0)
    del e
    c8 = torch.empty(n, dtype=torch.uint8, device=device)
    c16 = torch.empty(n, dtype=torch.uint16, device=device)
    y = torch.empty(n, dtype=torch.float32, device=device)
    kernels = {
        "bp8_encode_rtn": (lambda: ops.quantize_bp8(x, nearest=True, out=c8), 5),
        "bp8_decode": (lambda: _decode_into(ops, c8, y), 5),
        "bp16_encode_rtne": (lambda: ops.encode_bp16(x, rtne=True, out=c16), 6),
        "bp16_decode": (lambda: _decode_into(ops, c16, y), 6),
    }
    res = {}
    for name, (fn, bpe) in kernels.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        t.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(t) / steps
        if world > 1:
            tt = torch.tensor([ms], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        gbs = bpe * n * world / (ms * 1e-3) / 1e9
        res[name] = {"GB/s": round(gbs, 1), "ms": round(ms, 4), "bytes_per_elem": bpe,
                     "frac_of_measured_hbm_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4)}
    del x, c8, c16, y
    torch.cuda.empty_cache()
    return {"elements_per_gpu": n, "scaling": "weak", "l2": "1 GiB input > L2", "kernels": res}


def _decode_into(ops, codes, y):
    """decode through the C ABI straight into a preallocated output."""
    import ctypes

    import torch
    from bposit_b200 import _lib
    f = 8 if codes.dtype == torch.uint8 else 16
    _lib.check(_lib.lib().bp_decode(f, ctypes.c_void_p(codes.data_ptr()), codes.numel(),
                                    ctypes.c_void_p(y.data_ptr()),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from bposit_b200 import _lib, ops
    from bposit_b200.dist import FusedShardedQuireGemm, ShardedQuireGemm, assemble

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    peaks, peak_src = load_peaks()

    gen = torch.Generator(device=device).manual_seed(0)
    A = make_operand(ops, torch, M_, K_, gen, device)
    B = make_operand(ops, torch, N_, K_, gen, device)
    fused = args.gather == "fused"
    if fused:
        g = FusedShardedQuireGemm(M_, N_, device, algo=args.algo, K=K_)
        m0, m1, n0, n1 = g.block
        grid = g.grid
    else:
        g = ShardedQuireGemm(M_, N_, device, algo=args.algo)
        (n0, n1), (m0, m1), grid = g.plan.bounds, (0, M_), (1, world)
    A_full = A
    A = A_full[m0:m1].contiguous()
    Bs = B[n0:n1].contiguous()
    del B
    torch.cuda.empty_cache()
    ws = torch.empty(max(256, ops.gemm_workspace_size(8, m1 - m0, n1 - n0, K_, args.algo)), dtype=torch.uint8,
                     device=device)
    peers = [p + 4 * m0 * N_ for p in g.peer_ptrs] if fused else []

    def shard_step(A_, B_, ev=None):
        """One sharded GEMM + all-gather; `ev` brackets the GEMM launches."""
        if fused and world > 1:
            dist.all_reduce(g.flag)
        if ev is not None:
            ev[0].record(stream)
        if fused:
            ops.quire_gemm_multi(A_, B_, g.result[m0:m1, n0:n1], peers, n0, fmt=8, algo=args.algo,
                                 workspace=ws)
        else:
            ops.quire_gemm(A_, B_, 8, out=g.local[:, :n1 - n0] if world > 1 else g.result, algo=args.algo,
                           workspace=ws)
        if ev is not None:
            ev[1].record(stream)
        if world > 1:
            if fused:
                dist.all_reduce(g.flag)
            else:
                dist.all_gather_into_tensor(g.gathered.view(-1).view(torch.int32),
                                            g.local.view(-1).view(torch.int32))
                assemble(g.gathered, g.plan, g.result)
        return g.result

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]

    def gemm_only(i=None):
        return shard_step(A, Bs, None if i is None else kev[i])

    for _ in range(args.warmup):
        gemm_only()
    sync_all()
    clocks = Clocks(local) if local == 0 else None
    if clocks:
        clocks.start()
    launches0 = _lib.lib().bp_launch_count()
    s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_all()
    s.record(stream)
    for i in range(args.steps):
        gemm_only(i)
    t.record(stream)
    sync_all()
    launches = _lib.lib().bp_launch_count() - launches0
    clk = clocks.stop() if clocks else None
    ms = s.elapsed_time(t) / args.steps
    kms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    if world > 1:
        tt = torch.tensor([ms, kms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, kms = float(tt[0]), float(tt[1])
    tops = 2.0 * M_ * N_ * K_ / (ms * 1e-3) / 1e12
    per_rank_ops = 2.0 * (m1 - m0) * (n1 - n0) * K_
    k_tops = per_rank_ops / (kms * 1e-3) / 1e12
    int8_peak = 2.0 * peaks["bf16_tflops"]
    from bposit_b200 import ops as _ops
    slice_pairs = 9 if _ops.gemm_workspace_size(8, m1 - m0, n1 - n0, K_, 2) and args.algo != 1 else None

    # end to end with host buffers (pinned): one GPU through bp_quire_gemm_host;
    # several through H2D of each rank's blocks, the sharded step and a D2H of the result
    hA = A.cpu().pin_memory()
    hB = Bs.cpu().pin_memory()
    hOut = torch.empty((M_, N_), dtype=torch.uint32).pin_memory()
    dA = torch.empty_like(A)
    dB = torch.empty_like(Bs)

    def e2e_step():
        if world == 1:
            # the host-buffer C ABI: A streamed in row chunks (M >= N), copies overlapped with the GEMM
            ops.quire_gemm_host(hA, hB, 8, out=hOut, algo=args.algo)
            return
        dA.copy_(hA, non_blocking=True)
        dB.copy_(hB, non_blocking=True)
        shard_step(dA, dB)
        hOut.copy_(g.result, non_blocking=True)

    e2e_steps = max(1, min(args.steps, 5))
    e2e_step()
    sync_all()
    es, et = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    et.record(stream)
    sync_all()
    ems = es.elapsed_time(et) / e2e_steps
    if world > 1:
        tt = torch.tensor([ems], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ems = float(tt.item())
    e2e_tops = 2.0 * M_ * N_ * K_ / (ems * 1e-3) / 1e12
    # the box's host link, for reading the e2e figure: one plain pinned copy of A
    # (the e2e step is bound by its host-to-device bytes on a healthy link)
    hs, ht = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hs.record(stream)
    dA.copy_(hA, non_blocking=True)
    ht.record(stream)
    torch.cuda.synchronize()
    h2d_gbs = A.numel() * A.element_size() / (hs.elapsed_time(ht) * 1e-3) / 1e9
    del hA, hB, dA, dB

    codec = codec_sweep(ops, torch, device, world, 10, peaks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = max(1, len(os.sched_getaffinity(0)))
        An = A_full[:min(M_, 512)].cpu().numpy()   # room for a ~15 s sample
        Bn = Bs.cpu().numpy()
        v, rows, dt = cpu_reference(An, Bn, 15.0, threads)
        cpu = {"value": v, "unit": "TOPS", "cores": threads, "kind": "port",
               "sample": f"{rows} rows x N={N_} x K={K_} of the same operands ({dt:.1f} s)"}

    traffic, traffic_launches = None, None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            tj = json.load(f)
        ent = tj.get("quire_gemm_" + ("tc" if args.algo != 1 else "simt"))
        if ent and ent.get("shape") == [m1 - m0, n1 - n0, K_]:
            traffic = ent["dram_bytes_per_call"]
            traffic_launches = sum(k.get("launches", 1) for k in ent.get("kernels", {}).values())

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tops, 3), "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M_, "N": N_, "K": K_, "fmt": "bp8",
                       "parallelism": (f"{grid[0]}x{grid[1]} (M x N) block grid over {world} ranks + " +
                                       ("all-gather fused into the GEMM's finish kernel (NVLink peer stores)" if fused
                                        else "NCCL all-gather")),
                       "l2": "inputs 512 MiB > L2 (no flush needed)", "algo": args.algo},
            "roofline": {"bound": "tensor", "achieved": round(k_tops, 3), "peak": round(int8_peak, 1),
                         "unit": "TOPS", "frac": round(k_tops / int8_peak, 5), "traffic": traffic,
                         "peak_source": f"int8 dense = 2 x {peak_src} bf16 {peaks['bf16_tflops']} TF/s",
                         "kernel": "quire GEMM (all launches of one bp_quire_gemm call)",
                         "kernel_ms": round(kms, 3),
                         "traffic_note": (f"DRAM bytes read+written by one bp_quire_gemm call ({traffic_launches} "
                                          "launches), one ncu capture at this shape" if traffic
                                          else "no capture at this shape"),
                         "issued_int8_TOPS": round(k_tops * slice_pairs, 1) if slice_pairs else None,
                         "issued_frac": round(k_tops * slice_pairs / int8_peak, 4) if slice_pairs else None,
                         "slice_pairs_per_useful_mac": slice_pairs},
            "e2e": {"value": round(e2e_tops, 3), "unit": "TOPS", "ms_per_step": round(ems, 3),
                    "h2d_bytes_per_step": int((m1 - m0) * K_ + (n1 - n0) * K_),
                    "d2h_bytes_per_step": int(M_ * N_ * 4),
                    "h2d_link_gbs": round(h2d_gbs, 1)},
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clk,
            "encode_decode": codec,
        }
        print(json.dumps(line), flush=True)
    if fused:
        g.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--algo", type=int, default=0, help="0 auto, 1 CUDA cores, 2 tensor cores")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
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
