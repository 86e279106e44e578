"""Host logic of the N-sharded quire GEMM (bposit_b200/dist.py) on 2 CPU ranks
over gloo: shard bounds, the all-gather of column shards and the assembly into
[M, N] are checked bit-exactly against the unsharded oracle GEMM, including N
not divisible by the rank count and a rank that owns no columns.  The oracle
stands in for the device GEMM on CPU ranks (the GPU run of the same class is
tests/test_gpu_dist.py)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cases, q):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "open-bposit_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from bposit_b200.dist import ShardedQuireGemm
    from oracle import oracle
    try:
        for (M, N, K, seed) in cases:
            rng = np.random.default_rng(seed)
            A = rng.integers(0, 256, (M, K), dtype=np.uint8)
            B = rng.integers(0, 256, (N, K), dtype=np.uint8)

            def cpu_gemm(a, b, out_view, sa, sb):
                out_view.copy_(torch.from_numpy(oracle.quire_gemm(a.numpy(), b.numpy(), 8, nthreads=1).view(np.int32)).view(torch.uint32))

            g = ShardedQuireGemm(M, N, torch.device("cpu"), gemm_fn=cpu_gemm)
            n0, n1 = g.plan.bounds
            out = g(torch.from_numpy(A), torch.from_numpy(B[n0:n1].copy()))
            if rank == 0:
                ref = oracle.quire_gemm(A, B, 8, nthreads=1)
                q.put(((M, N, K), bool(np.array_equal(out.numpy(), ref))))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_gemm_gloo(world):
    cases = [(5, 8, 33, 1), (7, 7, 64, 2), (3, 1, 16, 3), (9, 13, 100, 4)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=5) for _ in cases]
    assert all(ok for _, ok in res), res


def test_shard_bounds():
    from bposit_b200.dist import shard_bounds
    for N in (0, 1, 7, 8, 4096):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(N, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(0 <= n0 <= n1 <= N for n0, n1 in spans)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 6, 8])
def test_block_grid_covers_output_once(world):
    """Every pm x pn grid (and the chosen one) tiles [M, N] exactly once: the
    large GEMM and the Qwen-shaped linears that nn.shard_linears splits."""
    from bposit_b200.dist import block_bounds, choose_grid
    for M, N, K in ((4096, 4096, 65536), (300, 777, 65536), (5, 3, 65536), (1, 64, 65536),
                    (8192, 1152, 896), (8192, 896, 896), (8192, 9728, 896), (8192, 896, 4864)):
        grids = [(pm, world // pm) for pm in range(1, world + 1) if world % pm == 0]
        chosen = choose_grid(world, M, N, K)
        assert chosen in grids
        for grid in grids:
            cover = np.zeros((M, N), np.int32)
            for r in range(world):
                m0, m1, n0, n1 = block_bounds(M, N, grid, r)
                assert 0 <= m0 <= m1 <= M and 0 <= n0 <= n1 <= N
                cover[m0:m1, n0:n1] += 1
            assert (cover == 1).all()


def _watchdog_worker(rank, world, port, q):
    """Rank 1 never joins rank 0's collective (it leaves between steps); rank 0's
    guarded all_reduce must end with BpositError once the watchdog trips."""
    import datetime
    import sys
    import time
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "open-bposit_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    from bposit_b200._lib import BpositError
    from bposit_b200.dist import CallWatchdog
    fired = []
    wd = CallWatchdog(1.0, on_timeout=lambda what: fired.append((what, time.monotonic())))
    t = torch.ones(1)
    with wd.guard("step 0"):          # both ranks: completes well inside the deadline
        dist.all_reduce(t)
    if rank == 1:
        time.sleep(8)                 # gone for rank 0's next step
        q.put(("rank1", True))
        wd.close()
        return
    t0 = time.monotonic()
    try:
        with wd.guard("step 1"):
            dist.all_reduce(t)       # rank 1 never joins: gloo's own timeout ends it
        q.put(("rank0", "no error"))
    except BpositError as exc:
        ok = bool(fired) and fired[0][0] == "step 1" and 0.8 < fired[0][1] - t0 < 5.0 and "deadline" in str(exc)
        try:
            with wd.guard("step 2"):  # tripped: later calls refuse at once
                pass
            ok = False
        except BpositError:
            pass
        q.put(("rank0", ok))
    except Exception as exc:          # noqa: BLE001
        q.put(("rank0", f"other error {type(exc).__name__}: {exc}"))
    wd.close()


def test_call_watchdog_gloo():
    """Host failure made on the host: a rank that never joins a step.  The
    watchdog fires its callback about 1 s into the step, the step raises
    BpositError naming the deadline, and the watchdog stays tripped."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_watchdog_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res["rank0"] is True, res
    assert res["rank1"] is True


def test_call_watchdog_quiet_when_fast():
    """Guarded blocks that end in time never fire the callback; errors inside
    a guard pass through unchanged."""
    from bposit_b200.dist import CallWatchdog
    fired = []
    wd = CallWatchdog(5.0, on_timeout=fired.append)
    for _ in range(100):
        with wd.guard("fast"):
            pass
    with pytest.raises(KeyError):
        with wd.guard("raises"):
            raise KeyError("x")
    wd.close()
    assert fired == [] and wd.tripped is None
