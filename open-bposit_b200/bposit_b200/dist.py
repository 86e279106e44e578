"""Multi-GPU quire GEMM: the output dimension N is sharded across ranks (one
process per GPU) and every rank ends with the whole bposit32 result.

Each rank holds all of A[M,K] and its row block B[n0:n1, K] of B[N,K] and
computes out[:, n0:n1] exactly; outputs are column-disjoint and no partial sum
ever crosses a rank, so the result is bit-identical for every rank count.

Two ways to all-gather the blocks:
  ShardedQuireGemm       -- one NCCL all_gather_into_tensor of the [M, N/p]
                            uint32 shards into [p, M, N/p], then a local
                            transpose into [M, N];
  FusedShardedQuireGemm  -- the GEMM's finish kernel stores every bposit32
                            straight into all ranks' [M, N] result buffers over
                            NVLink (peer stores into CUDA-IPC-shared memory);
                            two one-word NCCL all-reduces order the call
                            against the ranks' previous and next use of them.
                            The ranks may also form a pm x pn grid over
                            (M, N) blocks (choose_grid), which splits the
                            per-rank operand preparation of A as well.
"""
from __future__ import annotations

import contextlib
import threading
import time
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    """Column block [n0, n1) of rank `rank`: equal blocks of ceil(N / world)
    (the last ones may be short or empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    per = -(-N // world)
    n0 = min(N, rank * per)
    return n0, min(N, n0 + per)


@dataclass
class ShardPlan:
    M: int
    N: int
    world: int
    rank: int

    @property
    def per(self) -> int:
        return -(-self.N // self.world)

    @property
    def bounds(self) -> tuple[int, int]:
        return shard_bounds(self.N, self.world, self.rank)


def assemble(gathered: torch.Tensor, plan: ShardPlan, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[world, M, per] gathered shards -> [M, N] (drops the padding columns)."""
    full = gathered.permute(1, 0, 2).reshape(plan.M, plan.world * plan.per)
    if out is None:
        return full[:, :plan.N].contiguous()
    out.copy_(full[:, :plan.N])
    return out


class ShardedQuireGemm:
    """out = bp32(A @ B^T) with B's rows split over the process group.

    gemm_fn(A, B_shard, out_view, sa, sb_shard) must fill out_view[M, n1-n0]
    (default: the library's tensor/CUDA-core quire GEMM).  Buffers are
    allocated once; every call performs one GEMM launch sequence and one
    all-gather on the current stream.
    """

    def __init__(self, M: int, N: int, device, group=None, gemm_fn: Optional[Callable] = None,
                 fmt: int = 8, algo: int = 0, group_size: int = 128):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.plan = ShardPlan(M, N, self.world, self.rank)
        per = self.plan.per
        self.local = torch.zeros((M, per), dtype=torch.uint32, device=device)
        self.gathered = torch.empty((self.world, M, per), dtype=torch.uint32, device=device)
        self.result = torch.empty((M, N), dtype=torch.uint32, device=device)
        self.fmt, self.algo, self.group_size = fmt, algo, group_size
        self.gemm_fn = gemm_fn or self._library_gemm
        self.workspace = None

    def _library_gemm(self, A, Bs, out_view, sa, sbs):
        from . import ops
        if self.workspace is None:
            need = ops.gemm_workspace_size(self.fmt, A.shape[0], Bs.shape[0], A.shape[1], self.algo)
            self.workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=A.device)
        ops.quire_gemm(A, Bs, self.fmt, sa=sa, sb=sbs, group=self.group_size, out=out_view, algo=self.algo,
                       workspace=self.workspace)

    def __call__(self, A: torch.Tensor, B_shard: torch.Tensor, sa=None, sb_shard=None) -> torch.Tensor:
        n0, n1 = self.plan.bounds
        if B_shard.shape[0] != n1 - n0:
            raise ValueError(f"B shard has {B_shard.shape[0]} rows, rank {self.rank} owns {n1 - n0}")
        if n1 > n0:
            self.gemm_fn(A, B_shard, self.local[:, :n1 - n0], sa, sb_shard)
        if self.world == 1:
            self.result.copy_(self.local[:, :self.plan.N])
            return self.result
        dist.all_gather_into_tensor(self.gathered.view(-1).view(torch.int32),
                                    self.local.view(-1).view(torch.int32), group=self.group)
        return assemble(self.gathered, self.plan, self.result)


def block_bounds(M: int, N: int, grid: tuple[int, int], rank: int) -> tuple[int, int, int, int]:
    """Output block (m0, m1, n0, n1) of `rank` on a pm x pn rank grid (rank =
    rm * pn + rn); blocks of ceil(M / pm) rows and ceil(N / pn) columns."""
    pm, pn = grid
    m0, m1 = shard_bounds(M, pm, rank // pn)
    n0, n1 = shard_bounds(N, pn, rank % pn)
    return m0, m1, n0, n1


def choose_grid(world: int, M: int, N: int, K: int, fmt: int = 8, wave: int = 74) -> tuple[int, int]:
    """The pm x pn rank grid with the smallest modelled per-rank time: every rank
    prepares its M/pm rows of A and N/pn rows of B (time ~ rows * K), then runs
    its block's tiles (256 x 96 for bp8, 256 x 64 for bp16) in waves of `wave`
    tile pairs, the last partial wave split along K across the machine."""
    bn = 96 if fmt == 8 else 64
    slices = 9 if fmt == 8 else 16
    nkb = max(1, -(-K // 128) * 2)
    best, best_cost = (1, world), None
    for pm in range(1, world + 1):
        if world % pm:
            continue
        pn = world // pm
        mr, nr = -(-M // pm), -(-N // pn)
        prep = (mr + nr) * K * 1.05e-9                    # ~0.28 ms per 4096 x 65536 operand
        tiles = -(-mr // 256) * -(-nr // bn)
        W, R = divmod(tiles, wave)
        sp = min(wave // R, max(1, nkb // 16)) if R else 1
        waves = W + ((1.0 / sp) if (R and sp > 1) else (1.0 if R else 0.0))
        gemm = waves * K * slices * bn / 96 * 8.8e-7 / 9      # ~0.52 ms per bp8 tile at K = 65536
        cost = prep + gemm
        if best_cost is None or cost < best_cost * 0.995:
            best, best_cost = (pm, pn), cost
    return best


class CallWatchdog:
    """Host deadline for multi-GPU calls.

    `with wd.guard("gemm"): ...` runs the block under a deadline of
    `deadline_s` seconds.  A monitor thread that sees a guarded block outlive
    it calls `on_timeout(what)` -- by default it aborts the process group
    (`ProcessGroup.abort()`, which ends a collective still waiting on a rank
    that died or never joined with an error on this rank) -- and trips the
    watchdog: the block, and every later guarded block, raises BpositError.
    With `sync=True` the guard also waits for the current CUDA stream, so the
    deadline covers the call's device work (kernels, peer stores, NCCL).
    Kernel waits have their own bounds; this covers a peer process that is
    gone.
    """

    def __init__(self, deadline_s: float, on_timeout: Optional[Callable[[str], None]] = None, group=None,
                 sync: bool = False):
        if deadline_s <= 0:
            raise ValueError("deadline_s must be positive")
        self.deadline_s = float(deadline_s)
        self.group = group
        self.sync = sync
        self.on_timeout = on_timeout if on_timeout is not None else self._abort_group
        self.tripped: Optional[str] = None
        self._cv = threading.Condition()
        self._armed: Optional[tuple[str, float]] = None   # (what, deadline on time.monotonic)
        self._closed = False
        self._thread = threading.Thread(target=self._run, name="bposit-watchdog", daemon=True)
        self._thread.start()

    def _abort_group(self, what: str) -> None:
        pg = self.group if self.group is not None else dist.distributed_c10d._get_default_group()
        pg.abort()

    def _run(self) -> None:
        with self._cv:
            while not self._closed:
                if self._armed is None:
                    self._cv.wait()
                    continue
                what, due = self._armed
                left = due - time.monotonic()
                if left > 0:
                    self._cv.wait(timeout=left)
                    continue
                self._armed = None
                self.tripped = f"{what} exceeded its {self.deadline_s:g} s deadline"
                try:
                    self.on_timeout(what)
                except Exception as exc:   # the trip stands even if the abort fails
                    self.tripped += f" (abort failed: {exc})"

    @contextlib.contextmanager
    def guard(self, what: str = "call"):
        from ._lib import BP_ECUDA, BpositError
        if self.tripped:
            raise BpositError(BP_ECUDA, f"watchdog tripped earlier: {self.tripped}")
        with self._cv:
            self._armed = (what, time.monotonic() + self.deadline_s)
            self._cv.notify()
        err: Optional[BaseException] = None
        try:
            yield self
            if self.sync and torch.cuda.is_available():
                torch.cuda.current_stream().synchronize()
        except BaseException as exc:   # a collective that the abort ended
            err = exc
        finally:
            with self._cv:
                self._armed = None
                self._cv.notify()
        if self.tripped:
            raise BpositError(BP_ECUDA, f"watchdog: {self.tripped}") from err
        if err is not None:
            raise err

    def close(self) -> None:
        with self._cv:
            self._closed = True
            self._cv.notify()
        self._thread.join(timeout=5)


class FusedShardedQuireGemm:
    """N-sharded quire GEMM with the all-gather fused into the GEMM's finish kernel.

    Every rank allocates one [M, N] uint32 result in CUDA-IPC-shareable memory
    and maps every peer's result into its own device context; each rank's
    GEMM writes its column block [n0, n1) into its own result and, over
    NVLink, into every peer's.  A call is
        all_reduce(1 word)   -- no rank still reads its previous result
        GEMM + peer stores   -- bp_quire_gemm_multi
        all_reduce(1 word)   -- every peer's stores into this result are done
    all on the current stream.  The returned tensor stays valid until the
    next call.  Needs one node with peer access between all its GPUs and at
    most 9 ranks; call close() on every rank before destroying the group.
    """

    def __init__(self, M: int, N: int, device, group=None, fmt: int = 8, algo: int = 0,
                 group_size: int = 128, grid: Optional[tuple[int, int]] = None, K: Optional[int] = None,
                 deadline_s: Optional[float] = None):
        from . import ops
        self.group = group
        # optional host deadline per call (CallWatchdog, synchronizing)
        self.watchdog = CallWatchdog(deadline_s, group=group, sync=True) if deadline_s else None
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world - 1 > 8:
            raise ValueError("FusedShardedQuireGemm supports at most 9 ranks")
        if grid is None:
            grid = choose_grid(self.world, M, N, K, fmt) if K else (1, self.world)
        if grid[0] * grid[1] != self.world:
            raise ValueError(f"grid {grid} does not cover {self.world} ranks")
        self.grid = tuple(grid)
        self.M, self.N = M, N
        self.block = block_bounds(M, N, self.grid, self.rank)   # (m0, m1, n0, n1)
        self.plan = ShardPlan(M, N, self.world, self.rank)
        self.fmt, self.algo, self.group_size = fmt, algo, group_size
        dev = torch.device(device)
        self.device = dev
        self.result, handle, self._own = ops.ipc_alloc((M, N), dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self.peer_ptrs: list[int] = []
        if self.world > 1:
            objs = [None] * self.world
            dist.all_gather_object(objs, (dev.index, handle), group=group)
            with torch.cuda.device(dev):
                for r, (pdev, h) in enumerate(objs):
                    if r != self.rank:
                        ops.enable_peer_access(pdev)
                        self.peer_ptrs.append(ops.ipc_open(h))
        self.workspace = None

    def __call__(self, A_block: torch.Tensor, B_block: torch.Tensor, sa=None, sb=None) -> torch.Tensor:
        """A_block = A[m0:m1], B_block = B[n0:n1] (and their group exponents) for
        this rank's block (m0, m1, n0, n1) = self.block; with a 1 x world grid
        A_block is all of A."""
        from . import ops
        if self.result is None:
            raise RuntimeError("FusedShardedQuireGemm is closed")
        m0, m1, n0, n1 = self.block
        if A_block.shape[0] != m1 - m0 or B_block.shape[0] != n1 - n0:
            raise ValueError(f"rank {self.rank} owns rows [{m0}, {m1}) of A and [{n0}, {n1}) of B, got "
                             f"{A_block.shape[0]} and {B_block.shape[0]}")
        if self.watchdog is not None:
            with self.watchdog.guard("FusedShardedQuireGemm"):
                return self._call(A_block, B_block, sa, sb)
        return self._call(A_block, B_block, sa, sb)

    def _call(self, A_block, B_block, sa, sb) -> torch.Tensor:
        from . import ops
        m0, m1, n0, n1 = self.block
        if self.world > 1:
            dist.all_reduce(self.flag, group=self.group)
        if m1 > m0 and n1 > n0:
            if self.workspace is None:
                need = ops.gemm_workspace_size(self.fmt, m1 - m0, n1 - n0, A_block.shape[1], self.algo)
                self.workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=A_block.device)
            peers = [p + 4 * m0 * self.N for p in self.peer_ptrs]     # row m0 of every peer's result
            ops.quire_gemm_multi(A_block, B_block, self.result[m0:m1, n0:n1], peers, n0, fmt=self.fmt, sa=sa,
                                 sb=sb, group=self.group_size, algo=self.algo, workspace=self.workspace)
        if self.world > 1:
            dist.all_reduce(self.flag, group=self.group)
        return self.result

    def close(self) -> None:
        """Unmap the peers' results and free this rank's once no rank writes
        into them any more.  Collective: every rank calls it."""
        from . import ops
        if self.result is None:
            return
        if self.watchdog is not None:
            self.watchdog.close()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self.peer_ptrs:
                ops.ipc_close(p)
        self.peer_ptrs = []
        if self.world > 1:
            dist.barrier(group=self.group)
        self.result = None
        ops.ipc_free(self._own)
