"""Multi-GPU quire GEMM: the output dimension N is sharded across ranks (one
process per GPU) and the bposit32 result is all-gathered over NCCL.

Each rank holds all of A[M,K] and its row block B[n0:n1, K] of B[N,K] and
computes out[:, n0:n1] exactly; outputs are column-disjoint and no partial sum
ever crosses a rank, so the result is bit-identical for every rank count.
The gather is one all_gather_into_tensor of the [M, N/p] uint32 shards into a
[p, M, N/p] buffer followed by a local transpose into [M, N].
"""
from __future__ import annotations

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
