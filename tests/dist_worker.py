"""One rank of the multi-GPU quire GEMM check (launched by tests/test_gpu_dist.py
through torch.distributed.run, one process per GPU, NCCL).  Every rank computes
its N-shard on the tensor cores, the shards are all-gathered (NCCL, and the
fused epilogue peer stores), and every rank compares its whole bposit32 matrix
with an unsharded single-GPU GEMM: the quire result must be bit-identical for
any rank count.  Then the Qwen-shaped forward with every linear sharded
(nn.shard_linears) against the same forward on one GPU."""
from __future__ import annotations

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "open-bposit_b200")]

from bposit_b200 import ops  # noqa: E402
from bposit_b200.dist import FusedShardedQuireGemm, ShardedQuireGemm  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    results = []
    cases = ((512, 1001, 4096, 0), (300, 777, 1000, 128), (2048, 1536, 4096, 0), (2048, 1536, 2048, 128),
             (256, max(1, world - 1), 512, 0))   # the last one leaves the last rank an empty shard
    for (M, N, K, group) in cases:
        g = torch.Generator(device=dev).manual_seed(123)
        X = torch.randn((M, K), device=dev, generator=g)
        W = torch.randn((N, K), device=dev, generator=g) * 0.02
        if group:
            A, sa = ops.quantize_bp8_grouped(X, group=group)
            B, sb = ops.quantize_bp8_grouped(W, group=group)
        else:
            A, sa = ops.quantize_bp8(X), None
            B, sb = ops.quantize_bp8(W), None
        sg = ShardedQuireGemm(M, N, dev, group_size=group or 128)
        n0, n1 = sg.plan.bounds
        Bs = B[n0:n1].contiguous()
        sbs = None if sb is None else sb[n0:n1].contiguous()
        out = sg(A, Bs, sa, sbs).clone()
        # Fused epilogue all-gather (peer stores); two calls on different A so
        # the second one overwrites a live result buffer; an N-shard grid and,
        # where the rank count allows, an M x N block grid.
        A2 = A.flip(0).contiguous()
        sa2 = None if sa is None else sa.flip(0).contiguous()
        fused1 = fused2 = None
        grids = [(1, world)] + ([(2, world // 2)] if world % 2 == 0 and world > 2 else []) + \
                ([(world, 1)] if world > 1 else [])
        fused_ok = True
        for grid in grids:
            fg = FusedShardedQuireGemm(M, N, dev, group_size=group or 128, grid=grid)
            m0, m1, n0g, n1g = fg.block

            def blk(t, lo, hi):
                return None if t is None else t[lo:hi].contiguous()

            r1 = fg(blk(A, m0, m1), blk(B, n0g, n1g), blk(sa, m0, m1), blk(sb, n0g, n1g)).clone()
            r2 = fg(blk(A2, m0, m1), blk(B, n0g, n1g), blk(sa2, m0, m1), blk(sb, n0g, n1g)).clone()
            torch.cuda.synchronize()
            fg.close()
            if fused1 is None:
                fused1, fused2 = r1, r2
            else:
                fused_ok = fused_ok and torch.equal(r1.view(torch.int32), fused1.view(torch.int32)) and \
                    torch.equal(r2.view(torch.int32), fused2.view(torch.int32))
        ref, _ = ops.quire_gemm(A, B, 8, sa=sa, sb=sb, group=group or 128)
        ref2, _ = ops.quire_gemm(A2, B, 8, sa=sa2, sb=sb, group=group or 128)
        torch.cuda.synchronize()
        eq = lambda x, y: bool(torch.equal(x.view(torch.int32), y.view(torch.int32)))  # noqa: E731
        ok = [eq(out, ref), eq(fused1, ref), eq(fused2, ref2), fused_ok]
        flags = torch.tensor([int(all(ok))], device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        if rank == 0:
            results.append({"shape": [M, N, K], "group": group, "gather": ok[0], "fused": ok[1:],
                            "equal": bool(flags.item())})
    # The N-sharded Qwen-shaped forward (every linear's output block over the
    # ranks, all-gathered by the finish kernel) against the same model on this
    # GPU alone: identical bposit32 words give an identical forward.
    from bposit_b200.forward import qwen05, synthetic_ids
    from bposit_b200.nn import close_sharded, shard_linears
    ids = synthetic_ids(2, 256, seed=5, device=dev)
    one = qwen05(layers=2, device=dev, seed=3)
    h1 = one(ids)
    sh = shard_linears(qwen05(layers=2, device=dev, seed=3))
    h2 = sh(ids)
    h3 = sh(ids.flip(1))
    h4 = one(ids.flip(1))
    torch.cuda.synchronize()
    close_sharded()
    ok_f = bool(torch.equal(h1, h2)) and bool(torch.equal(h3, h4))
    flags = torch.tensor([int(ok_f)], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if rank == 0:
        results.append({"shape": "qwen05 2 layers x 512 tokens, sharded linears", "equal": bool(flags.item())})
    dist.barrier()
    if rank == 0:
        print(json.dumps({"world": world, "results": results}), flush=True)
    dist.destroy_process_group()
    ok = all(r["equal"] for r in results) if rank == 0 else True
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
