"""One rank of the multi-GPU quire GEMM check (launched by tests/test_gpu_dist.py
through torch.distributed.run, one process per GPU, NCCL).  Every rank computes
its N-shard on the tensor cores, the shards are all-gathered, and rank 0
compares the gathered bposit32 matrix with an unsharded single-GPU GEMM:
the quire result must be bit-identical for any rank count."""
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
from bposit_b200.dist import ShardedQuireGemm  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    results = []
    for (M, N, K, group) in ((512, 1001, 4096, 0), (300, 777, 1000, 128)):
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
        out = sg(A, B[n0:n1].contiguous(), sa, None if sb is None else sb[n0:n1].contiguous())
        torch.cuda.synchronize()
        if rank == 0:
            ref, _ = ops.quire_gemm(A, B, 8, sa=sa, sb=sb, group=group or 128)
            torch.cuda.synchronize()
            results.append({"shape": [M, N, K], "group": group,
                            "equal": bool(torch.equal(out.view(torch.int32), ref.view(torch.int32)))})
    dist.barrier()
    if rank == 0:
        print(json.dumps({"world": world, "results": results}), flush=True)
    dist.destroy_process_group()
    ok = all(r["equal"] for r in results) if rank == 0 else True
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
