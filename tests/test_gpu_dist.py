"""N-sharded quire GEMM on 2+ GPUs of one node (NCCL all-gather): the result
is bit-identical to the single-GPU GEMM.  Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_gemm_matches_single_gpu():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(REPO, "tests", "dist_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
    errors = [ln for ln in r.stderr.splitlines() if "rror" in ln and "frame #" not in ln][:20]
    assert r.returncode == 0, "\n".join(errors) + "\n" + r.stdout[-2000:] + r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    res = json.loads(line)
    assert res["world"] == n and all(x["equal"] for x in res["results"]), res
