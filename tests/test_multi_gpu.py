"""Column-parallel thin linears (NCCL all-gather, and the all-gather fused into
the GEMM over NVLink peer stores, waited for per call and deferred), the
expert-parallel MoE layer and the column-split verify forward (bit-identical
to one GPU) on 2 GPUs, one process per GPU.  Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_column_parallel_and_expert_parallel_on_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(REPO / "tests" / "dist_gpu_cases.py"), "column", "ep", "fused", "verify_tp"]
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=360)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
