"""Multi-GPU host logic on CPU: world_size-2 gloo runs of tests/dist_cases.py."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_dist(case: str, nproc: int = 2, timeout: int = 240) -> None:
    env = dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(REPO / "tests" / "dist_cases.py"), case]
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


def test_column_parallel_matches_full_linear_gloo():
    run_dist("column")


def test_expert_parallel_layer_matches_single_process_gloo():
    run_dist("ep_moe")


def test_column_range_rejects_uneven_split():
    sys.path.insert(0, str(REPO / "simsd-release_b200"))
    from kernels import parallel as P
    assert P.column_range(12, 1, 3) == (4, 8)
    with pytest.raises(ValueError):
        P.column_range(10, 0, 3)
    w = torch.arange(12.0).reshape(6, 2)
    assert torch.equal(P.column_shard(w, 2, 3), w[4:6])


def test_expert_range():
    sys.path.insert(0, str(REPO / "simsd-release_b200"))
    from kernels import moe_parallel as MP
    assert MP.expert_range(256, 3, 8) == (96, 128)
    with pytest.raises(ValueError):
        MP.expert_range(10, 0, 4)
