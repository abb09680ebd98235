"""Tensor-parallel collectives on the GPU: the NVLink one-shot all-reduce (qf_allreduce_bf16) against the fp32
rank-order sum of all ranks' inputs, eagerly and inside CUDA graphs.  World size 1 runs on any single B200;
world size 2 runs when two GPUs are visible (one torchrun process per GPU).  Each case is a child process."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_allreduce_single_rank(dev):
    r = subprocess.run([sys.executable, "-m", "tests._tp_case"], cwd=REPO, capture_output=True, text=True,
                       timeout=300, env=dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


def test_allreduce_two_ranks(dev):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           "-m", "tests._tp_case"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
