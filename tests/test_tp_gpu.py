"""Tensor-parallel streamed stack on 2 (or more) GPUs against the single-GPU stack (skipped with fewer GPUs): the
worker runs under torchrun on 127.0.0.1 with a bounded process-group timeout and an outer time limit."""

import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


def test_tp_stack_matches_single_gpu(cuda):
    n = cuda.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(REPO, "tests", "tp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("vs single GPU") == world


def test_sp_stack_matches_single_gpu(cuda):
    n = cuda.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", "29534",
           os.path.join(REPO, "tests", "sp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("vs single GPU") == 2 * world
