"""Tensor-parallel decode on 2 GPUs (skipped with fewer): tiny Qwen3 at TP2 through the engine
with the flagged-word NVLink all-reduce (plain peer stores), eager and graph-captured, against the
reference's greedy tokens."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_tiny_qwen3_matches_reference():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "540", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={29500 + os.getpid() % 1000}",
           os.path.join(HERE, "tp_gpu_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(proc.stdout[-4000:], proc.stderr[-4000:])
    assert proc.returncode == 0
