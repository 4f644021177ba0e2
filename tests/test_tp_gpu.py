"""Tensor-parallel decode on 2 GPUs (skipped with fewer): tiny Qwen3 at TP2 through the engine
with the flagged-word NVLink all-reduce (peer stores, or NVSwitch multicast stores), eager and
graph-captured, against the reference's greedy tokens."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("multicast", ["0", "1"])
def test_tp2_tiny_qwen3_matches_reference(multicast):
    """FB_TP_MULTICAST=0: plain peer stores (the worker checks no multicast object exists);
    =1: NVSwitch multicast stores where the driver provides a multicast object."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", FB_TP_MULTICAST=multicast)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={29500 + os.getpid() % 1000 + int(multicast)}",
           os.path.join(HERE, "tp_gpu_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(proc.stdout[-4000:], proc.stderr[-4000:])
    assert proc.returncode == 0
