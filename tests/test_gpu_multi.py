"""Multi-GPU parity of the sharded hot path over NCCL (skipped with fewer than two GPUs).

Runs ``multi_gpu_worker.py`` as one process per GPU under torchrun and requires every rank's
gathered outputs to equal the single-GPU engine's, eagerly and under CUDA-graph replay.
"""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("split", ["heads", "auto"])
def test_sharded_hot_path_over_nccl(split):
    n = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29561",
           os.path.join(HERE, "multi_gpu_worker.py"), split]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    tail = (res.stdout + res.stderr)[-3000:]
    assert res.returncode == 0, tail
    assert "multi-GPU parity ok" in res.stdout, tail
