"""Multi-GPU parity of the sharded hot path (skipped with fewer than two GPUs): the NCCL
all-gather exchange and the peer-to-peer scatter + barrier exchange.

Runs ``multi_gpu_worker.py`` as one process per GPU under torchrun and requires every rank's
full outputs to equal the single-GPU engine's, eagerly and under CUDA-graph replay.
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
@pytest.mark.parametrize("split,exchange", [("heads", "nccl"), ("auto", "nccl"),
                                            ("heads", "p2p"), ("auto", "p2p")])
def test_sharded_hot_path_across_gpus(split, exchange):
    n = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29561",
           os.path.join(HERE, "multi_gpu_worker.py"), split, exchange]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    log = os.environ.get("HEATKV_MULTI_GPU_LOG")
    if log:
        with open(f"{log}.{split}.{exchange}", "w") as fh:
            fh.write(res.stdout + res.stderr)
    tail = (res.stdout + res.stderr)[-3000:]
    assert res.returncode == 0, tail
    assert "multi-GPU parity ok" in res.stdout, tail


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_projected_workload_sharded_by_rows_across_gpus():
    """configs[4]'s projection-driven path with the batch sharded by rows over two GPUs: the
    gathered outputs equal one GPU's bit for bit, and match keep-mask attention."""
    n = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29563",
           os.path.join(HERE, "projected_multi_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    log = os.environ.get("HEATKV_MULTI_GPU_LOG")
    if log:
        with open(f"{log}.projected", "w") as fh:
            fh.write(res.stdout + res.stderr)
    tail = (res.stdout + res.stderr)[-3000:]
    assert res.returncode == 0, tail
    assert "projected multi-GPU parity ok" in res.stdout, tail
