"""Exact data parallelism over real GPUs and NCCL (skipped with fewer than two
GPUs): two ranks under torchrun shard the golden story batches and must end
with the single-GPU golden state hash on every rank."""

import socket
import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
def test_two_gpu_sharded_batches_match_single_gpu_golden(native_lib):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(HERE / "multi_gpu_worker.py"), "baseline1", "test-8", "baseline3-short"]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=900,
                          env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
