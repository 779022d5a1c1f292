"""Vocabulary parallelism over NCCL with one process per GPU (needs >= 2 GPUs; skipped otherwise)."""

from __future__ import annotations

import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
WORKER = Path(__file__).resolve().parent / "multigpu" / "vocab_parallel_worker.py"


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_vocab_parallel_over_nccl(cuda_device, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_port()}", str(WORKER)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    print(res.stdout[-3000:], res.stderr[-3000:])
    assert res.returncode == 0
