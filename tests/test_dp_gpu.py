"""Data-parallel peer-memory reduce-scatter / all-gather kernels and the GRPO step on 2, 4 and 8 GPUs."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from conftest import free_port  # noqa: E402


@pytest.mark.parametrize("world", [2, 4, 8])
def test_data_parallel_kernels_match_nccl(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(HERE, "dp_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=360, env=env)
    assert out.returncode == 0 and "DP_OK" in out.stdout, out.stdout[-3000:] + out.stderr[-3000:]
