"""Failure detection on 2 GPUs without a GPU fault: a rank that skips a fused collective makes its
peer's kernel give up after a short, run-time wait limit and report a status bit that the host
turns into an exception, while the parameter-update kernels refuse to apply the step. NVLS and
NVLink multicast are off (plain peer loads and stores only; the test's symmetric buffers live on
the WORLD group, where torch's symmetric memory accepts TORCH_SYMM_MEM_DISABLE_MULTICAST). Skipped
with < 2 GPUs."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_skipped_peer_times_out_and_raises():
    worker = Path(__file__).with_name("failure_worker.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29536", str(worker)]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(res.stdout[-4000:])
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-4000:]
    assert "skipped peer: raised" in res.stdout
