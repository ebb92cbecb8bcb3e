"""Fused tensor-parallel collectives (all-gather -> GEMM, GEMM -> reduce-scatter over NVLink peer
memory) on 2 GPUs against NCCL + an fp32 reference, and a sequence-parallel model's loss and
gradients fused vs the NCCL path. Runs `fused_tp_worker.py` under torchrun; skipped with < 2 GPUs."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_tp_two_gpus():
    worker = Path(__file__).with_name("fused_tp_worker.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MINT_PG_TIMEOUT_S="120")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533", str(worker)]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(res.stdout[-4000:])
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-4000:]
