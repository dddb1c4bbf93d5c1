"""Tensor-parallel engine on 2+ GPUs of one box (skipped with fewer GPUs).

Runs ``tests/tp_worker.py`` under torchrun; each rank checks every op's full
output against the oracle (relative L2 <= 1e-3).
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("bits,batch", [(3, 1), (2, 3), (4, 2)])
def test_tp_engine_parity(bits, batch):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    n = min(4, torch.cuda.device_count())
    env = dict(os.environ, TP_BITS=str(bits), TP_BATCH=str(batch), NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--nnodes=1", f"--nproc-per-node={n}",
           str(ROOT / "tests" / "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
