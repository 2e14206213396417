"""Sequence-parallel scan over NCCL on 2+ GPUs (config 5 recipe at a reduced
length): the segments scanned on separate GPUs, joined through the carry
all-gather, equal a one-GPU scan of the whole sequence (tolerance 2e-3: the
two paths cut the sequence into chunks at the same boundaries and differ
only by fp32 summation order in the carries)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_sp_two_gpus_matches_one_gpu_scan():
    n = min(torch.cuda.device_count(), 8)
    T = 8192 * n
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29533", str(ROOT / "tests" / "sp_worker.py"),
           str(T)]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert "rel_err" in res.stdout
