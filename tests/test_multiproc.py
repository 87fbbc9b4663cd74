"""Multi-process runs: torchrun with one rank per GPU (CUDA IPC peer mappings).

Skipped unless the box has at least two GPUs. The worker bounds every wait
(10 s device timeout, 60 s process-group timeout, `timeout -k` around
torchrun) so a broken peer ends the test with an error, never a hang.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import gpu_count

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("nproc", [2] + ([4] if gpu_count() >= 4 else []) +
                         ([8] if gpu_count() >= 8 else []))
def test_torchrun_ranks_match_oracle(nproc):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="4")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={29600 + nproc}", os.path.join(HERE, "mp_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    assert proc.stdout.count(": ok") == nproc, proc.stdout
