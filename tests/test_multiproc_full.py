"""Full-size multi-GPU parity (benchmark configs 2 and 3 at their sizes, K
split over the ranks) under torchrun, one rank per GPU: tests/mp_full_worker.py.

The kernel paths it calls are the ones test_multiproc.py checks against the
oracle at small sizes.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import gpu_count

HERE = os.path.dirname(os.path.abspath(__file__))

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.multigpu,
    pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs"),
]


@pytest.mark.parametrize("nproc", [2] + ([4] if gpu_count() >= 4 else []) +
                         ([8] if gpu_count() >= 8 else []))
def test_full_size_ranks_agree_with_fp32_reference(nproc):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="4")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={29650 + nproc}", os.path.join(HERE, "mp_full_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    assert proc.stdout.count(": ok") == nproc, proc.stdout
