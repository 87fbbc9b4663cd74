"""The event-tensor layouts the kernels index (tests/cpp/layout_check.cu,
compiled for the host with nvcc): every flag and counter word is distinct
and inside the size the host allocates, for the fused allreduce, the
all-gather and the single-launch MLP chain."""
from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_event_layouts_are_disjoint_and_in_bounds():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "layout_check")
        cmd = [nvcc, "-std=c++20", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
               "-I" + os.path.join(ROOT, "include"),
               "-I" + os.path.join(ROOT, "megacu_b200", "csrc"),
               os.path.join(ROOT, "tests", "cpp", "layout_check.cu"), "-o", exe]
        build = subprocess.run(cmd, capture_output=True, text=True)
        assert build.returncode == 0, build.stderr[-3000:]
        run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
        assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
