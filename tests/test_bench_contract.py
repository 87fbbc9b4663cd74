"""bench.py's JSON line, checked without a GPU.

The GPU leg (`run_gpu`) runs with CPU stand-ins for its CUDA calls: CUDA
events that report a fixed time per rank, a no-op in place of the fused
kernel and of cuBLAS, a team whose tensors are host tensors, and the "cuda"
device mapped to the host. bench.py itself is not changed: its source is
executed with `torch.device("cuda"` read as `torch.device("cpu"`. The numbers
mean nothing; the test checks that the line carries every key of the
driver's contract, that its arithmetic follows from the step times (value,
roofline fraction, bytes per step, launches), and, with two gloo ranks, that
the reported time is the max over ranks and only rank 0 prints. The
reference arm (`--impl reference`) runs for real, on a short sample.
"""
from __future__ import annotations

import contextlib
import io
import json
import os
import subprocess
import sys

import pytest

import host_fakes
from host_fakes import rank_ms as _rank_ms

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
M, N, K_TOTAL = 4096, 8192, 8192
STEPS, WARMUP, HEAT = 4, 3, 2


def _check_kernel(name, args, kwargs):
    import torch
    assert name == "gemm_allreduce"
    a, b, out = args
    assert a.dtype == b.dtype == out.dtype == torch.bfloat16
    assert out.shape == (M, N) and a.shape[1] == b.shape[0] == kwargs["problem"].k


def _install_fakes(rank, launches, patch):
    host_fakes.install(rank, patch, launches, _check_kernel)


def _bench_module():
    return host_fakes.load_source("bench.py")


def _args(cpu_seconds=0.2, no_cpu=False):
    import argparse
    return argparse.Namespace(steps=STEPS, warmup=WARMUP, heat_calls=HEAT,
                              cpu_seconds=cpu_seconds, no_cpu=no_cpu)


REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
            "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks"}


def _check_line(line, tp, ms):
    assert REQUIRED <= set(line), REQUIRED - set(line)
    assert line["n_gpus"] == tp and line["steps"] == STEPS and line["warmup"] == WARMUP
    assert line["ms_per_step"] == pytest.approx(ms)
    flops = 2.0 * M * N * K_TOTAL
    assert line["value"] == pytest.approx(flops / (ms * 1e-3) / 1e12)
    assert line["higher_is_better"] is True and line["scaling"] == "strong"
    assert line["config"]["workload"] and line["config"]["tp"] == tp
    roof = line["roofline"]
    assert {"bound", "achieved", "peak", "unit", "frac", "traffic"} <= set(roof)
    assert roof["achieved"] == pytest.approx(flops / tp / (ms * 1e-3) / 1e12)
    assert roof["frac"] == pytest.approx(roof["achieved"] / roof["peak"])
    e2e = line["e2e"]
    k = K_TOTAL // tp
    assert e2e["h2d_bytes_per_step"] == (M * k + k * N) * 2
    assert e2e["d2h_bytes_per_step"] == (M // tp) * N * 2
    assert line["gpu_launches"] == STEPS
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(line["clocks"])
    # the output check ran on the stand-ins' outputs (zeros against a zero
    # reference) and the counters of every call matched the oracle's graph
    par = line["parity"]
    assert {"max_rel_err", "max_rel_err_strict", "ranks_identical", "counters_ok",
            "unfused_cublas_nccl", "ok"} <= set(par)
    assert par["counters_ok"] is True and par["ok"] is True
    if tp > 1:
        assert {"bit_reproducible", "max_rel_err_strict"} <= set(par["deterministic"])
        assert line["deterministic"]["us"] == pytest.approx(ms * 1e3)


def test_one_gpu_line(monkeypatch):
    launches = []
    _install_fakes(0, launches, monkeypatch.setattr)
    bench = _bench_module()
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        bench.run_gpu(_args(), 0, 1, 0)
    lines = [x for x in buf.getvalue().splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    _check_line(line, 1, _rank_ms(0))
    cpu = line["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cpu) and cpu["kind"] == "port"
    assert cpu["value"] > 0 and cpu["cores"] >= 1
    # heat-up, warm-up and timed steps of the fused arm, then the end-to-end
    # arm's warm-up and steps: every one a single launch of the kernel
    e2e_steps, e2e_warmup = max(3, STEPS // 2), max(1, WARMUP // 2)
    assert len(launches) == HEAT + WARMUP + STEPS + e2e_warmup + e2e_steps


def _rank_main(rank, out_dir, port):
    os.environ.update(RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60))
    launches = []
    _install_fakes(rank, launches, setattr)
    bench = _bench_module()
    buf = io.StringIO()
    try:
        with contextlib.redirect_stdout(buf):
            bench.run_gpu(_args(no_cpu=True), rank, 2, rank)
    finally:
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump({"stdout": buf.getvalue(), "launches": len(launches)}, f)


def test_two_rank_line_takes_the_max_over_ranks(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_rank_main, args=(str(tmp_path), port), nprocs=2, join=True)
    got = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    assert not any(x.startswith("{") for x in got[1]["stdout"].splitlines())
    lines = [x for x in got[0]["stdout"].splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    _check_line(line, 2, max(_rank_ms(0), _rank_ms(1)))
    assert line["cpu_baseline"] is None  # rank 0 at N = 1 only
    assert line["exposed_comm"] is not None
    # both ranks launched the same sequence (every launch is a collective)
    assert got[0]["launches"] == got[1]["launches"]


def test_reference_arm_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "3", "--cpu-seconds", "0.5"], cwd=ROOT,
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [x for x in proc.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["value"] == line["value"]
    assert {"kind", "cores", "sample"} <= set(line["cpu_baseline"])


def test_reference_arm_under_torchrun_prints_once(tmp_path):
    """The driver launches the reference arm like the GPU arm (torchrun for
    N > 1): rank 0 alone works and prints; every rank exits 0."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    proc = subprocess.run(
        ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run",
         "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
         "--master-port", str(port), "bench.py", "--impl", "reference", "--gpus", "2",
         "--steps", "1", "--warmup", "3", "--cpu-seconds", "0.5"],
        cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [x for x in proc.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["config"]["tp"] == 2
