"""Measurement helpers shared by bench.py and the per-config timing tools
(``shapes_bench`` for configs 3 and 4, ``mlp_bench`` for config 5).

* ``seeded``: bf16 tensors drawn from N(0, std^2) in fp32 with a fixed seed,
  rounded to nearest even.
* ``peaks``: the roofline denominators, from MEASURED_PEAKS.json at the
  repository root (the driver's measurement on this pool's B200s) or the
  stated fallback.
* ``ClockSampler``: nvidia-smi SM clocks and throttle reasons, sampled while
  the timed region runs (reading only; no GPU setting is touched).
* ``NvlinkCounters``: NVML NVLink payload counters of one GPU.
* ``interleaved``: CUDA-event timing of several arms, interleaved step by
  step, the max over ranks of each step.
"""
from __future__ import annotations

import json
import os
import statistics
import subprocess
import threading

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0
NVLINK_GBS = 770.0  # measured peer copy per direction on this pool's B200s


def seeded(seed, shape, std):
    import torch
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)


def _peaks_file():
    try:
        with open(PEAKS_PATH) as f:
            return json.load(f)
    except Exception:
        return None


def peaks():
    """The dense bf16 peak for a kernel timed inside a long run of calls: the
    measured sustained cuBLAS figure (power-capped clocks), else the burst
    one, else the fallback."""
    p = _peaks_file()
    try:
        if "bf16_tflops_sustained" in p:
            return (float(p["bf16_tflops_sustained"]),
                    "measured (MEASURED_PEAKS.json bf16_tflops_sustained: cuBLAS back to back "
                    "under the power cap; the timed calls follow a heat-up run)")
        return float(p["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return FALLBACK_TFLOPS, "fallback (1.59 PFLOP/s, no MEASURED_PEAKS.json)"


def hbm_peak():
    """Measured copy bandwidth (GB/s, read + write bytes), else the fallback."""
    p = _peaks_file()
    try:
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, no MEASURED_PEAKS.json)"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


class NvlinkCounters:
    """NVML's NVLink data-throughput counters of one GPU (payload bytes sent
    and received, summed over its links); `read` gives None where NVML or the
    fields are unavailable. Reading counters changes no GPU setting."""

    def __init__(self, index):
        self.nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def read(self):
        if self.nvml is None:
            return None
        p = self.nvml
        try:
            ids = []
            for link in range(p.NVML_NVLINK_MAX_LINKS):
                ids.append((p.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX, link))
                ids.append((p.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX, link))
            vals = p.nvmlDeviceGetFieldValues(self.handle, ids)
            tx = rx = 0
            seen = False
            for i, v in enumerate(vals):
                if v.nvmlReturn != p.NVML_SUCCESS:
                    continue
                seen = True
                if i % 2 == 0:
                    tx += int(v.value.ullVal)
                else:
                    rx += int(v.value.ullVal)
            return (tx * 1024, rx * 1024) if seen else None  # the counters count KiB
        except Exception:
            return None


def interleaved(bodies, steps, warmup, align, stream, world, device=None):
    """Times each body ``steps`` times with CUDA events on ``stream``,
    interleaved step by step (body 0, body 1, ..., then the next step) so that
    every arm sees the same clocks and temperature. ``align()`` runs before
    every step outside the events (an L2 flush and a team barrier). Returns,
    per body, the list of per-step milliseconds, each the max over ranks
    (reduced on ``device``, the current CUDA device by default)."""
    import torch
    import torch.distributed as dist

    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())

    for _ in range(warmup):
        for body in bodies:
            align()
            body()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)] for _ in bodies]
    for i in range(steps):
        for body, evs in zip(bodies, ev):
            align()
            evs[i][0].record(stream)
            body()
            evs[i][1].record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([[s.elapsed_time(e) for s, e in evs] for evs in ev], dtype=torch.float64,
                      device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
    return ms.tolist()


def mean(xs):
    return sum(xs) / len(xs)


def p50(xs):
    return statistics.median(xs)
