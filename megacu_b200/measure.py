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
* ``reference_sum``, ``output_errors``, ``ranks_identical``,
  ``expected_counters``: the output check every timing tool runs on the
  calls it timed (an fp32 reference of the same inputs summed over the ranks
  by NCCL, both relative-error measures, bit identity across ranks, and the
  completion counters of megacu's task graph).
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


def burst_peak():
    """The dense bf16 peak of a kernel timed in isolation: the measured burst
    cuBLAS figure, else the sustained one, else the fallback."""
    p = _peaks_file()
    try:
        if "bf16_tflops" in p:
            return float(p["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
        return (float(p["bf16_tflops_sustained"]),
                "measured (MEASURED_PEAKS.json bf16_tflops_sustained)")
    except Exception:
        return FALLBACK_TFLOPS, "fallback (1.59 PFLOP/s, no MEASURED_PEAKS.json)"


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


def timer_tick_us(samples_ms):
    """The event timer's step as seen in per-step times (ms lists): the
    smallest positive difference between two distinct samples, in
    microseconds, or None with fewer than two distinct values. On some B200
    hosts CUDA events advance in 2.048 us steps, so a p50 of calls of a few
    tens of microseconds moves in those steps; the mean over many steps does
    not (the call's phase against the tick varies from step to step)."""
    values = sorted({round(x * 1e3, 4) for xs in samples_ms for x in xs})
    gaps = [b - a for a, b in zip(values, values[1:]) if b - a > 0]
    return round(min(gaps), 4) if gaps else None


# ---------------------------------------------------------------------------
# Output check of the timed calls
# ---------------------------------------------------------------------------

# Tolerance of the bf16 path (north star: max relative error 1e-2, bf16
# inputs, fp32 accumulate) and the floor of the strict measure: elements with
# |want| below STRICT_FLOOR x RMS(want) (about 0.8 % of a Gaussian output)
# are left out of max |got - want| / |want|. There the denominator nearly
# vanishes and any two fp32 accumulation orders differ by more than 1e-2 of
# the value: at C2 (K = 8192) cuBLAS's output against the fp32 reference
# reaches 1.5e-2 at a floor of 1e-3 x RMS, the same as the fused kernel's.
REL_TOL = 1e-2
STRICT_FLOOR = 1e-2


def reference_sum(a, b, world, rows=1024):
    """fp32 reference of the allreduced output and its condition: this rank's
    bf16 slices multiplied in fp32 (TF32 off), then summed over the ranks by
    NCCL in fp32. Returns (want, scale), scale = the sum over ranks of
    |partial| per element (what a bf16 partial's rounding is relative to)."""
    import torch
    import torch.distributed as dist
    torch.backends.cuda.matmul.allow_tf32 = False
    bf = b.float()
    m, n = a.shape[0], b.shape[1]
    want = torch.empty((m, n), dtype=torch.float32, device=a.device)
    scale = torch.empty_like(want)
    for r0 in range(0, m, rows):
        part = torch.matmul(a[r0:r0 + rows].float(), bf)
        want[r0:r0 + rows] = part
        scale[r0:r0 + rows] = part.abs()
    del bf
    if world > 1:
        dist.all_reduce(want)
        dist.all_reduce(scale)
    return want, scale


def output_errors(got, want, scale=None, rows=1024):
    """Both relative-error measures of `got` (any float dtype) against the
    fp32 `want`:

    * ``max_rel_err``: max |got - want| / (s + RMS(want)), s = |want|, or
      `scale` where given (the sum of the partials' magnitudes, for bf16
      partials on the wire, which are exact only to a bf16 ulp of
      themselves);
    * ``max_rel_err_strict``: max |got - want| / |want| over the elements with
      |want| >= STRICT_FLOOR x RMS(want).

    A NaN anywhere makes both NaN (which fails every comparison)."""
    import torch
    m = want.shape[0]
    sq = 0.0
    for r0 in range(0, m, rows):
        sq += float(want[r0:r0 + rows].double().pow(2).sum())
    rms = (sq / max(want.numel(), 1)) ** 0.5
    floor = STRICT_FLOOR * rms
    loose = strict = 0.0
    for r0 in range(0, m, rows):
        w = want[r0:r0 + rows]
        err = (got[r0:r0 + rows].float() - w).abs_()
        aw = w.abs()
        s = aw if scale is None else scale[r0:r0 + rows]
        loose = max(loose, float((err / (s + (rms + 1e-30))).max())) if err.numel() else loose
        keep = (aw >= floor) & (aw > 0)
        if bool(keep.any()):
            strict = max(strict, float((err[keep] / aw[keep]).max()))
        if bool(torch.isnan(err).any()):
            return {"max_rel_err": float("nan"), "max_rel_err_strict": float("nan")}
    return {"max_rel_err": loose, "max_rel_err_strict": strict}


def ranks_identical(t, world):
    """True on every rank when every rank's `t` holds the same bits as rank 0's."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return True
    ref = t.clone()
    dist.broadcast(ref, 0)
    same = torch.tensor([1 if torch.equal(ref, t) else 0], dtype=torch.int32, device=t.device)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    return bool(same.item())


def all_ranks(flag, world, device):
    """True when `flag` is true on every rank (every rank gets the answer)."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return bool(flag)
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def expected_counters(n_pes, me, m_tiles, n_tiles, tile_n, one_shot, mode=0):
    """Completion counters (layout.h's ctr_* order) that one call of the bf16
    kernel adds on PE `me`, for shapes whose every tile is whole (m a
    multiple of 128, n of tile_n). megacu's task graph per tile: task 0 (the
    GEMM tile) and its publish, per 32-row quarter, to each PE that reduces
    the tile; task 2 per (reduced tile, quarter, 64-column block), after
    acquiring every PE's partial of that quarter; in a two-shot allreduce the
    owner's stores into every PE's out count as final publishes, and each PE
    acquires every PE's done flag once. The tests pin this against the
    oracle's graph."""
    tiles = m_tiles * n_tiles
    blocks = tile_n // 64
    c = [0] * 8
    c[0] = tiles
    c[6] = 1
    if n_pes == 1:
        c[2] = tiles * 4
        return c
    c[2] = tiles * 4 * (n_pes if one_shot else 1)
    reduced = tiles if one_shot else (tiles - me + n_pes - 1) // n_pes
    c[1] = reduced * 4 * blocks
    c[3] = c[1] * n_pes
    if mode == 0 and not one_shot:
        c[4] = c[1] * n_pes
        c[5] = n_pes
    return c
