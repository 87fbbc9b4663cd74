"""Benchmark of the fused bf16 GEMM + allreduce megakernel (benchmark config 2).

Workload: row-parallel GEMM + allreduce, M = 4096, N = 8192, K = 8192 split
over tp = N GPUs (each PE: A [4096, 8192/tp], B [8192/tp, 8192], bf16 N(0,
0.02^2)), output [4096, 8192] bf16 allreduced. Total work is fixed as tp
grows (strong scaling). One "step" is one call of the megakernel.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints ONE JSON line on rank 0. Timing: every step is bracketed by CUDA
events on the launching stream; L2 is flushed (a 256 MiB write) and the PEs
are aligned by a device-side team barrier before every timed step, both
outside the events; the whole timed region is bracketed by a barrier and a
device synchronise; the reported time is the max over ranks.

After the timing, every rank checks the output of the last timed call
(``parity`` in the line): against an fp32 reference of the same inputs
(each rank's slices multiplied in fp32, summed over the ranks by NCCL in
fp32), bit identity of every rank's output, and the completion counters of
every call against megacu's task graph; likewise the deterministic mode
(fp32 partials on the wire, fixed PE-order sum), which must also give the
same bits twice. A failed check makes the run exit non-zero after printing.

``--impl reference`` times the reference's path on the host cores instead:
megacu has no CPU implementation of its GEMM/allreduce math (its numeric path
is CUDA only), so this is the CPU restatement of its tile-task graph
(oracle/, sequential-k fp32 tile GEMM + PE-order fp32 reduction), rank 0
only, on a bounded sample of the same workload's output tiles.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from megacu_b200.measure import (NVLINK_GBS, REL_TOL, STRICT_FLOOR, ClockSampler,  # noqa: E402
                                  NvlinkCounters, all_ranks, burst_peak, expected_counters,
                                  interleaved, mean, output_errors, peaks, ranks_identical,
                                  reference_sum, seeded)

M, N, K_TOTAL = 4096, 8192, 8192
WORKLOAD = "C2 row-parallel GEMM+allreduce M4096 N8192 K8192/tp bf16"
METRIC = "GEMM+allreduce TFLOP/s (whole job), C2 M4096 N8192 K8192 split over tp"
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "traffic.json")


def traffic_for(key):
    """DRAM bytes of one launch from profiles/traffic.json (an ncu capture), or None."""
    try:
        with open(TRAFFIC_PATH) as f:
            return json.load(f).get(key)
    except Exception:
        return None


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ---------------------------------------------------------------------------
# CPU leg (oracle on the host cores): the reference arm and cpu_baseline
# ---------------------------------------------------------------------------

def cpu_sample(tp, seconds, threads):
    """Times the CPU restatement on whole output tiles of the workload."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib
    k = K_TOTAL // tp
    a = [seeded(2000 + 10 * pe + 0, (M, k), 0.02).float().numpy() for pe in range(tp)]
    b = [seeded(2000 + 10 * pe + 1, (k, N), 0.02).float().numpy() for pe in range(tp)]
    tile_n = 256
    tiles = (M // 128) * (N // tile_n)
    rng = np.random.default_rng(0)
    order = rng.permutation(tiles).astype(np.int32)
    done, elapsed, i = 0, 0.0, 0
    batch = max(threads, 1)
    while (elapsed < seconds or done == 0) and i < tiles:
        ids = order[i:i + batch]
        t0 = time.perf_counter()
        oracle_lib.bf16_tiles(a, b, ids, m=M, n=N, k=k, tile_n=tile_n, wire_bytes=2,
                              threads=threads)
        elapsed += time.perf_counter() - t0
        done += len(ids)
        i += batch
    flops = 2.0 * 128 * tile_n * K_TOTAL * done
    return flops / elapsed / 1e12, done, elapsed


def run_reference(args, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    tp = args.gpus
    for _ in range(args.warmup):
        cpu_sample(tp, 0.0, threads)
    vals, per_step = [], []
    for _ in range(args.steps):
        v, done, el = cpu_sample(tp, args.cpu_seconds / max(args.steps, 1), threads)
        vals.append(v)
        per_step.append(el)
    value = float(np.mean(vals))
    sample = (f"{done} of {(M // 128) * (N // 256)} output tiles (128x256, full K={K_TOTAL} "
              f"over {tp} logical PEs) per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * float(np.mean(per_step)), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "m": M, "n": N, "k_total": K_TOTAL, "tp": tp},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "megacu's GEMM/allreduce math exists only as a CUDA kernel; this arm is the "
                "CPU restatement of its tile-task graph (oracle/) on the host cores",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

def exchange_rate(trace, plan, tp, rank, in_switch, dev):
    """NVLink bytes a PE sends and receives in one call, over its exchange
    window from the kernel's trace; per rank and their mean / min."""
    import torch
    import torch.distributed as dist
    rec = trace.view(-1, 4).cpu().numpy().astype(np.uint64)
    rec = rec[rec[:, 3] != 0]
    red = (rec[:, 0] & 0xFF) == 2
    window_s = float(rec[red, 3].max() - rec[red, 2].min()) * 1e-9 if red.any() else 0.0
    s_out = M * N * 2
    s_wire = M * N * plan.wire_bytes
    if in_switch:
        # the switch reads every PE's whole partial for the owners' reductions
        # and multicasts each owner's sum into every PE's out
        sent, received = s_wire + s_out / tp, s_wire / tp + s_out
    elif plan.one_shot:
        sent = received = (tp - 1) * s_wire
    else:
        sent = received = (tp - 1) / tp * (s_wire + s_out)
    mine = torch.zeros((tp, 3), dtype=torch.float64, device=dev)
    mine[rank] = torch.tensor([window_s, sent, received], dtype=torch.float64)
    dist.all_reduce(mine)
    rows = mine.tolist()
    rates = [(x[1] / x[0] / 1e9 if x[0] > 0 else 0.0, x[2] / x[0] / 1e9 if x[0] > 0 else 0.0)
             for x in rows]
    return {"sent_bytes_per_pe": sent, "received_bytes_per_pe": received,
            "window_us": [round(x[0] * 1e6, 2) for x in rows],
            "sent_gbs": [round(r[0], 1) for r in rates],
            "received_gbs": [round(r[1], 1) for r in rates],
            "sent_gbs_mean": sum(r[0] for r in rates) / tp,
            "received_gbs_mean": sum(r[1] for r in rates) / tp,
            "vs_measured_770_gbs": max(sum(r[0] for r in rates), sum(r[1] for r in rates))
            / tp / NVLINK_GBS,
            "vs_nominal_900_gbs": max(sum(r[0] for r in rates), sum(r[1] for r in rates))
            / tp / 900.0,
            "source": "one traced call: first to last reduce sub-task of each PE "
                      "(%globaltimer); bytes per PE from the plan "
                      + ("(in-switch: partial read by the switch + 1/tp multicast out; "
                         "(1/tp) reduced + out multicast in)" if in_switch else
                         "(peer loads)")}


def check_outputs(a, b, out, c, unfused, plan, tp, rank, dev, launched, events, stream,
                  det=None):
    """Checks the last timed call on every rank (the same collectives on every
    rank, in the same order): the output against the fp32 reference of the
    same inputs summed over the ranks, bit identity across ranks, and the
    completion counters of every call on `events` (`launched` counts them)
    against megacu's task graph; the unfused baseline's output against the
    same reference; the deterministic mode (`det`) likewise, run once more for
    bit identity with its last timed call."""
    import torch

    import megacu_b200 as mb
    torch.cuda.synchronize()
    want, scale = reference_sum(a, b, tp)
    bf16_wire = tp > 1 and plan.wire_bytes == 2
    parity = {"reference": "each rank's bf16 slices multiplied in fp32 (TF32 off), summed over "
                           "the ranks by NCCL in fp32",
              "tol": REL_TOL,
              "max_rel_err_denominator": "sum over ranks of |partial| + RMS(want) (bf16 "
                                         "partials on the wire)" if bf16_wire else
                                         "|want| + RMS(want)",
              "strict_floor": f"|want| >= {STRICT_FLOOR} x RMS(want)"}
    parity.update(output_errors(out, want, scale if bf16_wire else None))
    parity["ranks_identical"] = ranks_identical(out, tp)
    per_call = expected_counters(tp, rank, plan.m_tiles, plan.n_tiles, plan.tile_n,
                                 plan.one_shot)
    counters_ok = mb.events_counters(events, stream) == [launched["fused"] * x for x in per_call]
    ok = parity["max_rel_err"] < REL_TOL and parity["ranks_identical"] and counters_ok
    if not bf16_wire:
        ok = ok and parity["max_rel_err_strict"] < REL_TOL
    # the unfused cuBLAS + NCCL output of the same inputs, against the same reference
    unfused()
    torch.cuda.synchronize()
    parity["unfused_cublas_nccl"] = output_errors(c, want)
    if det is not None:
        det_prob, det_out, det_events, det_call, align = det
        first = det_out.clone()
        align()
        det_call()
        torch.cuda.synchronize()
        mb.events_status(det_events, stream)
        d = output_errors(det_out, want)
        d["bit_reproducible"] = bool(torch.equal(first, det_out))
        d["ranks_identical"] = ranks_identical(det_out, tp)
        det_plan = mb.plan(det_prob, tp)
        det_per_call = expected_counters(tp, rank, det_plan.m_tiles, det_plan.n_tiles,
                                         det_plan.tile_n, det_plan.one_shot)
        det_counters_ok = (mb.events_counters(det_events, stream) ==
                           [launched["deterministic"] * x for x in det_per_call])
        counters_ok = counters_ok and det_counters_ok
        ok = (ok and d["max_rel_err"] < REL_TOL and d["max_rel_err_strict"] < REL_TOL and
              d["bit_reproducible"] and d["ranks_identical"] and det_counters_ok)
        parity["deterministic"] = d
        del first
    del want, scale
    parity["counters_ok"] = all_ranks(counters_ok, tp, dev)
    parity["ok"] = all_ranks(ok, tp, dev)
    return parity


def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    tp = world
    k = K_TOTAL // tp
    stream = torch.cuda.current_stream()

    # ---- inputs (seeded per rank and tensor) ----
    a_host = seeded(2000 + 10 * rank + 0, (M, k), 0.02).pin_memory()
    b_host = seeded(2000 + 10 * rank + 1, (k, N), 0.02).pin_memory()
    a = a_host.to(dev)
    b = b_host.to(dev)

    prob = mb.Problem(M, N, k, timeout_ns=30_000_000_000)
    plan = mb.plan(prob, tp)
    ws_bytes = mb.workspace_bytes(prob, tp)
    ev_bytes = mb.events_bytes(prob, tp)
    # The deterministic mode (fp32 partials on the wire, PE-order sum over
    # peer loads, bit-reproducible) is timed and checked beside the default
    # at tp > 1, with buffers of its own.
    det_prob = mb.Problem(M, N, k, deterministic=True, timeout_ns=30_000_000_000)
    det_ws_bytes = mb.workspace_bytes(det_prob, tp) if tp > 1 else 0
    det_ev_bytes = mb.events_bytes(det_prob, tp) if tp > 1 else 0
    det_bytes = det_ws_bytes + det_ev_bytes + M * N * 2 if tp > 1 else 0
    heap = ws_bytes + ev_bytes + M * N * 2 + det_bytes + (64 << 20)
    exchange = mb.torch_exchange() if tp > 1 else None
    # Two-shot allreduce: workspace and out in a multicast region select the
    # in-switch reduction (NVLS); without one the exchange uses peer loads.
    want_mc = tp > 1 and not plan.one_shot
    team = mb.Team(rank, tp, local_rank, heap, exchange,
                   multicast_bytes=(ws_bytes + M * N * 2 + (1 << 20)) if want_mc else 0)
    use_mc = want_mc and team.multicast
    ws = team.tensor((max(ws_bytes, 16),), torch.uint8, multicast=use_mc)
    events = team.tensor((ev_bytes // 4,), torch.int32)
    out = team.tensor((M, N), torch.bfloat16, multicast=use_mc)
    exchange_kind = ("none" if tp == 1 else
                     "in-switch reduction (NVLS multimem) + peer flags" if use_mc else
                     "peer loads / stores over NVLink")
    # End to end, each rank reads back its own 1/tp of the output rows: every
    # rank holds the same allreduced result, so the job's result reaches the
    # host exactly once.
    rows_back = M // tp
    out_host = torch.empty((rows_back, N), dtype=torch.bfloat16).pin_memory()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    launched = {"fused": 0, "deterministic": 0}  # launches on each events buffer

    def call(aa, bb, trace=None):
        launched["fused"] += 1
        mb.gemm_allreduce(aa, bb, out, workspace=ws, events=events, problem=prob, stream=stream,
                          device=local_rank, team=team if tp > 1 else None, trace=trace)

    def align():
        flush.fill_(1)
        if tp > 1:
            team.barrier(stream)

    def timed_steps(bodies, steps, warmup):
        """Times each body `steps` times with CUDA events, interleaved step by
        step (body 0, body 1, ..., then the next step) so that every arm sees
        the same clocks and temperature; returns, per body, the ms of every
        step, each the max over ranks (megacu_b200.measure.interleaved)."""
        return interleaved(bodies, steps, warmup, align, stream, tp, device=dev)

    # ---- fused megakernel (inputs resident) and the unfused baseline ----
    # Unfused baseline: cuBLAS GEMM, then NCCL allreduce of its output.
    c = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

    def fused():
        call(a, b)

    def unfused():
        torch.matmul(a, b, out=c)
        if tp > 1:
            dist.all_reduce(c)

    def gemm_only():
        torch.matmul(a, b, out=c)

    # The same kernel without its exchange: this PE's GEMM (its K slice) as a
    # one-PE call into a local output. The fused call minus this is the
    # exchange time the kernel did not hide behind its GEMM.
    arms = [fused, unfused, gemm_only]
    if tp > 1:
        solo_prob = mb.Problem(M, N, k, timeout_ns=30_000_000_000)
        solo_events = torch.zeros(mb.events_bytes(solo_prob, 1) // 4, dtype=torch.int32,
                                  device=dev)
        solo_out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

        def kernel_without_exchange():
            mb.gemm_allreduce(a, b, solo_out, workspace=None, events=solo_events,
                              problem=solo_prob, stream=stream, device=local_rank)

        det_ws = team.tensor((max(det_ws_bytes, 16),), torch.uint8)
        det_events = team.tensor((det_ev_bytes // 4,), torch.int32)
        det_out = team.tensor((M, N), torch.bfloat16)

        def deterministic():
            launched["deterministic"] += 1
            mb.gemm_allreduce(a, b, det_out, workspace=det_ws, events=det_events,
                              problem=det_prob, stream=stream, device=local_rank, team=team)

        arms += [kernel_without_exchange, deterministic]

    # The clock sampler runs from the heat-up through the timed steps. The
    # heat-up (a fixed number of untimed calls of both arms, the same on every
    # rank: each call is a collective) brings the GPU to its power-capped
    # steady state and gives nvidia-smi time to sample it under load; the
    # arms are then timed interleaved.
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.heat_calls):
            fused()
            unfused()
        torch.cuda.synchronize()
        step_ms = timed_steps(arms, args.steps, args.warmup)
    times = [mean(x) for x in step_ms]
    ms_fused, ms_unfused, ms_gemm = times[:3]
    ms_solo = times[3] if tp > 1 else None
    ms_det = times[4] if tp > 1 else None
    fused_sorted = sorted(step_ms[0])
    last = len(fused_sorted) - 1
    fused_stats = {q: fused_sorted[min(last, int(frac * len(fused_sorted)))] * 1e3
                   for q, frac in (("p10", 0.1), ("p50", 0.5), ("p90", 0.9))}
    mb.events_status(events, stream)
    if tp > 1:
        mb.events_status(solo_events, stream)
        mb.events_status(det_events, stream)
    flops_total = 2.0 * M * N * K_TOTAL
    flops_rank = flops_total / tp
    value = flops_total / (ms_fused * 1e-3) / 1e12

    # ---- NVLink bytes of the fused call (NVML counters, best effort) ----
    # 20 back-to-back calls between two counter reads; per call and per GB/s
    # over their CUDA-event time, averaged over the ranks.
    nvlink = None
    if tp > 1:
        counters = NvlinkCounters(local_rank)
        calls = 20
        torch.cuda.synchronize()
        team.barrier(stream)
        before = counters.read()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(calls):
            fused()
        c1.record(stream)
        torch.cuda.synchronize()
        after = counters.read()
        ok = before is not None and after is not None
        per_call_s = c0.elapsed_time(c1) * 1e-3 / calls
        tx = (after[0] - before[0]) / calls if ok else 0.0
        rx = (after[1] - before[1]) / calls if ok else 0.0
        agg = torch.tensor([tx, rx, 1.0 if ok else 0.0, per_call_s], dtype=torch.float64, device=dev)
        dist.all_reduce(agg)
        if agg[2].item() == tp:
            tx_m, rx_m, _, sec = (agg / tp).tolist()
            nvlink = {"tx_bytes_per_call": tx_m, "rx_bytes_per_call": rx_m,
                      "tx_gbs": tx_m / sec / 1e9, "rx_gbs": rx_m / sec / 1e9,
                      "us_per_call": sec * 1e6,
                      "source": "NVML NVLINK_THROUGHPUT_DATA_TX/RX summed over links, "
                                "mean over ranks, 20 back-to-back calls"}

    # ---- end to end: pinned host inputs in, output back out ----
    def e2e_body():
        a.copy_(a_host, non_blocking=True)
        b.copy_(b_host, non_blocking=True)
        call(a, b)
        out_host.copy_(out[rank * rows_back:(rank + 1) * rows_back], non_blocking=True)

    (e2e_steps,) = timed_steps([e2e_body], max(3, args.steps // 2), max(1, args.warmup // 2))
    ms_e2e = mean(e2e_steps)
    h2d = a_host.numel() * 2 + b_host.numel() * 2
    d2h = out_host.numel() * 2

    # ---- exchange rate from the kernel's own trace (tp > 1) ----
    # One traced call (L2 flushed, PEs aligned): the exchange window of a PE
    # runs from its first reduce sub-task's start to its last one's end
    # (%globaltimer, trace kind 2); the bytes a PE sends and receives over
    # NVLink in it follow from the plan.
    nvlink_achieved = None
    if tp > 1:
        trace = torch.zeros(plan.tiles * 64 * 4, dtype=torch.int64, device=dev)
        align()
        call(a, b, trace=trace)
        torch.cuda.synchronize()
        mb.events_status(events, stream)
        nvlink_achieved = exchange_rate(trace, plan, tp, rank, use_mc, dev)
        del trace

    # ---- output check of the timed calls ----
    parity = check_outputs(a, b, out, c, unfused, plan, tp, rank, dev, launched, events, stream,
                           det=(det_prob, det_out, det_events, deterministic, align)
                           if tp > 1 else None)

    # ---- CPU baseline (rank 0, N = 1 only) ----
    cpu = None
    if rank == 0 and tp == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        v, done, el = cpu_sample(tp, args.cpu_seconds, threads)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{done} output tiles of 128x256 with full K={K_TOTAL} "
                         f"({el:.1f} s of CPU time, oracle/ restatement)"}

    # One call timed after an L2 flush is held against the burst peak; the
    # sustained one (a seconds-long cuBLAS loop under the power cap) is given
    # beside it.
    peak, peak_src = burst_peak()
    peak_sustained, _ = peaks()
    achieved = flops_rank / (ms_fused * 1e-3) / 1e12
    # North-star roofline: the slower of the GEMM at the measured peak and the
    # allreduce's bytes per PE over NVLink (its bus bytes, 2 (tp-1)/tp of the
    # bf16 output: what a two-shot exchange over peer memory moves each way,
    # and NCCL's busbw definition) at the measured 770 GB/s per direction.
    # The in-switch reduction moves fewer bytes per PE, (1 + 1/tp) of the
    # output each way; that figure is reported beside it.
    out_bytes = M * N * 2
    link_bytes = 2.0 * (tp - 1) / tp * out_bytes
    switch_bytes = (1.0 + 1.0 / tp) * out_bytes if use_mc else None
    t_gemm_us = flops_rank / (peak * 1e12) * 1e6
    t_link_us = link_bytes / (NVLINK_GBS * 1e9) * 1e6
    t_roof_us = max(t_gemm_us, t_link_us)
    traffic = traffic_for(f"gemm_ar_megakernel_tp{tp}")
    launches_per_step = 1  # the megakernel; the team barrier runs before each step's events
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_fused,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "m": M, "n": N, "k_total": K_TOTAL, "k_per_pe": k,
                       "tp": tp, "parallelism": f"tp{tp}", "tile": [plan.tile_m, plan.tile_n],
                       "one_shot": plan.one_shot, "cta_pairs": plan.cta_pairs,
                       "exchange": exchange_kind,
                       "l2": "flushed (256 MiB write) before every timed step"},
            "us_per_call": ms_fused * 1e3,
            "us_per_call_stats": dict(fused_stats, steps=args.steps,
                                      note="per-step max over ranks; us_per_call is their mean"),
            "tflops_per_gpu": achieved,
            "e2e": {"value": flops_total / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "readback": "each rank its 1/tp of the output rows (the result once per job)",
                    "ms_per_step": ms_e2e},
            "gpu_launches": args.steps * launches_per_step,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": peak_src,
                         "frac_of_sustained": achieved / peak_sustained,
                         "peak_sustained": peak_sustained,
                         "traffic": traffic,
                         "kernel": "gemm_ar_megakernel", "per_launch_flops": flops_rank},
            "roofline_call": {"bound": "nvlink" if t_link_us > t_gemm_us else "tensor",
                              "gemm_us_at_peak": t_gemm_us, "link_bytes_per_pe": link_bytes,
                              "link_us_at_770GBps": t_link_us, "roofline_us": t_roof_us,
                              "frac": t_roof_us / (ms_fused * 1e3),
                              "in_switch_link_bytes_per_pe": switch_bytes,
                              "note": "slower of GEMM at the measured peak and the allreduce "
                                      "bus bytes 2(tp-1)/tp x output at the measured 770 GB/s "
                                      "per direction (900 nominal)"},
            "exposed_comm": None if ms_solo is None else {
                "us": (ms_fused - ms_solo) * 1e3,
                "kernel_without_exchange_us": ms_solo * 1e3,
                "note": "fused call minus the same kernel on one PE with this PE's K slice "
                        "(no exchange), timed interleaved with the other arms"},
            "nvlink_measured": nvlink,
            "nvlink_achieved": nvlink_achieved,
            "deterministic": None if ms_det is None else {
                "us": ms_det * 1e3, "tflops": flops_total / (ms_det * 1e-3) / 1e12,
                "note": "deterministic = 1: fp32 partials over peer loads, PE-order sum, "
                        "bit-reproducible; timed interleaved with the other arms"},
            "parity": parity,
            "cpu_baseline": cpu,
            "unfused_cublas_nccl": {"us": ms_unfused * 1e3, "gemm_us": ms_gemm * 1e3,
                                    "comm_us": max(ms_unfused - ms_gemm, 0.0) * 1e3,
                                    "tflops": flops_total / (ms_unfused * 1e-3) / 1e12,
                                    "timing": "interleaved step by step with the fused "
                                              "arm, after the same heat-up"},
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    team.close()
    return parity["ok"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="megacu_b200", choices=["megacu_b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--heat-calls", type=int, default=1000,
                    help="untimed calls before the warm-up, while clocks are sampled")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        ok = run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if not ok:
        print(f"rank {rank}: output check failed (see the line's parity object)",
              file=sys.stderr, flush=True)
        sys.exit(1)


if __name__ == "__main__":
    main()
