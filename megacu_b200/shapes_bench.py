"""Timing of the fused megakernel at benchmark configs 3 and 4, and of the
all-gather + GEMM (bench.py times config 2, mlp_bench config 5).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \\
        --master-addr 127.0.0.1 --master-port 29700 -m megacu_b200.shapes_bench --config 3
    ... -m megacu_b200.shapes_bench --config 4 [--m 16,32,64,128]
    ... -m megacu_b200.shapes_bench --config ag

Config 3: GEMM + reduce-scatter along M (sequence-parallel down-projection),
M = 8192, N = 8192, K = 28672 split over tp; PE p keeps rows [p M/tp, (p+1)
M/tp). Config 4: decode-shape GEMM + allreduce, M in {16, 32, 64, 128}, N =
8192, K = 28672 split over tp (one-shot exchange: one tile row). All-gather
(`ag`, the symmetric counterpart of config 3: the sequence-parallel input of
the up-projection): M = 8192 rows gathered from M/tp per PE, K = 8192,
N = 28672/tp columns per PE. Inputs bf16 N(0, 0.02^2), seeded per PE and
tensor; synthetic data.

Arms, timed interleaved step by step after a common heat-up, with L2 flushed
(a 256 MiB write) and the PEs aligned by a team barrier before every step,
outside the CUDA events; every step's time is the max over ranks:
  fused                    the megakernel (reduce-scatter, allreduce or
                           all-gather + GEMM)
  unfused                  torch.matmul (cuBLAS), then NCCL reduce_scatter /
                           all_reduce of its output; for `ag` NCCL
                           all_gather of A, then torch.matmul
  gemm_only                torch.matmul alone
  kernel_without_exchange  the megakernel's GEMM on one PE (this PE's K
                           slice; for `ag` the whole gathered A) (tp > 1):
                           the fused time minus this is the exchange time
                           the kernel did not hide
Configs 3 and ag report the mean per call, config 4 the p50 (and the mean,
``us_per_call_mean``, beside the step of the event timer seen in the samples,
``timer_tick_us``: where events advance in 2.048 us steps, a p50 of calls of
a few tens of microseconds moves in those steps and the mean does not). Prints one JSON
line per shape on rank 0. After the timing every rank checks the last timed
fused call (``parity``): its output against an fp32 reference of the same
inputs (each rank's slices multiplied in fp32, summed over the ranks by NCCL
in fp32; for `ag` the gathered A from NCCL's all-gather times this PE's B in
fp32), every rank's allreduce output bit-identical, the completion counters
of every launch against megacu's task graph (configs 3 and 4), and for `ag`
the gathered A bit for bit; the unfused output is held to the same
reference. A failed check makes the run exit non-zero.

``--graph`` times every arm as the replay of a CUDA graph captured from it
(launch overhead out of the measurement; an arm whose capture fails is timed
as launched and marked so). ``--algo one|two`` forces the allreduce exchange
of config 4 (auto picks one-shot for one tile row), and ``--multicast`` puts
the workspace and output in the team's multicast region: the in-switch
reduction (each block's sum over the PEs read with one load through the
NVSwitch; a two-shot allreduce also stores through it).
"""
from __future__ import annotations

import argparse
import json
import os

from .measure import (NVLINK_GBS, REL_TOL, STRICT_FLOOR, ClockSampler, all_ranks,
                      expected_counters, hbm_peak, interleaved, mean, output_errors, p50,
                      peaks, ranks_identical, reference_sum, seeded, timer_tick_us)

C3 = dict(m=8192, n=8192, k_total=28672)
C4 = dict(m=(16, 32, 64, 128), n=8192, k_total=28672)
AG = dict(m=8192, n_total=28672, k=8192)


def roofline(config, m, n, k, tp, us, one_shot=True, in_switch=False):
    """Slower of the GEMM at the measured bf16 peak, the weight stream at the
    measured HBM bandwidth (it bounds the decode shapes) and the exchange's
    bytes per PE over NVLink at the measured 770 GB/s per direction. m, n, k
    are one PE's GEMM (for `ag`, m is the gathered rows)."""
    peak, peak_src = peaks()
    hbm, hbm_src = hbm_peak()
    flops = 2.0 * m * n * k
    out_bytes = m * n * 2
    # Bytes a PE moves in its busier NVLink direction. Through the switch a
    # reducer's load reads every PE's slot, the requester's own included.
    if config == 3 and in_switch:
        link = out_bytes                          # every partial tile read once by its owner
        link_kind = "in-switch reduce-scatter 1 x output"
    elif config == 3:
        link = (tp - 1) / tp * out_bytes          # reduce-scatter bus bytes
        link_kind = "reduce-scatter (tp-1)/tp x output"
    elif config == "ag":
        link = (tp - 1) / tp * m * k * 2          # the other PEs' shards of A, received
        link_kind = "all-gather (tp-1)/tp x A"
    elif one_shot and in_switch:
        link = tp * out_bytes                     # every PE reads every PE's partial
        link_kind = "in-switch one-shot tp x output"
    elif one_shot:
        link = (tp - 1) * out_bytes               # one-shot: every partial to every peer
        link_kind = "one-shot (tp-1) x output"
    elif in_switch:
        link = (1 + 1 / tp) * out_bytes           # NVLS: each PE's slots and sums once
        link_kind = "in-switch two-shot (1 + 1/tp) x output"
    else:
        link = 2 * (tp - 1) / tp * out_bytes      # two-shot bus bytes
        link_kind = "two-shot 2 (tp-1)/tp x output"
    # Bytes the GEMM must move through HBM at least once: A, B and the
    # partial / output tile writes (for `ag` also the gathered A's write).
    hbm_bytes = 2.0 * (m * k + k * n) + out_bytes
    if config == "ag":
        hbm_bytes += 2.0 * m * k
    terms = {"tensor": flops / (peak * 1e12) * 1e6,
             "hbm": hbm_bytes / (hbm * 1e9) * 1e6,
             "nvlink": link / (NVLINK_GBS * 1e9) * 1e6}
    bound = max(terms, key=terms.get)
    return {"bound": bound, "terms_us": terms, "roofline_us": terms[bound],
            "frac": terms[bound] / us, "flops_per_pe": flops, "hbm_bytes_per_pe": hbm_bytes,
            "link_bytes_per_pe": link, "link": link_kind, "peak_tflops": peak,
            "peak_source": peak_src, "hbm_gbs": hbm, "hbm_source": hbm_src}


def as_graphs(arms, names, stream):
    """CUDA-graph versions of the arms (each captured from one call after the
    warm-up); an arm that cannot be captured stays as it is. Returns the arms
    and, per arm, whether it is a graph replay. The arms launch on the current
    stream, which inside the capture is the capturing stream."""
    import torch

    out, graphed = [], {}
    for arm, name in zip(arms, names):
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                arm()
            torch.cuda.synchronize()
            out.append(g.replay)
            graphed[name] = True
        except Exception:  # noqa: BLE001 - the arm is then timed as launched
            torch.cuda.synchronize()
            out.append(arm)
            graphed[name] = False
    return out, graphed


def run_shape(args, config, m, n, k_total, rank, world, local, team_cache):
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    tp = world
    k = k_total // tp
    mode = mb.MODE_REDUCE_SCATTER if config == 3 else mb.MODE_ALLREDUCE
    algo = {"auto": mb.ALGO_AUTO, "one": mb.ALGO_ONE_SHOT, "two": mb.ALGO_TWO_SHOT}[args.algo]
    a = seeded(1000 * config + 10 * rank + 0, (m, k), 0.02).to(dev)
    b = seeded(1000 * config + 10 * rank + 1, (k, n), 0.02).to(dev)
    prob = mb.Problem(m, n, k, mode=mode, algo=algo if config == 4 else mb.ALGO_AUTO,
                      timeout_ns=30_000_000_000)
    pl = mb.plan(prob, tp)
    ws_bytes = max(mb.workspace_bytes(prob, tp), 16)
    ev_bytes = mb.events_bytes(prob, tp)
    rows = m // tp if config == 3 else m
    want_mc = args.multicast and tp > 1
    team = team_cache(ws_bytes + ev_bytes + rows * n * 2 + (64 << 20),
                      (ws_bytes + rows * n * 2 + (1 << 20)) if want_mc else 0)
    use_mc = want_mc and team.multicast
    ws = team.tensor((ws_bytes,), torch.uint8, multicast=use_mc)
    events = team.tensor((ev_bytes // 4,), torch.int32)
    out = team.tensor((rows, n), torch.bfloat16, multicast=use_mc)
    c = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    c_rs = torch.empty((rows, n), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def fused():
        mb.gemm_allreduce(a, b, out, workspace=ws, events=events, problem=prob,
                          stream=torch.cuda.current_stream(), device=local,
                          team=team if tp > 1 else None)

    def unfused():
        torch.matmul(a, b, out=c)
        if tp > 1:
            if config == 3:
                dist.reduce_scatter_tensor(c_rs, c)
            else:
                dist.all_reduce(c)

    def gemm_only():
        torch.matmul(a, b, out=c)

    arms, names = [fused, unfused, gemm_only], ["fused", "unfused", "gemm_only"]
    solo_events = None
    if tp > 1:
        solo_prob = mb.Problem(m, n, k, timeout_ns=30_000_000_000)
        solo_events = torch.zeros(mb.events_bytes(solo_prob, 1) // 4, dtype=torch.int32,
                                  device=dev)
        solo_out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

        def kernel_without_exchange():
            mb.gemm_allreduce(a, b, solo_out, workspace=None, events=solo_events,
                              problem=solo_prob, stream=torch.cuda.current_stream(), device=local)

        arms.append(kernel_without_exchange)
        names.append("kernel_without_exchange")

    def align():
        flush.fill_(1)
        if tp > 1:
            team.barrier(stream)

    heat = args.heat_calls if args.heat_calls >= 0 else (200 if config == 3 else 2000)
    graphed = None
    with ClockSampler(local) as clocks:
        for _ in range(heat):
            fused()
            unfused()
        torch.cuda.synchronize()
        if args.graph:
            arms, graphed = as_graphs(arms, names, stream)
        ms = interleaved(arms, args.steps, args.warmup, align, stream, world, device=dev)
    mb.events_status(events, stream)
    if solo_events is not None:
        mb.events_status(solo_events, stream)
    parity = check_shape(a, b, out, c, c_rs, unfused, pl, config, tp, rank, dev, events, stream,
                         launches=heat + args.warmup + args.steps)
    stat = mean if config == 3 else p50
    us = {name: stat(v) * 1e3 for name, v in zip(names, ms)}
    flops_job = 2.0 * m * n * k_total
    line = {
        "workload": (f"C3 GEMM+reduce-scatter M{m} N{n} K{k_total}/tp bf16" if config == 3 else
                     f"C4 decode GEMM+allreduce M{m} N{n} K{k_total}/tp bf16"),
        "tp": tp, "m": m, "n": n, "k_per_pe": k, "steps": args.steps, "warmup": args.warmup,
        "statistic": "mean" if config == 3 else "p50", "data": "synthetic",
        "us_per_call": us,
        "us_per_call_mean": {name: mean(v) * 1e3 for name, v in zip(names, ms)},
        "timer_tick_us": timer_tick_us(ms),
        "tflops_per_gpu": {name: flops_job / tp / (u * 1e-6) / 1e12 for name, u in us.items()},
        "plan": {"tile": [pl.tile_m, pl.tile_n], "tiles": pl.tiles, "one_shot": pl.one_shot,
                 "cta_pairs": pl.cta_pairs, "gemm_units": pl.gemm_units,
                 "in_switch": use_mc},
        "roofline_call": roofline(config, m, n, k, tp, us["fused"], one_shot=pl.one_shot,
                                  in_switch=use_mc),
        "exposed_comm_us": (us["fused"] - us["kernel_without_exchange"]) if tp > 1 else None,
        "l2": "flushed (256 MiB write) before every timed step",
        "cuda_graph_replay": graphed,
        "clocks": clocks.summary(),
        "parity": parity,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    return parity["ok"]


def _parity_header(bf16_wire):
    return {"reference": "each rank's bf16 slices multiplied in fp32 (TF32 off), summed over "
                         "the ranks by NCCL in fp32",
            "tol": REL_TOL,
            "max_rel_err_denominator": "sum over ranks of |partial| + RMS(want) (bf16 partials "
                                       "on the wire)" if bf16_wire else "|want| + RMS(want)",
            "strict_floor": f"|want| >= {STRICT_FLOOR} x RMS(want)"}


def check_shape(a, b, out, c, c_rs, unfused, pl, config, tp, rank, dev, events, stream,
                launches):
    """Checks the last timed fused call of configs 3 / 4 on every rank (the
    same collectives on every rank, in the same order)."""
    import torch

    import megacu_b200 as mb
    torch.cuda.synchronize()
    want, scale = reference_sum(a, b, tp)
    rows = out.shape[0]
    if config == 3:  # this PE's rows of the reduce-scattered sum
        want = want[rank * rows:(rank + 1) * rows]
        scale = scale[rank * rows:(rank + 1) * rows]
    bf16_wire = tp > 1 and pl.wire_bytes == 2
    parity = _parity_header(bf16_wire)
    parity.update(output_errors(out, want, scale if bf16_wire else None))
    parity["ranks_identical"] = ranks_identical(out, tp) if config == 4 else None
    mode = 1 if config == 3 else 0
    per_call = expected_counters(tp, rank, pl.m_tiles, pl.n_tiles, pl.tile_n, pl.one_shot, mode)
    whole = out.shape[0] % 128 == 0 or config == 3
    counters = mb.events_counters(events, stream)
    counters_ok = (counters == [launches * x for x in per_call]) if whole else (
        counters[6] == launches and counters[7] == 0)
    ok = parity["max_rel_err"] < REL_TOL and counters_ok and parity["ranks_identical"] is not False
    if not bf16_wire:
        ok = ok and parity["max_rel_err_strict"] < REL_TOL
    unfused()
    torch.cuda.synchronize()
    parity["unfused_cublas_nccl"] = output_errors(c_rs if (config == 3 and tp > 1) else c, want)
    del want, scale
    parity["counters_ok"] = all_ranks(counters_ok, tp, dev)
    parity["ok"] = all_ranks(ok, tp, dev)
    return parity


def run_allgather(args, rank, world, local, team_cache):
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    tp = world
    m, k = AG["m"], AG["k"]
    n = AG["n_total"] // tp
    rows = m // tp
    shard_host = seeded(6000 + 10 * rank + 0, (rows, k), 0.02)
    b = seeded(6000 + 10 * rank + 1, (k, n), 0.02).to(dev)
    prob = mb.Problem(m, n, k, mode=mb.MODE_ALLGATHER, timeout_ns=30_000_000_000)
    pl = mb.plan(prob, tp)
    ev_bytes = mb.events_bytes(prob, tp)
    team = team_cache(rows * k * 2 + ev_bytes + (64 << 20))
    shard = team.tensor((rows, k), torch.bfloat16)
    shard.copy_(shard_host)
    events = team.tensor((ev_bytes // 4,), torch.int32)
    gathered = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    g_nccl = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    c = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def fused():
        mb.allgather_gemm(shard, b, gathered, out, events=events, problem=prob,
                          stream=torch.cuda.current_stream(),
                          device=local, team=team if tp > 1 else None)

    def unfused():
        if tp > 1:
            dist.all_gather_into_tensor(g_nccl, shard)
        else:
            g_nccl.copy_(shard)
        torch.matmul(g_nccl, b, out=c)

    def gemm_only():
        torch.matmul(g_nccl, b, out=c)

    arms, names = [fused, unfused, gemm_only], ["fused", "unfused", "gemm_only"]
    solo_events = None
    if tp > 1:
        solo_prob = mb.Problem(m, n, k, timeout_ns=30_000_000_000)
        solo_events = torch.zeros(mb.events_bytes(solo_prob, 1) // 4, dtype=torch.int32,
                                  device=dev)
        solo_out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

        def kernel_without_exchange():
            mb.gemm_allreduce(g_nccl, b, solo_out, workspace=None, events=solo_events,
                              problem=solo_prob, stream=torch.cuda.current_stream(), device=local)

        arms.append(kernel_without_exchange)
        names.append("kernel_without_exchange")

    def align():
        flush.fill_(1)
        if tp > 1:
            team.barrier(stream)

    heat = args.heat_calls if args.heat_calls >= 0 else 200
    with ClockSampler(local) as clocks:
        for _ in range(heat):
            fused()
            unfused()
        torch.cuda.synchronize()
        ms = interleaved(arms, args.steps, args.warmup, align, stream, world, device=dev)
    mb.events_status(events, stream)
    if solo_events is not None:
        mb.events_status(solo_events, stream)
    # Check of the last timed call: the gathered A bit for bit against NCCL's
    # all-gather of the same shards (the unfused arm's g_nccl), the output
    # against g_nccl @ B in fp32 (one PE's GEMM: the strict measure applies).
    torch.cuda.synchronize()
    unfused()
    torch.cuda.synchronize()
    torch.backends.cuda.matmul.allow_tf32 = False
    want = torch.empty((m, n), dtype=torch.float32, device=dev)
    bf = b.float()
    for r0 in range(0, m, 1024):
        want[r0:r0 + 1024] = torch.matmul(g_nccl[r0:r0 + 1024].float(), bf)
    del bf
    parity = _parity_header(False)
    parity.update(output_errors(out, want))
    parity["gathered_bit_exact"] = bool(torch.equal(gathered, g_nccl))
    parity["unfused_cublas_nccl"] = output_errors(c, want)
    del want
    ok = (parity["max_rel_err"] < REL_TOL and parity["max_rel_err_strict"] < REL_TOL and
          parity["gathered_bit_exact"])
    parity["ok"] = all_ranks(ok, tp, dev)
    us = {name: mean(v) * 1e3 for name, v in zip(names, ms)}
    flops_pe = 2.0 * m * n * k
    line = {
        "workload": f"all-gather + GEMM M{m} (M/tp per PE) K{k} N{AG['n_total']}/tp bf16",
        "tp": tp, "m": m, "n_per_pe": n, "k": k, "steps": args.steps, "warmup": args.warmup,
        "statistic": "mean", "data": "synthetic",
        "us_per_call": us,
        "tflops_per_gpu": {name: flops_pe / (u * 1e-6) / 1e12 for name, u in us.items()},
        "plan": {"tile": [pl.tile_m, pl.tile_n], "tiles": pl.tiles,
                 "cta_pairs": pl.cta_pairs, "gemm_units": pl.gemm_units},
        "roofline_call": roofline("ag", m, n, k, tp, us["fused"]),
        "exposed_comm_us": (us["fused"] - us["kernel_without_exchange"]) if tp > 1 else None,
        "l2": "flushed (256 MiB write) before every timed step",
        "clocks": clocks.summary(),
        "parity": parity,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    return parity["ok"]


def main() -> int:
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--config", choices=("3", "4", "ag"), required=True)
    ap.add_argument("--m", default="", help="config 4: comma-separated token counts")
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--algo", choices=("auto", "one", "two"), default="auto",
                    help="config 4: the allreduce exchange (auto: one-shot for one tile row)")
    ap.add_argument("--multicast", action="store_true",
                    help="reduce in the switch (workspace and out in the team multicast region)")
    ap.add_argument("--graph", action="store_true",
                    help="time each arm as the replay of a CUDA graph captured from it")
    ap.add_argument("--k-total", type=int, default=0,
                    help="configs 3 and 4: the total K split over the PEs (default the "
                         "config's 28672); e.g. 3584 on one GPU is one PE's GEMM at tp = 8")
    ap.add_argument("--heat-calls", type=int, default=-1,
                    help="untimed calls of the fused and unfused arms before timing "
                         "(default: about two seconds of work)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    teams = []

    def team_cache(heap_bytes, multicast_bytes=0):
        # One team per shape (a team's heap is sized once); the previous one
        # is closed first, collectively.
        for t in teams:
            t.close()
        teams.clear()
        teams.append(mb.Team(rank, world, local, heap_bytes,
                             mb.torch_exchange() if world > 1 else None,
                             multicast_bytes=multicast_bytes))
        return teams[0]

    ok = True
    try:
        if args.config == "ag":
            ok = run_allgather(args, rank, world, local, team_cache)
        elif args.config == "3":
            ok = run_shape(args, 3, C3["m"], C3["n"], args.k_total or C3["k_total"], rank,
                           world, local, team_cache)
        else:
            ms = [int(x) for x in args.m.split(",") if x] or list(C4["m"])
            for m in ms:
                ok = run_shape(args, 4, m, C4["n"], args.k_total or C4["k_total"], rank,
                               world, local, team_cache) and ok
        for t in teams:
            t.close()
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
