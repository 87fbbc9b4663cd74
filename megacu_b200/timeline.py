"""Where the time of one fused call goes, per PE, from the kernel's own trace.

Run one process per GPU (torchrun); rank 0 prints one JSON line per PE:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \\
        --master-addr 127.0.0.1 --master-port 29600 -m megacu_b200.timeline

The workload is bench.py's (C2: M 4096, N 8192, K 8192 split over the PEs,
synthetic N(0, 0.02^2) inputs); two-shot plans put workspace and out in a
multicast region when the team can have one (``--no-multicast`` keeps the
peer exchange). After ``--calls`` untimed calls and 10 timed ones (L2 flushed
and a team barrier before each), one call runs with tracing on. Times are
microseconds from the first traced event of the PE (the first GEMM tile's
epilogue): GEMM tiles end (median, last), reduce sub-tasks (first start, last
end, median duration), the workers' completion fences, the done-flag store
and the final wait (trace kinds 0, 2, 3, 4, 5).

``--allgather`` traces the all-gather + GEMM instead (M = --m rows gathered
from M/tp per PE, K = --k-total, N = --n columns per PE): GEMM tiles, and the
copy chunks (kind 6: first start, last end, median duration, and the last end
per shard distance, so one sees whether the copies stay ahead of the GEMM).
"""
from __future__ import annotations

import argparse
import json
import os


def _summary(tr, np):
    t0 = tr["t0"].astype(np.int64)
    t1 = tr["t1"].astype(np.int64)
    if t0.size == 0:
        return {"records": 0}  # the traced call recorded nothing
    base = t0.min()

    def us(x):
        return round(float(x - base) / 1e3, 1)

    out = {}
    g = tr["kind"] == 0
    if g.any():
        out["gemm_tiles"] = int(g.sum())
        out["gemm_end_p50_us"] = us(np.percentile(t1[g], 50))
        out["gemm_end_us"] = us(t1[g].max())
    r = tr["kind"] == 2
    if r.any():
        out["reduce_tasks"] = int(r.sum())
        out["reduce_first_start_us"] = us(t0[r].min())
        out["reduce_end_us"] = us(t1[r].max())
        out["reduce_task_p50_us"] = round(float(np.percentile(t1[r] - t0[r], 50)) / 1e3, 1)
    c = tr["kind"] == 6
    if c.any():
        out["copy_chunks"] = int(c.sum())
        out["copy_first_start_us"] = us(t0[c].min())
        out["copy_end_us"] = us(t1[c].max())
        out["copy_chunk_p50_us"] = round(float(np.percentile(t1[c] - t0[c], 50)) / 1e3, 1)
        if "sub" in tr:
            hops = tr["sub"][c]
            out["copy_end_by_hops_us"] = {int(h): us(t1[c][hops == h].max())
                                          for h in sorted(set(hops.tolist()))}
    for kind, name in ((3, "fence"), (4, "done_flags"), (5, "final_wait")):
        k = tr["kind"] == kind
        if k.any():
            out[name + "_start_us"] = [us(t0[k].min()), us(t0[k].max())]
            out[name + "_end_us"] = [us(t1[k].min()), us(t1[k].max())]
    return out


def main() -> int:
    import numpy as np
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--k-total", type=int, default=8192)
    ap.add_argument("--calls", type=int, default=200)
    ap.add_argument("--no-multicast", action="store_true")
    ap.add_argument("--allgather", action="store_true")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    gen = torch.Generator().manual_seed(100 + rank)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    if args.allgather:
        m, n, k = args.m, args.n, args.k_total
        prob = mb.Problem(m, n, k, mode=mb.MODE_ALLGATHER, timeout_ns=20_000_000_000)
        plan = mb.plan(prob, world)
        ev_bytes = mb.events_bytes(prob, world)
        team = mb.Team(rank, world, local, (m // world) * k * 2 + ev_bytes + (64 << 20),
                       mb.torch_exchange() if world > 1 else None)
        use_mc = False
        shard = team.tensor((m // world, k), torch.bfloat16)
        shard.copy_((torch.randn(m // world, k, generator=gen) * 0.02).to(torch.bfloat16))
        b = (torch.randn(k, n, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
        events = team.tensor((ev_bytes // 4,), torch.int32)
        gathered = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

        def call(trace=None):
            mb.allgather_gemm(shard, b, gathered, out, events=events, problem=prob, stream=stream,
                              device=local, team=team if world > 1 else None, trace=trace)
    else:
        m, n, k = args.m, args.n, args.k_total // world
        a = (torch.randn(m, k, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
        b = (torch.randn(k, n, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
        prob = mb.Problem(m, n, k, timeout_ns=20_000_000_000)
        plan = mb.plan(prob, world)
        ws_bytes, ev_bytes = mb.workspace_bytes(prob, world), mb.events_bytes(prob, world)
        want_mc = world > 1 and not plan.one_shot and not args.no_multicast
        team = mb.Team(rank, world, local, ws_bytes + ev_bytes + m * n * 2 + (64 << 20),
                       mb.torch_exchange() if world > 1 else None,
                       multicast_bytes=(ws_bytes + m * n * 2 + (1 << 20)) if want_mc else 0)
        use_mc = want_mc and team.multicast
        ws = team.tensor((max(ws_bytes, 16),), torch.uint8, multicast=use_mc)
        events = team.tensor((ev_bytes // 4,), torch.int32)
        out = team.tensor((m, n), torch.bfloat16, multicast=use_mc)

        def call(trace=None):
            mb.gemm_allreduce(a, b, out, workspace=ws, events=events, problem=prob,
                              stream=stream, device=local, team=team if world > 1 else None,
                              trace=trace)

    def timed(trace=None):
        flush.fill_(1)
        team.barrier(stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call(trace)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3

    for _ in range(args.calls):
        call()
    times = [timed() for _ in range(10)]
    # records: GEMM tiles, reduce sub-tasks (16 per tile at most) or copy
    # chunks (up to 128 per tile row and shard), and a few per worker
    trace = torch.zeros((plan.tiles * 64 + plan.m_tiles * 128) * 4, dtype=torch.int64,
                        device=dev)
    traced_us = timed(trace)
    mb.events_status(events, stream)
    rec = trace.view(-1, 4).cpu().numpy().astype(np.uint64)
    rec = rec[rec[:, 3] != 0]
    tr = {"kind": (rec[:, 0] & 0xFF).astype(np.int64), "sub": ((rec[:, 0] >> 8) & 0xFF).astype(
        np.int64), "t0": rec[:, 2], "t1": rec[:, 3]}
    exchange = ("all-gather copies" if args.allgather else "in-switch" if use_mc else
                "peer" if world > 1 else "none")
    info = {"pe": rank, "tp": world, "exchange": exchange,
            "call_us_median": round(float(np.median(times)), 1),
            "traced_call_us": round(traced_us, 1)}
    info.update(_summary(tr, np))
    infos = [info]
    if world > 1:
        infos = [None] * world
        dist.all_gather_object(infos, info)
    if rank == 0:
        for x in infos:
            print(json.dumps(x), flush=True)
    del trace
    if world > 1:
        dist.barrier()
    team.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
