"""One rank of the full-size multi-GPU parity test (torchrun, one GPU each).

BASELINE's configs 2 and 3 at their full sizes, K split over the ranks:
  C2  allreduce       M 4096, N 8192, K 8192 / tp
  C3  reduce-scatter  M 8192, N 8192, K 28672 / tp
Each case runs the fused kernel twice (the second call uses the other parity
plane of the event tensor) and checks properties that do not need the CPU
oracle's GEMM at this size:
  * the output against torch's fp32 GEMM of the same bf16 inputs, summed over
    ranks by NCCL in fp32, within the bf16-wire tolerance (max |err| over the
    per-element sum of the partials' magnitudes plus the reference's RMS,
    below 1e-2);
  * allreduce: every rank's output is bit-identical to rank 0's (every PE
    reduces each element in PE order, or receives the owner's final tile);
  * the event tensor and the completion counters equal the oracle's graph for
    the same m, n, tiles and PEs (they do not depend on k or the data, so the
    oracle runs with k = 8 on rank 0).
Exit code 0 = all checks passed on this rank.
"""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import megacu_b200 as mb  # noqa: E402
import oracle_lib  # noqa: E402
from gpu_util import REL_TOL  # noqa: E402

CASES = [
    ("C2", 4096, 8192, 8192, mb.MODE_ALLREDUCE),
    ("C3", 8192, 8192, 28672, mb.MODE_REDUCE_SCATTER),
]


def seeded_on(dev, seed, shape, std):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std).to(
        torch.bfloat16)


def oracle_graph(world, m, n, pl, mode):
    """Event words and counters of two calls (epochs 1, 2) of every PE."""
    k = 8
    a = [np.zeros((m, k), np.float32) for _ in range(world)]
    b = [np.zeros((k, n), np.float32) for _ in range(world)]
    ev0 = [np.zeros(oracle_lib.event_tensor_words(world, pl.tiles), np.uint32)
           for _ in range(world)]
    kw = dict(m=m, n=n, k=k, tile_n=pl.tile_n, mode=mode, one_shot=pl.one_shot,
              wire_bytes=pl.wire_bytes)
    ref = oracle_lib.bf16_call(a, b, epoch=1, events=ev0, **kw)
    ref2 = oracle_lib.bf16_call(a, b, epoch=2, events=ref["events"], **kw)
    return ([e.copy() for e in ref2["events"]], [(2 * c).tolist() for c in ref["counters"]])


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    nccl = dist.new_group(backend="nccl")
    need = 0
    for _, m, n, k_total, mode in CASES:
        prob = mb.Problem(m, n, k_total // world, mode=mode)
        rows = m // world if mode == mb.MODE_REDUCE_SCATTER else m
        # the team heap is not reused between cases: room for every case
        need += (mb.workspace_bytes(prob, world) + mb.events_bytes(prob, world)
                 + rows * n * 2 + (1 << 20))
    team = mb.Team(rank, world, local, need + (64 << 20), mb.torch_exchange())
    stream = torch.cuda.Stream()
    failures = []
    for idx, (name, m, n, k_total, mode) in enumerate(CASES):
        if mode == mb.MODE_REDUCE_SCATTER and m % (world * 128):
            continue
        k = k_total // world
        prob = mb.Problem(m, n, k, mode=mode, timeout_ns=10_000_000_000)
        pl = mb.plan(prob, world)
        rows = m // world if mode == mb.MODE_REDUCE_SCATTER else m
        ws = team.tensor((max(mb.workspace_bytes(prob, world), 16),), torch.uint8)
        ev = team.tensor((mb.events_bytes(prob, world) // 4,), torch.int32)
        out = team.tensor((rows, n), torch.bfloat16)
        a = seeded_on(dev, 3000 + 100 * idx + 10 * rank, (m, k), 1.0)
        b = seeded_on(dev, 3001 + 100 * idx + 10 * rank, (k, n), 0.02)
        torch.cuda.synchronize()
        for _ in range(2):
            mb.gemm_allreduce(a, b, out, workspace=ws, events=ev, problem=prob, stream=stream,
                              device=local, team=team)
        mb.events_status(ev, stream)
        torch.cuda.synchronize()

        # fp32 reference and the per-element condition of the sum
        part = torch.matmul(a.float(), b.float())
        scale = part.abs()
        dist.all_reduce(part, group=nccl)
        dist.all_reduce(scale, group=nccl)
        if mode == mb.MODE_REDUCE_SCATTER:
            part = part[rank * rows:(rank + 1) * rows]
            scale = scale[rank * rows:(rank + 1) * rows]
        rms = part.double().pow(2).mean().sqrt().item()
        err = ((out.float() - part).abs() / (scale + rms + 1e-30)).max().item()
        if not err < REL_TOL:
            failures.append(f"{name}: rel error {err}")
        del scale

        if mode == mb.MODE_ALLREDUCE:
            first = out.clone()
            dist.broadcast(first, src=0, group=nccl)
            torch.cuda.synchronize()
            if not torch.equal(first, out):
                failures.append(f"{name}: output differs from rank 0's")
            del first
        del part

        graph = [None]
        if rank == 0:
            graph = [oracle_graph(world, m, n, pl, mode)]
        dist.broadcast_object_list(graph, src=0)
        want_events, want_counters = graph[0]
        words = ev[64:].cpu().numpy().view(np.uint32)
        if not np.array_equal(words, want_events[rank]):
            failures.append(f"{name}: event tensor differs from the oracle's graph")
        counters = mb.events_counters(ev, stream)
        if counters != want_counters[rank]:
            failures.append(f"{name}: counters {counters} != {want_counters[rank]}")
        print(f"rank {rank}: {name} tp={world} rel error {err:.3e}", flush=True)
        del ws, ev, out, a, b
        dist.barrier()
    torch.cuda.synchronize()
    dist.barrier()
    team.close()
    dist.destroy_process_group()
    for f in failures:
        print(f"rank {rank}: {f}", flush=True)
    print(f"rank {rank}: {'ok' if not failures else 'FAILED'}", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
