"""One rank of the multi-process GPU test (run under torchrun, one GPU each).

Every rank builds its team over torch.distributed (gloo carries the 128-byte
CUDA IPC handles), runs the fused bf16 kernel for several modes twice each,
and checks its own output, event tensor and completion counters against the
oracle's n-PE graph (every rank regenerates every rank's seeded inputs).
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
from gpu_util import REL_TOL, errors, f32, inputs, wire_scale  # noqa: E402

CASES = [
    # m, n, k, mode, algo, deterministic, tile_n (0 = auto), in the multicast region
    (512, 1024, 256, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 0, False),
    (64, 2048, 512, mb.MODE_ALLREDUCE, mb.ALGO_ONE_SHOT, False, 0, False),
    (384, 520, 136, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, True, 0, False),
    (1024, 768, 320, mb.MODE_REDUCE_SCATTER, mb.ALGO_AUTO, False, 0, False),
    (1024, 1024, 128, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 128, False),  # CTA pairs
    (1024, 512, 128, mb.MODE_REDUCE_SCATTER, mb.ALGO_AUTO, True, 256, False),  # pairs to 4 PEs
    # in-switch reduction (workspace and out in the multicast region)
    (512, 1024, 256, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 0, True),
    (384, 520, 136, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 0, True),  # ragged m, n
    (768, 1024, 200, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 256, True),  # CTA pairs
    (64, 2048, 512, mb.MODE_ALLREDUCE, mb.ALGO_ONE_SHOT, False, 0, True),  # one-shot (decode)
    (300, 1000, 200, mb.MODE_ALLREDUCE, mb.ALGO_ONE_SHOT, False, 0, True),  # one-shot, ragged
    (1024, 768, 320, mb.MODE_REDUCE_SCATTER, mb.ALGO_AUTO, False, 0, True),
    (1024, 512, 128, mb.MODE_REDUCE_SCATTER, mb.ALGO_AUTO, False, 256, True),  # RS, CTA pairs
]
MULTICAST_BYTES = 1 << 29


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    team = mb.Team(rank, world, local, 1 << 30, mb.torch_exchange(),
                   multicast_bytes=MULTICAST_BYTES)
    stream = torch.cuda.Stream()
    failures = []
    if not team.multicast:
        failures.append(f"no multicast region: {team.multicast_error}")
    for idx, (m, n, k, mode, algo, det, tile_n, mc) in enumerate(CASES):
        if mode == mb.MODE_REDUCE_SCATTER and m % (world * 128):
            continue
        if mc and not team.multicast:
            continue
        prob = mb.Problem(m, n, k, mode=mode, algo=algo, deterministic=det, tile_n=tile_n,
                          timeout_ns=10_000_000_000)
        pl = mb.plan(prob, world)
        rows = m // world if mode == mb.MODE_REDUCE_SCATTER else m
        ws = team.tensor((max(mb.workspace_bytes(prob, world), 16),), torch.uint8, multicast=mc)
        ev = team.tensor((mb.events_bytes(prob, world) // 4,), torch.int32)
        out = team.tensor((rows, n), torch.bfloat16, multicast=mc)
        a, b = inputs(100 + idx, world, m, n, k)
        ad, bd = a[rank].cuda(), b[rank].cuda()
        ev0 = [np.zeros(oracle_lib.event_tensor_words(world, pl.tiles), np.uint32)
               for _ in range(world)]
        for _ in range(2):
            mb.gemm_allreduce(ad, bd, out, workspace=ws, events=ev, problem=prob, stream=stream,
                              device=local, team=team)
        mb.events_status(ev, stream)
        ref = oracle_lib.bf16_call([f32(x) for x in a], [f32(x) for x in b], m=m, n=n, k=k,
                                   tile_n=pl.tile_n, mode=mode, one_shot=pl.one_shot,
                                   wire_bytes=pl.wire_bytes, epoch=1, events=ev0)
        ref2 = oracle_lib.bf16_call([f32(x) for x in a], [f32(x) for x in b], m=m, n=n, k=k,
                                    tile_n=pl.tile_n, mode=mode, one_shot=pl.one_shot,
                                    wire_bytes=pl.wire_bytes, epoch=2, events=ref["events"])
        rows = (slice(rank * (m // world), (rank + 1) * (m // world))
                if mode == mb.MODE_REDUCE_SCATTER else None)
        scale = None if det else wire_scale(a, b, rows)
        err, strict, line = errors(f32(out), ref["out"][rank], scale)
        print(f"rank {rank}: case {idx}: {line}", flush=True)
        if not err < REL_TOL or (det and not strict < REL_TOL):
            failures.append(f"case {idx}: {line}")
        words = ev[64:].cpu().numpy().view(np.uint32)
        if not np.array_equal(words, ref2["events"][rank]):
            failures.append(f"case {idx}: event tensor differs")
        counters = mb.events_counters(ev, stream)
        if counters != (2 * ref["counters"][rank]).tolist():
            failures.append(f"case {idx}: counters {counters} != {2 * ref['counters'][rank]}")
        dist.barrier()
    if team.multicast:
        # A workspace in the multicast region of a call that cannot reduce in
        # the switch (fp32 partials on the wire) is refused before any launch.
        prob = mb.Problem(64, 2048, 64, algo=mb.ALGO_ONE_SHOT, deterministic=True)
        ws = team.tensor((mb.workspace_bytes(prob, world),), torch.uint8, multicast=True)
        ev = team.tensor((mb.events_bytes(prob, world) // 4,), torch.int32)
        out = team.tensor((64, 2048), torch.bfloat16, multicast=True)
        a = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
        b = torch.zeros(64, 2048, dtype=torch.bfloat16, device="cuda")
        try:
            mb.gemm_allreduce(a, b, out, workspace=ws, events=ev, problem=prob, stream=stream,
                              device=local, team=team)
            failures.append("fp32-wire call with multicast buffers was not refused")
        except mb.MegacuError as err:
            if err.detail != 28:
                failures.append(f"fp32-wire call with multicast buffers: {err}")
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
