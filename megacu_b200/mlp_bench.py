"""Timing of the tensor-parallel MLP chain (benchmark config 5).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \\
        --master-addr 127.0.0.1 --master-port 29600 -m megacu_b200.mlp_bench

Workload (defaults = config 5): `layers` Llama-style MLP blocks, tokens T,
hidden H, intermediate I split over the PEs (I/tp columns per PE); gate/up
column-parallel, down row-parallel with the allreduce of its output; bf16
random weights N(0, 0.02^2), activations N(0, 1); synthetic data.

Three arms, timed interleaved step by step after a common heat-up (L2 flushed
and the PEs aligned by a team barrier before every step, outside the CUDA
events; each step's time is the max over ranks, and the mean over steps is
reported):
  two_launches   megacu_cuda_mlp_chain_bf16, two launches per block
  single_launch  the same, all blocks in one persistent launch
  unfused        torch: x @ gate, x @ up (cuBLAS), silu(g) * u, act @ down,
                 then NCCL allreduce, per block
Prints one JSON line on rank 0, with the call roofline (the slower of the
GEMMs at the measured bf16 peak and the allreduces' bus bytes over NVLink at
770 GB/s per direction) and each fused arm's largest difference from the
unfused arm's output, relative to that output's largest magnitude.
"""
from __future__ import annotations

import argparse
import json
import os

from .measure import NVLINK_GBS, ClockSampler, interleaved, mean, peaks


def main() -> int:
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=14336, help="total intermediate size")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--heat-calls", type=int, default=200)
    ap.add_argument("--skip-single-launch", action="store_true")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    t, h, layers = args.tokens, args.hidden, args.layers
    if args.inter % world:
        raise SystemExit("inter must split evenly over the PEs")
    i = args.inter // world
    gen = torch.Generator().manual_seed(5000 + rank)
    rnd = lambda shape, std: (torch.randn(*shape, generator=gen) * std).to(torch.bfloat16).to(dev)
    x = rnd((t, h), 1.0)
    wg = [rnd((h, i), 0.02) for _ in range(layers)]
    wu = [rnd((h, i), 0.02) for _ in range(layers)]
    wd = [rnd((i, h), 0.02) for _ in range(layers)]

    arms_modes = [False] + ([] if args.skip_single_launch else [True])
    probs = {s: mb.MlpChainProblem(t, h, i, layers=layers, single_launch=s,
                                   timeout_ns=30_000_000_000) for s in arms_modes}
    sizes = {s: mb.mlp_chain_sizes(probs[s], world) for s in arms_modes}
    need = max(sz["workspace"] + sz["events_down"] + 2 * sz["x_work"] for sz in sizes.values())
    team = mb.Team(rank, world, local, need * len(arms_modes) + (64 << 20),
                   mb.torch_exchange() if world > 1 else None)
    stream = torch.cuda.current_stream()
    bufs = {}
    for s in arms_modes:
        sz = sizes[s]
        bufs[s] = dict(act=torch.empty(sz["act"] // 2, dtype=torch.bfloat16, device=dev),
                       workspace=team.tensor((max(sz["workspace"], 16),), torch.uint8),
                       x_work=team.tensor((t, h), torch.bfloat16),
                       events_swiglu=torch.zeros(sz["events_swiglu"] // 4, dtype=torch.int32,
                                                 device=dev),
                       events_down=team.tensor((sz["events_down"] // 4,), torch.int32))
    outs = {s: team.tensor((t, h), torch.bfloat16) for s in arms_modes}

    def fused(single):
        def body():
            mb.mlp_chain(x, wg, wu, wd, outs[single], problem=probs[single], stream=stream,
                         device=local, team=team if world > 1 else None, **bufs[single])
        return body

    def unfused():
        cur = x
        for l in range(layers):
            act = torch.nn.functional.silu(cur @ wg[l]) * (cur @ wu[l])
            cur = act @ wd[l]
            if world > 1:
                dist.all_reduce(cur)
        return cur

    arms = [fused(s) for s in arms_modes] + [unfused]
    names = ["single_launch" if s else "two_launches" for s in arms_modes] + ["unfused"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def align():
        flush.fill_(1)
        team.barrier(stream)

    with ClockSampler(local) as clocks:
        for _ in range(args.heat_calls):
            for arm in arms:
                arm()
        torch.cuda.synchronize()
        ms = interleaved(arms, args.steps, args.warmup, align, stream, world, device=dev)
    us = [mean(v) * 1e3 for v in ms]
    for s in arms_modes:
        mb.events_status(bufs[s]["events_down"], stream)
        mb.events_status(bufs[s]["events_swiglu"], stream)

    # Work and bytes per PE of one chain call.
    flops = 2.0 * t * h * (2 * i) * layers + 2.0 * t * i * h * layers
    out_bytes = t * h * 2
    link = 2.0 * (world - 1) / world * out_bytes * layers
    peak, peak_src = peaks()
    t_gemm = flops / (peak * 1e12) * 1e6
    t_link = link / (NVLINK_GBS * 1e9) * 1e6
    # Parity of the last fused calls against the unfused chain (collective:
    # every rank runs it).
    ref = unfused().float()
    torch.cuda.synchronize()
    scale = float(ref.abs().max())
    rel_err = {("single_launch" if s else "two_launches"):
               float((outs[s].float() - ref).abs().max()) / max(scale, 1e-30)
               for s in arms_modes}
    if rank == 0:
        line = {"workload": f"C5 {layers} MLP blocks T{t} H{h} I{args.inter}/tp bf16",
                "tp": world, "steps": args.steps, "data": "synthetic",
                "us_per_call": dict(zip(names, us)),
                "tflops_per_gpu": {n: flops / (u * 1e-6) / 1e12 for n, u in zip(names, us)},
                "flops_per_pe": flops, "allreduce_bus_bytes_per_pe": link,
                "roofline_call": {
                    "gemm_us_at_peak": t_gemm, "link_us_at_770GBps": t_link,
                    "roofline_us": max(t_gemm, t_link),
                    "frac": {n: max(t_gemm, t_link) / u for n, u in zip(names, us)},
                    "peak_tflops": peak, "peak_source": peak_src,
                    "note": "slower of the GEMMs at the measured peak and the allreduces' "
                            "bus bytes 2(tp-1)/tp x output per block over NVLink"},
                "max_rel_err_vs_unfused": rel_err,
                "l2": "flushed (256 MiB write) before every timed step",
                "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    team.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
