"""The fused call captured in a CUDA graph and replayed: the event tensor's
epoch comes from the launch counter in `events` (no per-call memset, no host
barrier), so each replay is a complete call. One PE on cuda:0; the output of
every replay must equal the directly launched call's bit for bit, and the
completion counters must count every replay.
"""
from __future__ import annotations

import pytest
import torch

import megacu_b200 as mb
from gpu_util import inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k,pairs", [(512, 1024, 256, mb.CTA_PAIRS_AUTO),
                                         (128, 4096, 512, mb.CTA_PAIRS_OFF)])
def test_fused_call_replays_from_a_cuda_graph(m, n, k, pairs):
    dev = torch.device("cuda", 0)
    a_h, b_h = inputs(61, 1, m, n, k)
    a, b = a_h[0].to(dev), b_h[0].to(dev)
    prob = mb.Problem(m, n, k, cta_pairs=pairs, timeout_ns=5_000_000_000)
    events = torch.zeros(mb.events_bytes(prob, 1) // 4, dtype=torch.int32, device=dev)
    direct = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream()
    # A direct call first: the reference result, and the one-time launch set-up
    # (function attributes) happens outside the capture.
    mb.gemm_allreduce(a, b, direct, workspace=None, events=events, problem=prob, stream=stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        mb.gemm_allreduce(a, b, out, workspace=None, events=events, problem=prob,
                          stream=torch.cuda.current_stream())
    for replay in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, direct), f"replay {replay}"
    mb.events_status(events)
    counters = mb.events_counters(events)
    assert counters[6] == 1 + 3                    # launches: the direct call + 3 replays
    assert counters[0] == 4 * mb.plan(prob, 1).tiles
