"""All-gather + GEMM through the C ABI against the oracle's graph: the gathered
A bit for bit, the output within the bf16 tolerance, the event tensor words
and the completion counters exactly, over two consecutive calls (epochs 1
and 2). One PE on cuda:0; two PEs on two GPUs driven by one process.

Every case has passed on B200s with the bounds-checked and the regular
library. The host side (plan, sizes, validation) and the oracle are covered
without a GPU in test_allgather.py.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

import megacu_b200 as mb
import oracle_lib
from conftest import gpu_count
from gpu_util import assert_close, f32, same_process_team, seeded_bf16

pytestmark = pytest.mark.gpu


def _inputs(seed, n_pes, m, n, k):
    shards = [seeded_bf16(seed * 100 + 10 * pe, (m // n_pes, k), 1.0) for pe in range(n_pes)]
    bs = [seeded_bf16(seed * 100 + 10 * pe + 1, (k, n), 0.02) for pe in range(n_pes)]
    return shards, bs


def _check(prob, shards, bs, gathered, outs, events):
    """Two calls were made; compares every PE's buffers with the oracle."""
    n_pes = len(shards)
    m, n, k = prob.m, prob.n, prob.k
    pl = mb.plan(prob, n_pes)
    words = oracle_lib.gather_events_words(n_pes, pl.tiles, pl.m_tiles // n_pes)
    ev0 = [np.zeros(words, np.uint32) for _ in range(n_pes)]
    s32, b32 = [f32(x) for x in shards], [f32(x) for x in bs]
    ref1 = oracle_lib.allgather_gemm(s32, b32, m=m, n=n, k=k, tile_n=pl.tile_n,
                                     group_m=pl.group_m, epoch=1, events=ev0)
    ref2 = oracle_lib.allgather_gemm(s32, b32, m=m, n=n, k=k, tile_n=pl.tile_n,
                                     group_m=pl.group_m, epoch=2, events=ref1["events"])
    for pe in range(n_pes):
        assert np.array_equal(f32(gathered[pe]), np.concatenate(s32)), f"PE {pe}: gathered A"
        assert_close(f32(outs[pe]), ref2["out"][pe], what=f"PE {pe}:")
        got = events[pe][64:].cpu().numpy().view(np.uint32)
        assert np.array_equal(got, ref2["events"][pe]), f"PE {pe}: event tensor"
        counters = mb.events_counters(events[pe])
        want = (ref1["counters"][pe] + ref2["counters"][pe]).tolist()
        assert counters == want, f"PE {pe}: counters {counters} != {want}"


@pytest.mark.parametrize("m,n,k,tile_n,pairs", [
    (512, 384, 192, 0, mb.CTA_PAIRS_AUTO),
    (512, 512, 256, 256, mb.CTA_PAIRS_ON),
    (384, 448, 200, 64, mb.CTA_PAIRS_OFF),
    (256, 1024, 8192, 128, mb.CTA_PAIRS_OFF),   # 4-row copy chunks
])
def test_allgather_one_pe(m, n, k, tile_n, pairs):
    prob = mb.Problem(m, n, k, mode=mb.MODE_ALLGATHER, tile_n=tile_n, cta_pairs=pairs,
                      timeout_ns=10_000_000_000)
    shards, bs = _inputs(31, 1, m, n, k)
    dev = torch.device("cuda", 0)
    a, b = shards[0].to(dev), bs[0].to(dev)
    gathered = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    events = torch.zeros(mb.events_bytes(prob, 1) // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(2):
        mb.allgather_gemm(a, b, gathered, out, events=events, problem=prob, stream=stream)
    mb.events_status(events, stream)
    _check(prob, shards, bs, [gathered], [out], [events])


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m,n,k,tile_n", [(1024, 384, 192, 0), (1024, 512, 4096, 256)])
def test_allgather_two_pes(m, n, k, tile_n):
    teams = same_process_team([0, 1])
    try:
        prob = mb.Problem(m, n, k, mode=mb.MODE_ALLGATHER, tile_n=tile_n,
                          timeout_ns=10_000_000_000)
        shards, bs = _inputs(32, 2, m, n, k)
        ev_words = mb.events_bytes(prob, 2) // 4
        a = [t.tensor((m // 2, k), torch.bfloat16) for t in teams]
        events = [t.tensor((ev_words,), torch.int32) for t in teams]
        gathered, outs, bd, streams = [], [], [], []
        for pe, t in enumerate(teams):
            dev = torch.device("cuda", t.device)
            a[pe].copy_(shards[pe])
            bd.append(bs[pe].to(dev))
            gathered.append(torch.empty((m, k), dtype=torch.bfloat16, device=dev))
            outs.append(torch.empty((m, n), dtype=torch.bfloat16, device=dev))
            streams.append(torch.cuda.Stream(device=dev))
        for pe in range(2):
            torch.cuda.synchronize(pe)
        for _ in range(2):
            for pe, t in enumerate(teams):
                with torch.cuda.device(t.device):
                    mb.allgather_gemm(a[pe], bd[pe], gathered[pe], outs[pe], events=events[pe],
                                      problem=prob, stream=streams[pe], device=t.device, team=t)
        for pe in range(2):
            mb.events_status(events[pe], streams[pe])
        _check(prob, shards, bs, gathered, outs, events)
    finally:
        for pe in range(2):
            torch.cuda.synchronize(pe)
        for t in teams:
            t.close()
