"""Multi-PE paths through the C ABI.

* One process driving two GPUs (a team with direct peer access): two-shot and
  one-shot allreduce, reduce-scatter, the fp32-wire deterministic mode and
  megacu's fp32 launcher, each against the oracle's n-PE graph (outputs,
  event tensors, completion counts). Skipped with fewer than two GPUs.
* Failure detection on one GPU: a two-PE team whose second PE never
  launches. The first PE's cross-GPU waits run out (nothing sets the flags),
  the kernel returns, and the host reads backend_error / detail 40.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import megacu_b200 as mb
import oracle_lib
from conftest import gpu_count
from gpu_util import assert_close, f32, inputs, same_process_team, wire_scale

pytestmark = pytest.mark.gpu


class TeamCall:
    def __init__(self, teams, problem: mb.Problem):
        self.teams, self.problem = teams, problem
        n = len(teams)
        self.plan = mb.plan(problem, n)
        ws = mb.workspace_bytes(problem, n)
        ev = mb.events_bytes(problem, n)
        rows = problem.m // n if problem.mode == mb.MODE_REDUCE_SCATTER else problem.m
        self.ws = [t.tensor((max(ws, 16),), torch.uint8) for t in teams]
        self.events = [t.tensor((ev // 4,), torch.int32) for t in teams]
        self.out = [t.tensor((rows, problem.n), torch.bfloat16) for t in teams]
        self.streams = [torch.cuda.Stream(device=t.device) for t in teams]

    def event_words(self):
        return [e[64:].cpu().numpy().view(np.uint32).copy() for e in self.events]

    def launch(self, a, b, pes=None):
        for pe, t in enumerate(self.teams):
            if pes is not None and pe not in pes:
                continue
            with torch.cuda.device(t.device):
                mb.gemm_allreduce(a[pe], b[pe], self.out[pe], workspace=self.ws[pe],
                                  events=self.events[pe], problem=self.problem,
                                  stream=self.streams[pe], device=t.device, team=t)

    def finish(self, pes=None):
        for pe, t in enumerate(self.teams):
            if pes is None or pe in pes:
                mb.events_status(self.events[pe], self.streams[pe])


need2 = pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")


@need2
@pytest.mark.parametrize("m,n,k,mode,algo,det,tile_n", [
    (512, 1024, 256, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 0),
    (64, 2048, 512, mb.MODE_ALLREDUCE, mb.ALGO_ONE_SHOT, False, 0),
    (300, 520, 200, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, True, 0),
    (1024, 768, 320, mb.MODE_REDUCE_SCATTER, mb.ALGO_AUTO, False, 0),
    (2048, 4096, 1024, mb.MODE_ALLREDUCE, mb.ALGO_AUTO, False, 0),        # CTA pairs
    (1024, 640, 320, mb.MODE_REDUCE_SCATTER, mb.ALGO_AUTO, True, 128),   # CTA pairs, ragged n
    (768, 1024, 200, mb.MODE_ALLREDUCE, mb.ALGO_TWO_SHOT, False, 256),   # CTA pairs, two-shot
])
def test_two_gpu_matches_oracle(m, n, k, mode, algo, det, tile_n):
    teams = same_process_team([0, 1])
    prob = mb.Problem(m, n, k, mode=mode, algo=algo, deterministic=det, tile_n=tile_n,
                      timeout_ns=5_000_000_000)
    call = TeamCall(teams, prob)
    a, b = inputs(7, 2, m, n, k)
    ad = [a[pe].to(f"cuda:{pe}") for pe in range(2)]
    bd = [b[pe].to(f"cuda:{pe}") for pe in range(2)]
    ev0 = call.event_words()
    for _ in range(2):  # two calls: both parity planes, no reset in between
        call.launch(ad, bd)
        call.finish()
    ref = oracle_lib.bf16_call([f32(x) for x in a], [f32(x) for x in b], m=m, n=n, k=k,
                               tile_n=call.plan.tile_n, mode=mode, one_shot=call.plan.one_shot,
                               wire_bytes=call.plan.wire_bytes, epoch=1, events=ev0)
    ref2 = oracle_lib.bf16_call([f32(x) for x in a], [f32(x) for x in b], m=m, n=n, k=k,
                                tile_n=call.plan.tile_n, mode=mode, one_shot=call.plan.one_shot,
                                wire_bytes=call.plan.wire_bytes, epoch=2, events=ref["events"])
    for pe in range(2):
        rows = slice(pe * (m // 2), (pe + 1) * (m // 2)) if mode == mb.MODE_REDUCE_SCATTER else None
        scale = None if det else wire_scale(a, b, rows)
        # the deterministic mode (fp32 partials) meets the strict measure too
        assert_close(f32(call.out[pe]), ref["out"][pe], scale, strict=det, what=f"PE {pe}:")
        assert np.array_equal(call.event_words()[pe], ref2["events"][pe])
        counters = mb.events_counters(call.events[pe])
        assert counters == (2 * ref["counters"][pe]).tolist()
    if mode == mb.MODE_ALLREDUCE:  # every PE holds the same bits
        assert torch.equal(call.out[0].cpu(), call.out[1].cpu())
    for t in teams:
        t.close()


@need2
def test_two_gpu_f32_kat_twelve():
    """nvshmem_two_rank_smoke.cc: A = pe + 1, B = 1, K = 4 -> 12, on two GPUs."""
    teams = same_process_team([0, 1])
    m, n, k = 2, 3, 4
    bufs = []
    for pe, t in enumerate(teams):
        with torch.cuda.device(t.device):
            a = torch.full((m, k), float(pe + 1), device=f"cuda:{pe}")
            b = torch.ones(k, n, device=f"cuda:{pe}")
            partial = t.tensor((2 * m * n,), torch.float32)
            events = t.tensor((32,), torch.int32)
            out = torch.zeros(m, n, device=f"cuda:{pe}")
            bufs.append((a, b, partial, out, events, torch.cuda.Stream(device=t.device)))
    for pe, t in enumerate(teams):
        a, b, partial, out, events, s = bufs[pe]
        d = mb.driver_view(s, t.device, t)
        with torch.cuda.device(t.device):
            mb.check(mb.cuda_nvshmem_gemm_allreduce_phased_orchestrate(
                d, a, b, partial, out, events, m, n, k, m, n))
    for pe in range(2):
        bufs[pe][5].synchronize()
        assert torch.all((bufs[pe][3].cpu() - 12.0).abs() < 1e-4)
    for t in teams:
        t.close()


@pytest.mark.skipif(gpu_count() < 1, reason="needs a CUDA GPU")
def test_missing_peer_times_out_with_status():
    """A flag nothing sets: the bounded wait ends the kernel with an error."""
    teams = same_process_team([0, 0])  # PE 1 never launches
    m, n, k = 256, 512, 128
    prob = mb.Problem(m, n, k, algo=mb.ALGO_TWO_SHOT, timeout_ns=200_000_000)
    call = TeamCall(teams, prob)
    a, b = inputs(9, 2, m, n, k)
    call.launch([x.cuda() for x in a], [x.cuda() for x in b], pes={0})
    with pytest.raises(mb.MegacuError) as err:
        call.finish(pes={0})
    assert err.value.code == 3 and err.value.detail == 40
    # the context still works afterwards
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0
    for t in teams:
        t.close()
