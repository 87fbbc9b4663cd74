"""All-gather + GEMM, host side (no GPU): the plan the C ABI makes against the
oracle's restatement of the schedule, buffer sizes, argument validation
(null stream = validate only), and the oracle's own graph against a float64
restatement."""
from __future__ import annotations

import numpy as np
import pytest

import megacu_b200 as mb
from megacu_b200 import _capi

import oracle_lib

FAKE = 0x100000  # never dereferenced: validation-only calls


def _ag(m, n, k, **kw):
    return mb.Problem(m, n, k, mode=mb.MODE_ALLGATHER, **kw)


@pytest.mark.parametrize("m,n,k,n_pes,tile_n", [
    (256, 512, 128, 1, 0), (1024, 768, 256, 2, 128), (2048, 1024, 64, 4, 256),
    (1024, 3584, 8192, 8, 0), (4096, 448, 200, 8, 64)])
def test_raster_matches_oracle_on_every_pe(m, n, k, n_pes, tile_n):
    prob = _ag(m, n, k, tile_n=tile_n)
    pl = mb.plan(prob, n_pes)
    mq = pl.m_tiles // n_pes
    for pe in range(n_pes):
        seen = []
        for r in range(pl.tiles):
            got = mb.plan_tile(prob, n_pes, r, pe)
            assert got == oracle_lib.locate_gather(pl.m_tiles, pl.n_tiles, n_pes, pe,
                                                   pl.group_m, r)
            row, col, shard, local = got
            # whole shards, this PE's own first, then 1, 2, ... hops away
            assert shard == (pe + r // (mq * pl.n_tiles)) % n_pes
            assert shard * mq <= row < (shard + 1) * mq
            seen.append(row * pl.n_tiles + col)
        assert sorted(seen) == list(range(pl.tiles))


def test_pairs_are_neighbours_in_one_shard():
    prob = _ag(2048, 1024, 128, tile_n=256)
    n_pes = 4
    pl = mb.plan(prob, n_pes)
    assert pl.cta_pairs and pl.gemm_units == pl.tiles // 2
    for q in range(pl.gemm_units):
        r0, r1 = mb.plan_pair(prob, n_pes, q)
        assert (r0, r1) == oracle_lib.pair_raster(n_pes, 0, q)
        for pe in range(n_pes):
            t0, t1 = mb.plan_tile(prob, n_pes, r0, pe), mb.plan_tile(prob, n_pes, r1, pe)
            assert t0[0] % 2 == 0 and t1[0] == t0[0] + 1 and t0[1] == t1[1] and t0[2] == t1[2]
    # one tile row per shard: no pairs
    assert not mb.plan(_ag(512, 1024, 128, tile_n=256), 4).cta_pairs


@pytest.mark.parametrize("m,n,k,n_pes", [(256, 512, 128, 1), (1024, 768, 8192, 2),
                                         (8192, 3584, 8192, 8)])
def test_sizes(m, n, k, n_pes):
    prob = _ag(m, n, k, deterministic=True)
    pl = mb.plan(prob, n_pes)
    assert mb.workspace_bytes(prob, n_pes) == 0
    assert pl.slots_per_src == 0 and not pl.one_shot and pl.wire_bytes == 2
    words = oracle_lib.gather_events_words(n_pes, pl.tiles, pl.m_tiles // n_pes)
    assert mb.events_bytes(prob, n_pes) == 256 + 4 * words
    rows = oracle_lib.gather_chunk_rows(k)
    assert 128 % rows == 0 and (rows == 1 or rows * k * 2 <= 65536)


def _driver(n_pes=1):
    d = mb.driver_view(None, 0)
    d.team.team_n_pes, d.team.world_n_pes = n_pes, n_pes
    return d


def _call(d, prob, a=FAKE, b=FAKE, g=FAKE, out=FAKE, ev=FAKE):
    s = _capi.load().megacu_cuda_allgather_gemm_bf16(d, a, b, g, out, ev, prob.to_c())
    return s.code, s.detail


def test_validation_only():
    good = _ag(1024, 512, 128)
    assert _call(_driver(), good) == (0, 0)
    # the mode is set by the entry point
    assert _call(_driver(), mb.Problem(1024, 512, 128)) == (0, 0)
    assert _call(_driver(2), _ag(1024 + 128, 512, 128)) == (2, 26)   # m not a multiple of tp*128
    assert _call(_driver(), _ag(1000, 512, 128)) == (2, 26)
    assert _call(_driver(), _ag(1024, 510, 128)) == (1, 21)
    assert _call(_driver(), _ag(1024, 512, 128, tile_n=96)) == (2, 22)
    assert _call(_driver(), good, a=None) == (1, 2)
    assert _call(_driver(), good, g=None) == (1, 2)
    assert _call(_driver(), good, ev=None) == (1, 2)
    assert _call(_driver(), good, g=FAKE + 8) == (1, 21)
    assert _call(_driver(2), good) == (2, 13)                         # no team handle
    assert _call(_driver(), _ag(1024, 512, 128, cta_pairs=mb.CTA_PAIRS_ON, tile_n=64)) == (2, 27)
    # the allreduce entries refuse the all-gather mode
    s = _capi.load().megacu_cuda_gemm_allreduce_bf16_orchestrate(
        _driver(), FAKE, FAKE, FAKE, FAKE, FAKE, _ag(1024, 512, 128).to_c())
    assert (s.code, s.detail) == (1, 1)


@pytest.mark.parametrize("n_pes", [1, 2, 4])
def test_oracle_graph(n_pes):
    rng = np.random.default_rng(7 + n_pes)
    m, n, k, tile_n = 256 * n_pes, 192, 96, 64
    shards = [oracle_lib.round_bf16(rng.standard_normal((m // n_pes, k)).astype(np.float32))
              for _ in range(n_pes)]
    bs = [oracle_lib.round_bf16(0.1 * rng.standard_normal((k, n)).astype(np.float32))
          for _ in range(n_pes)]
    tiles = (m // 128) * (n // tile_n)
    mq = (m // 128) // n_pes
    words = oracle_lib.gather_events_words(n_pes, tiles, mq)
    ev = [np.full(words, 0xdead, np.uint32) for _ in range(n_pes)]
    epoch = 3
    res = oracle_lib.allgather_gemm(shards, bs, m=m, n=n, k=k, tile_n=tile_n, epoch=epoch,
                                    events=ev)
    full = np.concatenate(shards).astype(np.float64)
    chunks = n_pes * mq * (128 // oracle_lib.gather_chunk_rows(k))
    base = 2 * tiles * 4
    for pe in range(n_pes):
        assert np.array_equal(res["gathered"][pe], np.concatenate(shards))
        want = full @ bs[pe].astype(np.float64)
        assert np.max(np.abs(res["out"][pe] - want)) < 1e-4 * (1 + np.max(np.abs(want)))
        assert sorted(res["gemm_order"][pe].tolist()) == list(range(tiles))
        e = res["events"][pe]
        assert (e[(epoch & 1) * tiles * 4:((epoch & 1) + 1) * tiles * 4] == epoch).all()
        peers = [q for q in range(n_pes) if q != pe]
        assert all(e[base + q] == epoch for q in peers)             # ready[q]
        assert all(e[base + n_pes + q] == epoch for q in peers)     # read_done[q]
        assert (e[base + 2 * n_pes:] == 0).all()                    # counters zeroed
        c = res["counters"][pe].tolist()
        assert c == [tiles, chunks, tiles * 4, tiles * (n_pes - 1) // n_pes, n_pes - 1,
                     n_pes - 1, 1, 0]
