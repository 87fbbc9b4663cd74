"""The CPU oracle against the reference's golden vectors and its own invariants.

Pins: the reference's known-answer tests (tests/golden/kat_gemm_allreduce.json,
transcribed from its test sources by tests/golden/make_golden.py) and benchmark
config 1 (512^3 fp32, 128x128 tiles = 16 tile tasks, 2 logical ranks).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle_lib

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kat_gemm_allreduce.json")


@pytest.fixture(scope="module")
def kat():
    with open(GOLDEN) as f:
        return json.load(f)


def test_kat_single_pe(kat):
    """cuda_gemm_allreduce_correctness.cc: 2x4 @ 4x3, tile 1x2, tol 1e-4."""
    k = kat["single_pe"]
    a = np.array(k["a"], np.float32).reshape(k["m"], k["k"])
    b = np.array(k["b"], np.float32).reshape(k["k"], k["n"])
    outs, events = oracle_lib.phased_f32([a], [b], k["m"], k["n"], k["k"], k["tile_m"],
                                         k["tile_n"])
    want = np.array(k["expected"], np.float32).reshape(k["m"], k["n"])
    assert np.max(np.abs(outs[0] - want)) < k["tolerance"]
    tiles = events[0].shape[1]
    assert events[0].tolist() == [[t + 1 for t in range(tiles)]]


def test_kat_two_pe(kat):
    """nvshmem_two_rank_smoke.cc: A = pe + 1, B = 1, K = 4 -> 12 everywhere."""
    k = kat["two_pe"]
    a = [np.full((k["m"], k["k"]), v, np.float32) for v in k["a_value_per_pe"]]
    b = [np.full((k["k"], k["n"]), k["b_value"], np.float32) for _ in a]
    outs, events = oracle_lib.phased_f32(a, b, k["m"], k["n"], k["k"], k["tile_m"], k["tile_n"])
    for pe, out in enumerate(outs):
        assert np.all(np.abs(out - k["expected_value"]) < k["tolerance"]), pe
        assert np.all(events[pe] == 1)  # one tile, ready value tile + 1


def test_config1_host_plumbing():
    """benchmark config 1: 512^3 fp32, N(0,1) seed 0, 16 tile tasks, 2 ranks x K/2."""
    rng = np.random.default_rng(0)
    m = n = k = 512
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    halves_a = [np.ascontiguousarray(a[:, :256]), np.ascontiguousarray(a[:, 256:])]
    halves_b = [np.ascontiguousarray(b[:256]), np.ascontiguousarray(b[256:])]
    outs, events = oracle_lib.phased_f32(halves_a, halves_b, m, n, k // 2, 128, 128)
    want = a.astype(np.float64) @ b.astype(np.float64)
    for out in outs:
        rel = np.max(np.abs(out - want)) / np.max(np.abs(want))
        assert rel < 1e-5
    assert outs[0].tobytes() == outs[1].tobytes()  # same PE-order sum on every rank
    for ev in events:
        assert ev.shape == (2, 16)
        assert np.all(ev == np.arange(1, 17)[None, :])


def test_gemm_matches_float64():
    rng = np.random.default_rng(7)
    a = rng.standard_normal((67, 45), dtype=np.float32)
    b = rng.standard_normal((45, 33), dtype=np.float32)
    c = oracle_lib.gemm_f32(a, b, threads=3)
    assert np.allclose(c, a.astype(np.float64) @ b, rtol=1e-5, atol=1e-4)
    # thread count does not change a single bit (k order is per element)
    assert oracle_lib.gemm_f32(a, b, threads=1).tobytes() == c.tobytes()


def test_round_bf16_matches_c():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, np.inf, -np.inf],
                                 np.float32)])
    lib = oracle_lib.load()
    want = np.array([lib.oracle_round_bf16(float(v)) for v in x], np.float32)
    got = oracle_lib.round_bf16(x)
    assert got.tobytes() == want.tobytes()
    assert oracle_lib.round_bf16(np.array([1.0 + 2 ** -8], np.float32))[0] == 1.0  # tie to even


def _bf16_inputs(rng, n_pes, m, n, k):
    a = [oracle_lib.round_bf16(rng.normal(0, 1, (m, k)).astype(np.float32)) for _ in range(n_pes)]
    b = [oracle_lib.round_bf16(rng.normal(0, 0.5, (k, n)).astype(np.float32)) for _ in range(n_pes)]
    return a, b


@pytest.mark.parametrize("n_pes,mode,one_shot,m,n,tile_n", [
    (1, 0, False, 200, 136, 64),
    (2, 0, False, 300, 520, 128),
    (2, 0, True, 96, 256, 64),
    (4, 0, False, 512, 384, 128),
    (4, 1, False, 1024, 200, 64),
    (3, 0, True, 130, 64, 64),
])
def test_bf16_graph_counts_and_events(n_pes, mode, one_shot, m, n, tile_n):
    """The task graph's output, completion counts and event tensor are consistent."""
    rng = np.random.default_rng(11)
    k = 40
    a, b = _bf16_inputs(rng, n_pes, m, n, k)
    m_tiles, n_tiles = -(-m // 128), -(-n // tile_n)
    tiles = m_tiles * n_tiles
    events = [np.zeros(oracle_lib.event_tensor_words(n_pes, tiles), np.uint32)
              for _ in range(n_pes)]
    r = oracle_lib.bf16_call(a, b, m=m, n=n, k=k, tile_n=tile_n, mode=mode, one_shot=one_shot,
                             wire_bytes=4, epoch=5, events=events)
    full = sum(x.astype(np.float64) @ y for x, y in zip(a, b))
    for pe in range(n_pes):
        want = full[pe * (m // n_pes):(pe + 1) * (m // n_pes)] if mode == 1 else full
        assert np.allclose(r["out"][pe], want, rtol=1e-4, atol=1e-3)
    # every raster index maps to a distinct tile
    assert sorted(r["gemm_order"].tolist()) == list(range(tiles))
    active = sum(1 for t in range(tiles) for q in range(4) if (t // n_tiles) * 128 + q * 32 < m)
    blocks = [(t, q, cb) for t in range(tiles) for q in range(4) for cb in range(tile_n // 64)
              if (t // n_tiles) * 128 + q * 32 < m and (t % n_tiles) * tile_n + cb * 64 < n]
    c = r["counters"]
    assert np.all(c[:, 0] == tiles) and np.all(c[:, 6] == 1) and np.all(c[:, 7] == 0)
    reduced = [sum(1 for t in ro if t >= 0) for ro in r["reduce_order"]]
    reduced_tiles = [sorted(set(int(t) for t in ro if t >= 0)) for ro in r["reduce_order"]]
    if n_pes == 1:
        assert c[0, 2] == active and c[0, 1] == 0
    elif one_shot:
        assert all(x == len(blocks) for x in reduced)
        assert np.all(c[:, 2] == active * n_pes)
    else:
        assert sum(reduced) == len(blocks)  # every existing block reduced exactly once
        assert np.all(c[:, 2] == active)
    assert c[:, 1].tolist() == reduced
    assert np.all(c[:, 3] == np.array(reduced) * n_pes)
    two_shot_ar = n_pes > 1 and mode == 0 and not one_shot
    # two-shot: each PE acquires every PE's "all my blocks are written" flag
    assert np.all(c[:, 5] == (n_pes if two_shot_ar else 0))
    assert np.all(c[:, 4] == (np.array(reduced) * n_pes if two_shot_ar else 0))
    # the event tensor holds the epoch exactly where the graph published
    for pe in range(n_pes):
        words = r["events"][pe]
        arrive = words[:2 * n_pes * tiles * 4].reshape(2, n_pes, tiles, 4)
        done = words[2 * n_pes * tiles * 4:].reshape(2, n_pes)
        assert np.all(arrive[0] == 0) and np.all(done[0] == 0)  # epoch 5: parity plane 1
        assert set(np.unique(arrive[1]).tolist()) <= {0, 5}
        assert np.all(done[1] == (5 if two_shot_ar else 0))
        # every reduced tile's active quarters arrived from every PE
        for t in reduced_tiles[pe]:
            for q in range(4):
                if (t // n_tiles) * 128 + q * 32 < m:
                    assert np.all(arrive[1, :, t, q] == 5)


def test_locate_matches_product_schedule():
    """oracle_locate restates the device queue's raster order exactly."""
    import megacu_b200 as mb
    cases = [(4096, 8192, 1, 0), (4096, 8192, 8, 0), (8192, 8192, 8, 1), (16, 8192, 8, 0),
             (1000, 2000, 3, 0), (2048, 512, 4, 1), (130, 72, 2, 0)]
    for m, n, n_pes, mode in cases:
        prob = mb.Problem(m, n, 64, mode=mode)
        pl = mb.plan(prob, n_pes)
        seen = set()
        for r in range(pl.tiles):
            got = mb.plan_tile(prob, n_pes, r)
            assert got == oracle_lib.locate(pl.m_tiles, pl.n_tiles, n_pes, mode, pl.group_m, r)
            seen.add(got[0] * pl.n_tiles + got[1])
            if mode == 1:  # reduce-scatter: the owner holds the tile's rows
                assert got[0] // (pl.m_tiles // n_pes) == got[2]
        assert len(seen) == pl.tiles


def test_pair_schedule_matches_oracle_and_pairs_neighbours():
    """CTA pairs: every pair ticket maps (product and oracle alike) to two
    vertically adjacent 128-row tiles of one column, the upper one first, with
    the same owner in reduce-scatter; the tickets cover every tile once."""
    import megacu_b200 as mb
    cases = [(4096, 8192, 1, 0, 0), (4096, 8192, 8, 0, 0), (8192, 8192, 8, 1, 0),
             (4096, 8192, 2, 1, 0), (1024, 2000, 3, 0, 128), (2048, 512, 4, 1, 256),
             (200, 264, 1, 0, 128)]
    for m, n, n_pes, mode, tile_n in cases:
        prob = mb.Problem(m, n, 64, mode=mode, tile_n=tile_n)
        pl = mb.plan(prob, n_pes)
        assert pl.cta_pairs and pl.gemm_units == pl.tiles // 2, (m, n, n_pes, mode)
        seen = set()
        for q in range(pl.gemm_units):
            pair = mb.plan_pair(prob, n_pes, q)
            assert pair == oracle_lib.pair_raster(n_pes, mode, q)
            up, low = (mb.plan_tile(prob, n_pes, r) for r in pair)
            assert up[0] % 2 == 0 and low[0] == up[0] + 1 and low[1] == up[1]
            if mode == 1:
                assert up[2] == low[2]
            seen.add(up[0] * pl.n_tiles + up[1])
            seen.add(low[0] * pl.n_tiles + low[1])
        assert len(seen) == pl.tiles


def test_pair_plan_choices():
    import megacu_b200 as mb
    # odd tile rows, tile_n 64 (decode shapes), or an odd per-PE row block: no pairs
    for prob, n_pes in [(mb.Problem(384, 8192, 64), 1), (mb.Problem(16, 8192, 3584), 8),
                        (mb.Problem(256, 512, 64, tile_n=64), 1),
                        (mb.Problem(3072, 8192, 64, mode=mb.MODE_REDUCE_SCATTER), 8)]:
        pl = mb.plan(prob, n_pes)
        assert not pl.cta_pairs and pl.gemm_units == pl.tiles
        prob.cta_pairs = mb.CTA_PAIRS_ON
        with pytest.raises(mb.MegacuError) as err:
            mb.plan(prob, n_pes)
        assert err.value.detail == 27
    prob = mb.Problem(4096, 8192, 1024, cta_pairs=mb.CTA_PAIRS_OFF)
    pl = mb.plan(prob, 8)
    assert not pl.cta_pairs and pl.gemm_units == pl.tiles
    with pytest.raises(mb.MegacuError):
        mb.plan_pair(prob, 8, 0)
    prob.cta_pairs = 3
    with pytest.raises(mb.MegacuError):
        mb.plan(prob, 8)


def test_mlp_chain_matches_float64_restatement():
    """oracle_mlp_chain against a numpy float64 restatement of the same
    semantics (bf16 roundings at act, at the wire and at each block's output)."""
    rng = np.random.default_rng(5)
    t, h, i, layers, n_pes = 48, 64, 40, 2, 3
    rb = oracle_lib.round_bf16
    x = rb(rng.normal(0, 1, (t, h)).astype(np.float32))
    wg = [[rb(rng.normal(0, 0.1, (h, i)).astype(np.float32)) for _ in range(n_pes)]
          for _ in range(layers)]
    wu = [[rb(rng.normal(0, 0.1, (h, i)).astype(np.float32)) for _ in range(n_pes)]
          for _ in range(layers)]
    wd = [[rb(rng.normal(0, 0.1, (i, h)).astype(np.float32)) for _ in range(n_pes)]
          for _ in range(layers)]
    for wire in (2, 4):
        got = oracle_lib.mlp_chain(x, wg, wu, wd, wire_bytes=wire)
        cur = x.astype(np.float64)
        for l in range(layers):
            total = np.zeros((t, h))
            for p in range(n_pes):
                g = cur @ wg[l][p]
                u = cur @ wu[l][p]
                act = rb((g / (1 + np.exp(-g)) * u).astype(np.float32)).astype(np.float64)
                part = (act @ wd[l][p]).astype(np.float32)
                total += rb(part) if wire == 2 else part
            cur = rb(total.astype(np.float32)).astype(np.float64)
        scale = np.abs(cur).max()
        assert np.max(np.abs(got - cur)) < 1e-2 * scale, wire
        assert np.all(np.isfinite(got))


@pytest.mark.parametrize("layers,n_pes,tokens,hidden,inter", [
    (1, 1, 128, 256, 128), (2, 2, 200, 512, 384), (3, 8, 1000, 1024, 640)])
def test_chain_event_oracle_is_consistent(layers, n_pes, tokens, hidden, inter):
    """The single-launch chain's event words: every owner holds every PE's
    flag for each active quarter of its tiles; counters add up across PEs."""
    r = oracle_lib.chain_events(layers, n_pes, tokens, hidden, inter, epoch=5)
    mt, dn, gn = -(-tokens // 128), -(-hidden // 256), -(-inter // 128)
    aq = [min(4, -(-(tokens - 128 * row) // 32)) for row in range(mt)]
    quarters = sum(aq)
    base = layers * n_pes * mt * dn * 4
    flags = sum(int((e[:base] == 5).sum()) for e in r["events"])
    assert flags == (layers * n_pes * dn * quarters if n_pes > 1 else 0)
    c = r["counters"]
    for pe in range(n_pes):
        e = r["events"][pe]
        assert e[base:base + layers * mt].tolist() == [q * gn for q in aq] * layers
        assert e[base + layers * mt:].tolist() == [q * dn for q in aq] * layers
        assert c[pe, 0] == layers * mt * (gn + dn) and c[pe, 2] == layers * quarters * (gn + dn)
    if n_pes > 1:
        assert int(c[:, 1].sum()) == layers * dn * quarters    # every (tile, quarter) reduced once
        assert (c[:, 3] == c[:, 1] * n_pes).all() and (c[:, 5] == n_pes).all()


@pytest.mark.parametrize("n_pes,mode,one_shot", [(2, 0, True), (3, 0, False), (4, 1, False)])
def test_bf16_graph_does_not_depend_on_k_or_data(n_pes, mode, one_shot):
    """The event words and counters of a call depend on m, n, the tiles and
    the PEs only: the full-size multi-GPU test computes them with k = 8."""
    m, n, tile_n = 512, 384, 128
    rng = np.random.default_rng(5)
    graphs = []
    for k, zero in ((8, True), (64, False)):
        a = [np.zeros((m, k), np.float32) if zero else
             rng.standard_normal((m, k)).astype(np.float32) for _ in range(n_pes)]
        b = [np.zeros((k, n), np.float32) if zero else
             rng.standard_normal((k, n)).astype(np.float32) for _ in range(n_pes)]
        tiles = -(-m // 128) * -(-n // tile_n)
        ev0 = [np.zeros(oracle_lib.event_tensor_words(n_pes, tiles), np.uint32)
               for _ in range(n_pes)]
        kw = dict(m=m, n=n, k=k, tile_n=tile_n, mode=mode, one_shot=one_shot)
        r1 = oracle_lib.bf16_call(a, b, epoch=1, events=ev0, **kw)
        r2 = oracle_lib.bf16_call(a, b, epoch=2, events=r1["events"], **kw)
        graphs.append(([e.copy() for e in r2["events"]], r1["counters"] + r2["counters"]))
    (ev_a, c_a), (ev_b, c_b) = graphs
    assert all(np.array_equal(x, y) for x, y in zip(ev_a, ev_b))
    assert np.array_equal(c_a, c_b)
