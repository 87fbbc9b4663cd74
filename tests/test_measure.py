"""Host-side arithmetic of the timing tools (no GPU)."""
import pytest

from megacu_b200 import measure, shapes_bench


def test_decode_roofline_is_the_weight_stream(monkeypatch):
    monkeypatch.setattr(measure, "PEAKS_PATH", "/nonexistent")
    monkeypatch.setattr(shapes_bench, "peaks", measure.peaks)
    monkeypatch.setattr(shapes_bench, "hbm_peak", measure.hbm_peak)
    m, n, k, tp = 16, 8192, 28672 // 8, 8
    r = shapes_bench.roofline(4, m, n, k, tp, us=10.0)
    hbm_bytes = 2.0 * (m * k + k * n) + m * n * 2
    assert r["bound"] == "hbm"
    assert r["hbm_bytes_per_pe"] == hbm_bytes
    assert r["terms_us"]["hbm"] == pytest.approx(hbm_bytes / 6650e9 * 1e6)
    assert r["link_bytes_per_pe"] == 7 * m * n * 2          # one-shot: to every peer
    assert r["terms_us"]["tensor"] == pytest.approx(2.0 * m * n * k / 1590e12 * 1e6)
    assert r["frac"] == pytest.approx(r["roofline_us"] / 10.0)
    assert "fallback" in r["peak_source"] and "fallback" in r["hbm_source"]


def test_reduce_scatter_roofline_is_the_gemm():
    m, n, k, tp = 8192, 8192, 28672 // 8, 8
    r = shapes_bench.roofline(3, m, n, k, tp, us=300.0)
    assert r["link_bytes_per_pe"] == pytest.approx(7 / 8 * m * n * 2)
    assert r["bound"] == "tensor"
    assert r["flops_per_pe"] == 2.0 * m * n * k


def test_clock_summary_reads_reasons():
    s = measure.ClockSampler(0)
    assert s.summary()["reasons"] == ["unsampled"]
    s.rows = [["0", "1500", "1965", "900", "0x4", "Not Active", "Not Active", "Not Active",
               "Active"],
              ["0", "1300", "1965", "990", "0x4", "Not Active", "Not Active", "Not Active",
               "Active"]]
    out = s.summary()
    assert out["sm_mhz"] == 1400 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 2


def test_allgather_roofline_counts_the_gathered_rows():
    m, n, k, tp = 8192, 28672 // 8, 8192, 8
    r = shapes_bench.roofline("ag", m, n, k, tp, us=400.0)
    assert r["link_bytes_per_pe"] == pytest.approx(7 / 8 * m * k * 2)
    assert r["hbm_bytes_per_pe"] == 2.0 * (m * k + k * n) + m * n * 2 + 2.0 * m * k
    assert r["bound"] == "tensor"


def test_interleaved_orders_arms_and_takes_the_max_over_ranks(monkeypatch):
    """The timing loop with fake CUDA events: warm-up untimed, arms
    interleaved step by step with align() before each, one value per step and
    arm, the max over ranks (two gloo ranks emulated by a fake all_reduce)."""
    import torch
    import torch.distributed as dist

    log = []
    clock = [0.0]

    class FakeEvent:
        def __init__(self, enable_timing=False):
            self.t = None

        def record(self, stream=None):
            self.t = clock[0]

        def elapsed_time(self, end):
            return end.t - self.t

    def body(i):
        def run():
            log.append(("body", i))
            clock[0] += 1.0 + i   # arm i takes 1 + i ms
        return run

    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    reduced = []

    def fake_all_reduce(t, op=None):
        reduced.append(op)
        t.mul_(2.0)           # the other rank was twice as slow
    monkeypatch.setattr(dist, "all_reduce", fake_all_reduce)
    monkeypatch.setattr(dist, "barrier", lambda *a, **k: None)
    ms = measure.interleaved([body(0), body(1)], steps=3, warmup=2,
                             align=lambda: log.append(("align",)), stream=None, world=2,
                             device="cpu")
    assert ms == [[2.0] * 3, [4.0] * 3]
    assert reduced == [dist.ReduceOp.MAX]
    bodies = [x[1] for x in log if x[0] == "body"]
    assert bodies == [0, 1] * 5                      # 2 warm-up + 3 timed rounds
    assert sum(1 for x in log if x[0] == "align") == 10


def test_decode_link_bytes_by_exchange():
    m, n, k, tp = 128, 8192, 3584, 8
    out = m * n * 2
    one = shapes_bench.roofline(4, m, n, k, tp, us=20.0)
    two = shapes_bench.roofline(4, m, n, k, tp, us=20.0, one_shot=False)
    nvls = shapes_bench.roofline(4, m, n, k, tp, us=20.0, one_shot=False, in_switch=True)
    assert one["link_bytes_per_pe"] == 7 * out
    assert two["link_bytes_per_pe"] == pytest.approx(2 * 7 / 8 * out)
    assert nvls["link_bytes_per_pe"] == pytest.approx(9 / 8 * out)
    # at M = 128 the one-shot exchange, not the weight stream, bounds the call
    assert one["bound"] == "nvlink" and two["bound"] == "hbm"


@pytest.mark.parametrize("n_pes,m,n,tile_n,one_shot,mode", [
    (1, 512, 768, 256, False, 0), (2, 512, 1024, 256, True, 0), (2, 1024, 512, 128, False, 0),
    (4, 1024, 1024, 256, False, 0), (8, 1024, 2048, 256, False, 0), (8, 128, 1024, 64, True, 0),
    (4, 1024, 768, 256, False, 1), (8, 2048, 512, 128, False, 1)])
def test_expected_counters_equal_the_oracle_graph(n_pes, m, n, tile_n, one_shot, mode):
    """The timing tools' closed form of one call's completion counters is the
    oracle's task graph (which depends on the shape, not on k or the data)."""
    import numpy as np

    import oracle_lib
    k = 8
    a = [np.zeros((m, k), np.float32)] * n_pes
    b = [np.zeros((k, n), np.float32)] * n_pes
    ref = oracle_lib.bf16_call(a, b, m=m, n=n, k=k, tile_n=tile_n, mode=mode,
                               one_shot=one_shot)
    for pe in range(n_pes):
        got = measure.expected_counters(n_pes, pe, m // 128, n // tile_n, tile_n, one_shot, mode)
        assert got == ref["counters"][pe].tolist(), pe


def test_output_errors_measures():
    import torch
    want = torch.tensor([[1.0, -2.0, 1e-6, 4.0]])
    got = torch.tensor([[1.005, -2.0, 0.0, 4.0]])
    e = measure.output_errors(got, want)
    rms = float(want.pow(2).mean().sqrt())
    assert e["max_rel_err_strict"] == pytest.approx(0.005, rel=1e-4)  # 1e-6 is below the floor
    assert e["max_rel_err"] == pytest.approx(0.005 / (1.0 + rms), rel=1e-4)
    scaled = measure.output_errors(got, want, scale=torch.full_like(want, 10.0))
    assert scaled["max_rel_err"] == pytest.approx(0.005 / (10.0 + rms), rel=1e-4)
    bad = measure.output_errors(torch.tensor([[float("nan"), 1.0, 1.0, 1.0]]), want)
    assert not bad["max_rel_err"] < 1.0 and not bad["max_rel_err_strict"] < 1.0


def test_timer_tick_is_the_smallest_step_between_samples():
    tick = 2.048e-3  # ms
    samples = [[14 * tick, 15 * tick, 14 * tick], [9 * tick, 12 * tick]]
    assert measure.timer_tick_us(samples) == pytest.approx(2.048)
    assert measure.timer_tick_us([[0.0301, 0.03042, 0.0301]]) == pytest.approx(0.32)
    assert measure.timer_tick_us([[0.03, 0.03]]) is None
    assert measure.timer_tick_us([[]]) is None
