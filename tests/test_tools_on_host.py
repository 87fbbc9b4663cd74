"""The timing tools' Python logic on the CPU (host stand-ins for CUDA, see
host_fakes.py): `shapes_bench` (config 4 decode shapes, both exchange
choices, CUDA-graph arms) and `mlp_bench` (config 5, small sizes) parse their
options, size their buffers within the team heap, time every arm, and print
one JSON line on rank 0 whose time is the max over ranks; `timeline` (fused
call and all-gather) prints on rank 0 one line per PE with that PE's own
times."""
from __future__ import annotations

import contextlib
import io
import json
import os
import socket
import sys

import pytest

import host_fakes

# case name -> (tool module, its options)
TOOLS = {
    "shapes_bench": ("shapes_bench", ["--config", "4", "--m", "16,64", "--steps", "2",
                                      "--heat-calls", "1"]),
    "shapes_bench_two_shot_graph": ("shapes_bench", ["--config", "4", "--m", "64", "--algo",
                                                     "two", "--graph", "--steps", "2",
                                                     "--heat-calls", "1"]),
    "mlp_bench": ("mlp_bench", ["--tokens", "256", "--hidden", "512", "--inter", "1024",
                                "--layers", "2", "--steps", "2", "--heat-calls", "1"]),
    "timeline": ("timeline", ["--m", "512", "--n", "1024", "--k-total", "512", "--calls", "2"]),
    "timeline_allgather": ("timeline", ["--m", "512", "--n", "1024", "--k-total", "512",
                                        "--calls", "2", "--allgather"]),
}


def _run_tool(name, argv):
    module = TOOLS[name][0]
    mod = host_fakes.load_source(f"megacu_b200/{module}.py", package="megacu_b200")
    old = sys.argv
    sys.argv = [module, *argv]
    buf = io.StringIO()
    try:
        with contextlib.redirect_stdout(buf):
            rc = mod.main()
        if rc != 0:
            print(buf.getvalue()[-3000:], file=sys.stderr)
        assert rc == 0
    finally:
        sys.argv = old
    return [json.loads(x) for x in buf.getvalue().splitlines() if x.startswith("{")]


def _check(name, lines, tp):
    ms = host_fakes.rank_ms(tp - 1)  # the slowest rank's step time
    if name.startswith("timeline"):
        assert [x["pe"] for x in lines] == list(range(tp))
        for pe, x in enumerate(lines):
            assert x["tp"] == tp
            assert x["call_us_median"] == pytest.approx(host_fakes.rank_ms(pe) * 1e3)
            assert x["exchange"] == ("all-gather copies" if name.endswith("allgather") else
                                     "peer" if tp > 1 else "none")
    elif name.startswith("shapes_bench"):
        assert [x["m"] for x in lines] == ([16, 64] if name == "shapes_bench" else [64])
        for x in lines:
            assert x["tp"] == tp and x["n"] == 8192 and x["k_per_pe"] == 28672 // tp
            assert x["us_per_call"]["fused"] == pytest.approx(ms * 1e3)
            assert x["us_per_call_mean"] == pytest.approx(x["us_per_call"])  # constant stand-in
            assert x["timer_tick_us"] is None  # every stand-in step takes the same time
            assert {"tensor", "hbm", "nvlink"} <= set(x["roofline_call"]["terms_us"])
            assert ("kernel_without_exchange" in x["us_per_call"]) == (tp > 1)
        if name != "shapes_bench":
            assert lines[0]["plan"]["one_shot"] is False  # --algo two
    else:
        (x,) = lines
        assert x["tp"] == tp
        assert set(x["us_per_call"]) == {"two_launches", "single_launch", "unfused"}
        assert all(u == pytest.approx(ms * 1e3) for u in x["us_per_call"].values())
        roof = x["roofline_call"]
        assert roof["roofline_us"] == max(roof["gemm_us_at_peak"], roof["link_us_at_770GBps"])
        assert set(x["max_rel_err_vs_unfused"]) == {"two_launches", "single_launch"}


@pytest.mark.parametrize("name", list(TOOLS))
def test_tool_on_one_rank(name, monkeypatch):
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("LOCAL_RANK", "0")
    launches = []
    host_fakes.install(0, monkeypatch.setattr, launches)
    lines = _run_tool(name, TOOLS[name][1])
    _check(name, lines, 1)
    assert launches


def _rank_main(rank, out_dir, ports):
    launches = []
    host_fakes.install(rank, setattr, launches)
    got = {}
    for (name, (_, argv)), port in zip(TOOLS.items(), ports):
        os.environ.update(RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank),
                          MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        before = len(launches)
        got[name] = {"lines": _run_tool(name, argv), "launches": len(launches) - before}
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(got, f)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tools_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    ports = [_free_port() for _ in TOOLS]
    mp.spawn(_rank_main, args=(str(tmp_path), ports), nprocs=2, join=True)
    got = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    for name in TOOLS:
        assert got[1][name]["lines"] == []  # rank 0 alone prints
        _check(name, got[0][name]["lines"], 2)
        assert got[0][name]["launches"] == got[1][name]["launches"] > 0
