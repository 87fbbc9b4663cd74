"""Host-runtime scenarios run through tests/cpp/host_runtime_harness.cc.

Used by tests/golden/make_golden.py (against the reference's compiled host
runtime) and by tests/test_host_runtime.py (against ours). The scenarios
cover megacu's contract tests (tests/build/runtime_components_contracts.cc:
59-184, tests/build/runtime_linked_surface_contract.cc:74-118) plus seeded
random dependency graphs.
"""
from __future__ import annotations

import ctypes
import random

MAX_DEPS = 8


def _scenario(name, kinds, deps, tile_grid=None, ev_attr=None, events=(), mode=0, progress=0,
              fail_at=-1):
    n = len(kinds)
    return dict(name=name, kinds=list(kinds), deps=[list(d) for d in deps],
                tile_grid=[list(t) for t in (tile_grid or [[0, 0]] * n)],
                ev_attr=list(ev_attr or [0] * n), events=[list(e) for e in events], mode=mode,
                progress=progress, fail_at=fail_at)


def scenarios() -> list[dict]:
    out = [
        # first, second, second-after-first (components_contracts.cc:84-106)
        _scenario("asap_order", [0, 0, 0], [[], [], [0]]),
        # tile_grid(2, 3) -> 6 tiles (components_contracts.cc:110-122)
        _scenario("tile_grid", [0], [[]], tile_grid=[[2, 3]]),
        # publish -> sync(join) -> acquire over shape(2, 3) (components_contracts.cc:133-164)
        _scenario("event_sync", [0, 1, 0], [[], [0], [1]], ev_attr=[1, 4, 2], events=[[2, 3]]),
        # the orchestration of linked_surface_contract.cc:45-66 run with a launcher
        _scenario("launcher_only", [0, 1, 0], [[], [0], [1]], tile_grid=[[1, 1], [0, 0], [0, 0]],
                  ev_attr=[1, 4, 2], events=[[1, 1]], mode=1),
        # co_resident_persistent is rejected (components_contracts.cc:170-173)
        _scenario("progress_unsupported", [0], [[]], progress=1),
        _scenario("progress_unsupported_launcher", [0], [[]], progress=1, mode=1),
        # a cycle and a dangling dependency -> invalid_argument 2
        _scenario("cycle", [0, 0], [[1], [0]]),
        _scenario("dangling", [0, 0], [[], [7]]),
        # an operator body failing stops the walk with its own status
        _scenario("body_failure", [0, 0, 0], [[], [0], [1]], fail_at=1),
        # the megakernel phase of the GEMM + allreduce orchestration
        _scenario("gemm_allreduce_phase", [0, 1, 0], [[], [0], [1]],
                  tile_grid=[[32, 32], [0, 0], [0, 0]], ev_attr=[1, 4, 2], events=[[32, 32]],
                  mode=1),
    ]
    rng = random.Random(20261201)
    for i in range(150):
        n = rng.randint(1, 20)
        kinds = [1 if rng.random() < 0.3 else 0 for _ in range(n)]
        deps = []
        for t in range(n):
            pool = list(range(n)) if rng.random() < 0.15 else list(range(t))
            k = min(len(pool), rng.randint(0, 4))
            deps.append(rng.sample(pool, k) if k else [])
        grids = [[rng.randint(0, 5), rng.randint(1, 7)] for _ in range(n)]
        ev_attr = [rng.randint(0, 7) for _ in range(n)]
        n_events = rng.randint(0, 3)
        events = [[rng.randint(1, 9), rng.randint(1, 9)] for _ in range(n_events)]
        # from the 25th on, also a rejected progress model or a failing body
        progress = 1 if i >= 24 and rng.random() < 0.1 else 0
        fail_at = rng.randrange(n) if i >= 24 and rng.random() < 0.15 else -1
        out.append(_scenario(f"random_{i}", kinds, deps, grids, ev_attr, events,
                             mode=rng.randint(0, 1), progress=progress, fail_at=fail_at))
    return out


def run_scenario(lib: ctypes.CDLL, sc: dict) -> dict:
    n = len(sc["kinds"])
    kinds = (ctypes.c_int32 * max(n, 1))(*sc["kinds"])
    flat = []
    for d in sc["deps"]:
        flat += list(d) + [-1] * (MAX_DEPS - len(d))
    deps = (ctypes.c_int32 * max(len(flat), 1))(*flat)
    grid = (ctypes.c_int64 * max(2 * n, 1))(*[v for g in sc["tile_grid"] for v in g])
    ev_attr = (ctypes.c_int32 * max(n, 1))(*sc["ev_attr"])
    n_events = len(sc["events"])
    shapes = (ctypes.c_int64 * max(2 * n_events, 1))(*[v for e in sc["events"] for v in e])
    order = (ctypes.c_int32 * (n + 2))()
    order_len = ctypes.c_int32()
    counts = (ctypes.c_int64 * 9)()
    status = (ctypes.c_int32 * 2)()
    lib.harness_phase(n, kinds, deps, grid, ev_attr, n_events, shapes, sc["mode"],
                      sc["progress"], sc["fail_at"], order, ctypes.byref(order_len), counts,
                      status)
    return dict(order=list(order[: order_len.value]), counts=list(counts),
                status=list(status))


def run_fixed(lib: ctypes.CDLL) -> dict:
    out = {}
    for tasks, events in [(1, 1), (2, 1), (3, 1), (2, 2), (3, 2)]:
        status = (ctypes.c_int32 * 2)()
        ti, ei = ctypes.c_int32(), ctypes.c_int32()
        lib.harness_capacity(tasks, events, status, ctypes.byref(ti), ctypes.byref(ei))
        out[f"capacity_{tasks}_{events}"] = dict(status=list(status), task_invalid=ti.value,
                                                 event_invalid=ei.value)
    status = (ctypes.c_int32 * 2)()
    lib.harness_missing_entry(status)
    out["missing_entry"] = dict(status=list(status))
    out["attr_capacity"] = lib.harness_attr_capacity(12)
    comps = (ctypes.c_int32 * 8)()
    lib.harness_components(comps)
    out["components"] = list(comps)
    return out
