"""Co-resident persistent progress, host side (no GPU): the lowering of a
phase into one persistent launch's unit graph (megacu/runtime/co_resident.h,
a B200 extension; megacu's own scheduler rejects this progress model,
src/scheduler/explicit_asap.cc:34-39)."""
from __future__ import annotations

import ctypes
import random

import pytest

MAX_DEPS = 8


@pytest.fixture(scope="module")
def lib():
    from megacu_b200 import build
    return ctypes.CDLL(build.build_harness())


def lower(lib, kinds, deps, grids=None, ev=None, events=(), progress=1, storage=0xFFFF, ev2=None):
    """ev[i] = [published, acquired, joined] event tensor of task i (-1 = none);
    ev2[i] = a second acquired tensor. Node publish / acquire come back as bit masks."""
    n = len(kinds)
    grids = grids or [[0, 0]] * n
    ev = ev or [[-1, -1, -1]] * n
    ev2 = ev2 or [-1] * n
    flat = []
    for d in deps:
        flat += list(d) + [-1] * (MAX_DEPS - len(d))
    i32, i64 = ctypes.c_int32, ctypes.c_int64
    status = (i32 * 2)()
    header = (i64 * 3)()
    nodes = (i64 * (8 * 16))()
    evs = (i64 * (2 * 16))()
    lib.harness_co_resident(
        n, (i32 * max(n, 1))(*kinds), (i32 * max(len(flat), 1))(*flat),
        (i64 * max(2 * n, 1))(*[v for g in grids for v in g]),
        (i32 * max(3 * n, 1))(*[v for e in ev for v in e]), (i32 * max(n, 1))(*ev2), len(events),
        (i64 * max(2 * len(events), 1))(*[v for e in events for v in e]), storage, progress,
        status,
        header, nodes, evs)
    out = dict(status=list(status), node_count=header[0], units=header[1])
    out["nodes"] = [dict(task=nodes[8 * k], publish=nodes[8 * k + 1], acquire=nodes[8 * k + 2],
                         wait=nodes[8 * k + 3], units=nodes[8 * k + 4],
                         first=nodes[8 * k + 5], pos=nodes[8 * k + 6])
                    for k in range(header[0])]
    out["events"] = [dict(slots=evs[2 * e], publisher=evs[2 * e + 1]) for e in range(header[2])]
    return out


def test_only_co_resident_progress(lib):
    assert lower(lib, [0], [[]], progress=0)["status"] == [2, 1]


def test_reference_orchestration_becomes_tile_level(lib):
    """gemm_allreduce_orchestrate_common.h:24-76: GEMM tile_grid + publish,
    sync (depends_on GEMM, join), reduce (depends_on sync, acquire, no grid)."""
    g = lower(lib, [0, 1, 0], [[], [0], [1]], grids=[[4, 3], [0, 0], [0, 0]],
              ev=[[0, -1, -1], [-1, -1, 0], [-1, 0, -1]], events=[[4, 3]])
    assert g["status"] == [0, 0] and g["node_count"] == 2 and g["units"] == 24
    gemm, red = g["nodes"]
    assert (gemm["task"], gemm["units"], gemm["first"], gemm["publish"]) == (0, 12, 0, 0b1)
    # one unit per slot, waited for tile by tile: no whole-task wait
    assert (red["task"], red["units"], red["first"], red["acquire"], red["wait"]) == (2, 12, 12, 0b1, 0)
    assert g["events"] == [dict(slots=12, publisher=0)]


def test_sync_without_join_is_a_barrier(lib):
    g = lower(lib, [0, 1, 0], [[], [0], [1]], grids=[[2, 2], [0, 0], [2, 2]],
              ev=[[0, -1, -1], [-1, -1, -1], [-1, 0, -1]], events=[[2, 2]])
    assert g["status"] == [0, 0] and g["nodes"][1]["wait"] == 0b1


def test_direct_dependency_on_the_publisher_is_tile_level(lib):
    g = lower(lib, [0, 0], [[], [0]], grids=[[2, 2], [2, 2]],
              ev=[[0, -1, -1], [-1, 0, -1]], events=[[2, 2]])
    assert g["status"] == [0, 0] and g["nodes"][1]["wait"] == 0


def test_joining_sync_keeps_its_other_dependencies(lib):
    # P (0) publishes E, Q (1) unrelated, S (2) depends on P and Q and joins E,
    # C (3) depends on S and acquires E: C waits for all of Q, P tile by tile.
    g = lower(lib, [0, 0, 1, 0], [[], [], [0, 1], [2]], grids=[[1, 4], [0, 0], [0, 0], [1, 4]],
              ev=[[0, -1, -1], [-1, -1, -1], [-1, -1, 0], [-1, 0, -1]], events=[[1, 4]])
    assert g["status"] == [0, 0]
    assert [nd["units"] for nd in g["nodes"]] == [4, 1, 4]
    assert g["nodes"][2]["wait"] == 0b10


def test_unit_ranges_follow_the_asap_order(lib):
    # task 0 depends on task 1: the queue runs 1 first
    g = lower(lib, [0, 0], [[1], []], grids=[[1, 3], [1, 5]])
    assert g["status"] == [0, 0]
    a, b = g["nodes"]
    assert (b["first"], b["pos"], a["first"], a["pos"]) == (0, 0, 5, 1)
    assert a["wait"] == 0b10


@pytest.mark.parametrize("kinds,deps,grids,ev,events,want", [
    ([0, 0], [[1], [0]], None, None, (), [1, 2]),                       # cycle
    ([0, 0], [[], [9]], None, None, (), [1, 2]),                        # dangling
    ([0, 0, 0], [[], [], [0, 1]], None,
     [[0, -1, -1], [0, -1, -1], [-1, -1, -1]], [[1, 1]], [2, 9]),       # two publishers
    ([0, 0], [[], [0]], [[1, 2], [1, 2]],
     [[-1, -1, -1], [-1, 0, -1]], [[1, 2]], [1, 6]),                    # nobody publishes
    ([0, 0], [[], [0]], [[1, 2], [1, 3]],
     [[0, -1, -1], [-1, 0, -1]], [[1, 2]], [1, 6]),                     # tiles != slots
    ([0, 0], [[], []], [[1, 2], [1, 2]],
     [[-1, 0, -1], [0, -1, -1]], [[1, 2]], [1, 6]),                     # publisher queued later
    ([0], [[]], [[1, 2]], [[0, 0, -1]], [[1, 2]], [1, 6]),              # acquires its own
])
def test_rejections(lib, kinds, deps, grids, ev, events, want):
    assert lower(lib, kinds, deps, grids, ev, events)["status"] == want


def test_device_event_tensors_need_storage(lib):
    args = ([0, 0], [[], [0]], [[1, 2], [1, 2]], [[0, -1, -1], [-1, 0, -1]], [[1, 2]])
    assert lower(lib, *args)["status"] == [0, 0]
    assert lower(lib, *args, storage=0)["status"] == [1, 6]
    # a tensor nobody publishes or acquires on the device may go without
    assert lower(lib, [0], [[]], events=[[1, 2]], storage=0)["status"] == [0, 0]


def test_two_acquired_tensors_are_both_tile_level(lib):
    # P0 publishes E0, P1 publishes E1 (same shape); C acquires both and
    # depends on both directly: no whole-node wait, one unit per slot.
    g = lower(lib, [0, 0, 0], [[], [], [0, 1]], grids=[[2, 3], [2, 3], [0, 0]],
              ev=[[0, -1, -1], [1, -1, -1], [-1, 0, -1]], ev2=[-1, -1, 1],
              events=[[2, 3], [2, 3]])
    assert g["status"] == [0, 0]
    c = g["nodes"][2]
    assert (c["acquire"], c["units"], c["wait"]) == (0b11, 6, 0)
    # different slot counts cannot both be one per tile
    g = lower(lib, [0, 0, 0], [[], [], [0, 1]], grids=[[2, 3], [1, 3], [0, 0]],
              ev=[[0, -1, -1], [1, -1, -1], [-1, 0, -1]], ev2=[-1, -1, 1],
              events=[[2, 3], [1, 3]])
    assert g["status"] == [1, 6]


def test_a_sync_joining_one_of_two_tensors(lib):
    # S joins E0 only: through S, P0 is tile-level but P1 is a whole-node wait.
    g = lower(lib, [0, 0, 1, 0], [[], [], [0, 1], [2]], grids=[[1, 4], [1, 4], [0, 0], [0, 0]],
              ev=[[0, -1, -1], [1, -1, -1], [-1, -1, 0], [-1, 0, -1]], ev2=[-1, -1, -1, 1],
              events=[[1, 4], [1, 4]])
    assert g["status"] == [0, 0]
    assert g["nodes"][2]["wait"] == 0b10


def test_published_tensor_needs_one_slot_per_tile(lib):
    # 8 tiles publishing into 4 slots would write past the tensor
    assert lower(lib, [0], [[]], grids=[[2, 4]], ev=[[0, -1, -1]],
                 events=[[2, 2]])["status"] == [1, 6]
    assert lower(lib, [0], [[]], grids=[[2, 4]], ev=[[0, -1, -1]],
                 events=[[2, 4]])["status"] == [0, 0]


def test_node_capacity(lib):
    assert lower(lib, [0] * 16, [[]] * 16)["status"] == [0, 0]
    assert lower(lib, [0] * 17, [[]] * 17)["status"] == [2, 8]
    assert lower(lib, [0] * 16 + [1] * 4, [[]] * 20)["status"] == [0, 0]  # syncs are no nodes


def _asap(kinds, deps):
    done, order = set(), []
    while len(order) < len(kinds):
        pick = next(i for i in range(len(kinds))
                    if i not in done and all(d in done for d in deps[i]))
        done.add(pick)
        order.append(pick)
    return order


def _reachable_ops(i, kinds, deps):
    """Operator tasks task i depends on, directly or through sync tasks."""
    out, stack, seen = set(), list(deps[i]), set()
    while stack:
        x = stack.pop()
        if x in seen:
            continue
        seen.add(x)
        if kinds[x] == 0:
            out.add(x)
        else:
            stack += deps[x]
    return out


@pytest.mark.parametrize("seed", range(40))
def test_random_graphs_cover_every_dependency(lib, seed):
    rng = random.Random(9100 + seed)
    n = rng.randint(1, 14)
    kinds = [1 if rng.random() < 0.3 else 0 for _ in range(n)]
    deps = [sorted(rng.sample(range(t), min(t, rng.randint(0, 3)))) for t in range(n)]
    n_ev = rng.randint(0, 3)
    shapes = [[rng.randint(1, 3), rng.randint(1, 4)] for _ in range(n_ev)]
    ev = [[-1, -1, -1] for _ in range(n)]
    grids = [[0, 0] for _ in range(n)]
    publishers = {}
    for e in range(n_ev):
        # a publisher has the tensor's tile grid; an acquirer has it too, or
        # no grid (one unit per slot)
        ops = [i for i in range(n) if kinds[i] == 0 and ev[i][0] < 0 and ev[i][1] < 0
               and grids[i] == [0, 0]]
        if not ops:
            break
        p = rng.choice(ops)
        ev[p][0], publishers[e] = e, p
        grids[p] = list(shapes[e])
        later = [i for i in range(p + 1, n) if kinds[i] == 0 and ev[i][1] < 0 and ev[i][0] < 0
                 and grids[i] == [0, 0]]
        for c in rng.sample(later, min(len(later), 2)):
            ev[c][1] = e
            if rng.random() < 0.5:
                grids[c] = list(shapes[e])
            if p not in deps[c]:
                deps[c] = sorted(set(deps[c]) | {p})
        syncs = [i for i in range(n) if kinds[i] == 1]
        if syncs:
            ev[rng.choice(syncs)][2] = e
    for i in range(n):
        if kinds[i] == 0 and grids[i] == [0, 0] and ev[i][1] < 0 and rng.random() < 0.5:
            grids[i] = [rng.randint(1, 3), rng.randint(1, 3)]
    g = lower(lib, kinds, deps, grids, ev, shapes)
    assert g["status"] == [0, 0], (kinds, deps, grids, ev)
    ops = [i for i in range(n) if kinds[i] == 0]
    node_of = {t: k for k, t in enumerate(ops)}
    assert [nd["task"] for nd in g["nodes"]] == ops
    # queue: the ASAP order of the operator tasks, units back to back
    queue = [t for t in _asap(kinds, deps) if kinds[t] == 0]
    first = 0
    for pos, t in enumerate(queue):
        nd = g["nodes"][node_of[t]]
        assert (nd["pos"], nd["first"]) == (pos, first)
        first += nd["units"]
    assert g["units"] == first
    for t in ops:
        nd = g["nodes"][node_of[t]]
        need = {node_of[x] for x in _reachable_ops(t, kinds, deps)}
        waits = {j for j in range(len(ops)) if (nd["wait"] >> j) & 1}
        assert waits <= need                                   # no spurious waits
        acquired = [e for e in range(len(shapes)) if (nd["acquire"] >> e) & 1]
        pubs = {g["events"][e]["publisher"] for e in acquired}
        assert need - waits <= pubs                            # the rest: tile by tile
        for j in waits | pubs:
            assert g["nodes"][j]["pos"] < nd["pos"]             # waits target earlier units
        for e in acquired:
            pub = g["events"][e]["publisher"]
            assert g["nodes"][pub]["units"] == nd["units"] == shapes[e][0] * shapes[e][1]


FAKE = 0x100000  # never dereferenced: validation-only calls


def test_f32_entry_validation_only():
    import megacu_b200 as mb
    from megacu_b200 import _capi
    lib = _capi.load()
    d = mb.driver_view(None, 0)
    d.team.team_n_pes, d.team.world_n_pes = 2, 2
    p = _capi.GemmArProblem(m=256, n=256, k=64, tile_m=128, tile_n=128)
    fn = lib.megacu_cuda_gemm_allreduce_f32_co_resident
    st = fn(d, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, p)
    assert (st.code, st.detail) == (0, 0)
    st = fn(d, FAKE, FAKE, FAKE, FAKE, FAKE, None, p)
    assert (st.code, st.detail) == (1, 2)
    bad = _capi.GemmArProblem(m=0, n=256, k=64, tile_m=128, tile_n=128)
    st = fn(d, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, bad)
    assert (st.code, st.detail) == (1, 1)
    # the state holds the graph (16 nodes, 16 event tensors) and the counters
    assert mb.co_resident_control_bytes() >= 16 * 32 + 16 * 24 + 4 * (4 + 16)


def build_example(out_dir):
    """Compiles tests/cpp/co_resident_example.cu (a three-task phase with
    per-tile dataflow and its own device operators, built on the public
    headers) against libmegacu_b200.so; returns the executable's path."""
    import os
    import shutil
    import subprocess

    from megacu_b200 import build
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not found")
    exe = os.path.join(out_dir, "co_resident_example")
    cmd = [nvcc, "-std=c++20", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I" + os.path.join(build.ROOT, "include"),
           os.path.join(build.ROOT, "tests", "cpp", "co_resident_example.cu"),
           "-L" + build.LIB_DIR, "-lmegacu_b200", "-Xlinker", "-rpath=" + build.LIB_DIR,
           "-o", exe]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-3000:]
    return exe


def test_example_program_builds(tmp_path):
    assert build_example(str(tmp_path))
