"""Host stand-ins for the CUDA calls of bench.py and the timing tools, so their
Python logic (argument handling, buffer sizing, the timing loop, the JSON
line) runs on the CPU. Test infrastructure: the numbers they produce mean
nothing.

* CUDA events report a fixed time per rank (``rank_ms``); streams, device
  selection and synchronisation do nothing. A CUDA graph records the
  package's launches made while it is captured (they do not run then) and
  makes them again on every replay.
* ``torch.matmul`` returns its ``out`` (or zeros): no host GEMM of full size.
* The team's tensors are host tensors, counted against its heap.
* The package's launches (``gemm_allreduce``, ``allgather_gemm``,
  ``mlp_chain``) record their name and optionally check their arguments.
  ``events_counters`` returns, per events buffer, the number of
  ``gemm_allreduce`` launches on it times the counters of one call in the
  oracle's task graph (``graph_counters``), or those of a ``counters``
  callback.
* A source file executed through ``load_source`` reads
  ``torch.device("cuda"`` as ``torch.device("cpu"``; the file itself is
  unchanged.
"""
from __future__ import annotations

import contextlib
import os
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LAUNCHES = ("gemm_allreduce", "allgather_gemm", "mlp_chain")


def rank_ms(rank):
    return 1.0 + 0.5 * rank  # higher ranks are slower: the max over ranks is visible


_GRAPH = {}


def graph_counters(problem, n_pes, pe):
    """One call's completion counters on PE `pe` in the oracle's task graph
    (they depend on the shape and the plan, not on k or the data)."""
    import numpy as np

    import megacu_b200 as mb
    import oracle_lib
    plan = mb.plan(problem, n_pes)
    key = (problem.m, problem.n, problem.mode, n_pes, plan.tile_n, plan.one_shot)
    if key not in _GRAPH:
        a = [np.zeros((problem.m, 8), np.float32)] * n_pes
        b = [np.zeros((8, problem.n), np.float32)] * n_pes
        _GRAPH[key] = oracle_lib.bf16_call(a, b, m=problem.m, n=problem.n, k=8,
                                           tile_n=plan.tile_n, mode=problem.mode,
                                           one_shot=plan.one_shot, threads=2)["counters"]
    return _GRAPH[key][pe].tolist()


def install(rank, patch, launches, check=None, counters=graph_counters):
    """Installs the stand-ins with ``patch(obj, name, value)`` (pytest's
    monkeypatch.setattr, or setattr in a child process); every launch appends
    its name to ``launches`` after ``check(name, args, kwargs)``."""
    import torch
    import torch.distributed as dist

    import megacu_b200 as mb

    class Event:
        def __init__(self, enable_timing=False):
            pass

        def record(self, stream=None):
            pass

        def elapsed_time(self, other):
            return rank_ms(rank)

    capturing = []  # the graph being captured, if any

    class Graph:
        def __init__(self):
            self.recorded = []

        def replay(self):
            for body, args, kwargs in self.recorded:
                body(*args, **kwargs)

    @contextlib.contextmanager
    def graph(g, **kw):
        capturing.append(g)
        try:
            yield
        finally:
            capturing.pop()

    class Team:
        def __init__(self, rank, tp, device, heap, exchange, multicast_bytes=0):
            self.multicast = False
            self.heap, self.used = heap, 0
            self.my_pe, self.n_pes = rank, tp

        def tensor(self, shape, dtype, multicast=False):
            t = torch.zeros(shape, dtype=dtype)
            self.used += t.numel() * t.element_size()
            assert self.used <= self.heap, f"team heap overflow: {self.used} > {self.heap}"
            return t

        def barrier(self, stream=None):
            pass

        def close(self):
            pass

    # events buffer address -> [launches, problem, n_pes, pe, the buffer]; the
    # entry keeps the buffer alive, so a later buffer never reuses its address
    per_events = {}

    def launch(name):
        def body(*args, **kwargs):
            if capturing:
                capturing[-1].recorded.append((body, args, kwargs))
                return
            if check is not None:
                check(name, args, kwargs)
            launches.append(name)
            if name == "gemm_allreduce":
                team = kwargs.get("team")
                events = kwargs["events"]
                entry = per_events.setdefault(events.data_ptr(), [0, None, 1, 0, events])
                entry[0] += 1
                entry[1] = kwargs["problem"]
                if team is not None:
                    entry[2], entry[3] = team.n_pes, team.my_pe
        return body

    def events_counters(events, stream=None):
        calls, problem, n_pes, pe, _ = per_events.get(events.data_ptr(), [0, None, 1, 0, None])
        if problem is None:
            return [0] * 8
        return [calls * x for x in counters(problem, n_pes, pe)]

    init = dist.init_process_group

    def init_gloo(backend=None, **kw):
        kw.pop("device_id", None)
        return init("gloo", **kw)

    patch(torch.cuda, "Event", Event)
    patch(torch.cuda, "CUDAGraph", Graph)
    patch(torch.cuda, "graph", graph)
    patch(torch.cuda, "set_device", lambda *a: None)
    patch(torch.cuda, "synchronize", lambda *a: None)
    patch(torch.cuda, "current_stream", lambda *a: None)
    patch(torch.cuda, "current_device", lambda: 0)
    patch(torch.cuda, "Stream", lambda *a, **kw: None)
    patch(torch.Tensor, "pin_memory", lambda self: self)
    patch(torch, "matmul", lambda a, b, out=None: out if out is not None else
          torch.zeros(a.shape[0], b.shape[1], dtype=a.dtype))
    patch(dist, "init_process_group", init_gloo)
    patch(mb, "Team", Team)
    patch(mb, "events_status", lambda *a, **kw: None)
    patch(mb, "events_counters", events_counters)
    for name in LAUNCHES:
        patch(mb, name, launch(name))


def load_source(rel, package=None):
    """Executes the file ``rel`` (relative to the repository root) as a new
    module with "cuda" devices read as host devices."""
    path = os.path.join(ROOT, rel)
    src = open(path).read()
    assert src.count('torch.device("cuda"') >= 1, rel
    mod = types.ModuleType(os.path.splitext(os.path.basename(rel))[0] + "_on_host")
    mod.__file__ = path
    if package:
        mod.__package__ = package
    exec(compile(src.replace('torch.device("cuda"', 'torch.device("cpu"'), path, "exec"),
         mod.__dict__)
    return mod
