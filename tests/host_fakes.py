"""Host stand-ins for the CUDA calls of bench.py and the timing tools, so their
Python logic (argument handling, buffer sizing, the timing loop, the JSON
line) runs on the CPU. Test infrastructure: the numbers they produce mean
nothing.

* CUDA events report a fixed time per rank (``rank_ms``); streams, device
  selection, synchronisation and CUDA graphs do nothing.
* ``torch.matmul`` returns its ``out`` (or zeros): no host GEMM of full size.
* The team's tensors are host tensors, counted against its heap.
* The package's launches (``gemm_allreduce``, ``allgather_gemm``,
  ``mlp_chain``) record their name and optionally check their arguments.
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


def install(rank, patch, launches, check=None):
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

    class Graph:
        def replay(self):
            pass

    class Team:
        def __init__(self, rank, tp, device, heap, exchange, multicast_bytes=0):
            self.multicast = False
            self.heap, self.used = heap, 0

        def tensor(self, shape, dtype, multicast=False):
            t = torch.zeros(shape, dtype=dtype)
            self.used += t.numel() * t.element_size()
            assert self.used <= self.heap, f"team heap overflow: {self.used} > {self.heap}"
            return t

        def barrier(self, stream=None):
            pass

        def close(self):
            pass

    def launch(name):
        def body(*args, **kwargs):
            if check is not None:
                check(name, args, kwargs)
            launches.append(name)
        return body

    init = dist.init_process_group

    def init_gloo(backend=None, **kw):
        kw.pop("device_id", None)
        return init("gloo", **kw)

    patch(torch.cuda, "Event", Event)
    patch(torch.cuda, "CUDAGraph", Graph)
    patch(torch.cuda, "graph", lambda g, **kw: contextlib.nullcontext())
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
