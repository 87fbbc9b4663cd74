"""Helpers shared by the GPU tests: seeded inputs, one-call runners, checks."""
from __future__ import annotations

import numpy as np
import torch

import megacu_b200 as mb
from megacu_b200.measure import STRICT_FLOOR

# Tolerance of the bf16 path (north star: max relative error 1e-2, bf16 inputs,
# fp32 accumulate), on two measures:
#  * strict: max |got - want| / |want| over the elements with |want| >=
#    STRICT_FLOOR x RMS(want) (1e-2: below it any two fp32 accumulation
#    orders of K >= 4096 products differ by more than 1e-2 of the value);
#    required of every one-PE output and of the deterministic (fp32-wire)
#    multi-PE mode;
#  * conditioned: |got - want| / (s + RMS(want)), s = |want|, or for bf16
#    partials on the wire (the default multi-PE mode) the sum of the
#    partials' magnitudes: a bf16 partial is exact only to 2^-8 of itself, so
#    a sum that cancels is judged on the scale of its terms. Required always.
REL_TOL = 1e-2


def rel_error(got: np.ndarray, want: np.ndarray, scale: np.ndarray | None = None) -> float:
    """max |got - want| / (s + RMS(want)), s = |want| or, when given, `scale`.

    With bf16 partials on the wire (the default multi-PE mode) each partial is
    exact only to a bf16 ulp of itself, so there the per-element scale is the
    sum of the partials' magnitudes (`wire_scale`), the condition of the sum.
    """
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if not want.size:
        return 0.0
    rms = float(np.sqrt(np.mean(want ** 2)))
    s = np.abs(want) if scale is None else np.asarray(scale, np.float64)
    return float(np.max(np.abs(got - want) / (s + rms + 1e-30)))


def strict_rel_error(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / |want| over elements with |want| >= STRICT_FLOOR x RMS(want)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if not want.size:
        return 0.0
    rms = float(np.sqrt(np.mean(want ** 2)))
    aw = np.abs(want)
    keep = (aw >= STRICT_FLOOR * rms) & (aw > 0)
    if not keep.any():
        return 0.0
    return float(np.max(np.abs(got - want)[keep] / aw[keep]))


def errors(got, want, scale=None) -> tuple[float, float, str]:
    """(conditioned, strict, a line naming both) for an output check."""
    loose = rel_error(got, want, scale)
    strict = strict_rel_error(got, want)
    what = "sum |partial|" if scale is not None else "|want|"
    return loose, strict, (f"max_rel_err {loose:.3e} (over {what} + RMS), strict {strict:.3e} "
                           f"(|want| >= {STRICT_FLOOR} x RMS)")


def assert_close(got, want, scale=None, strict: bool = True, what: str = "") -> None:
    """Both measures are computed and printed; the conditioned one must be
    below REL_TOL, and the strict one too when `strict`."""
    loose, st, line = errors(got, want, scale)
    print(f"{what} {line}".strip())
    assert loose < REL_TOL, f"{what} {line}"
    if strict:
        assert st < REL_TOL, f"{what} {line}"


def wire_scale(a_list, b_list, rows: slice | None = None) -> np.ndarray:
    """Per element, sum over PEs of |a_pe @ b_pe| (fp32 inputs as given)."""
    total = None
    for a, b in zip(a_list, b_list):
        a = f32(a) if isinstance(a, torch.Tensor) else a
        b = f32(b) if isinstance(b, torch.Tensor) else b
        if rows is not None:
            a = a[rows]
        part = np.abs(a.astype(np.float32) @ b.astype(np.float32)).astype(np.float64)
        total = part if total is None else total + part
    return total


def seeded_bf16(seed: int, shape, std: float) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)


def inputs(seed: int, n_pes: int, m: int, n: int, k: int, std_a: float = 1.0,
           std_b: float = 0.02):
    """Per-PE bf16 A [m, k] and B [k, n] (host tensors) from per-(PE, tensor) seeds."""
    a = [seeded_bf16(seed * 100 + 10 * pe + 0, (m, k), std_a) for pe in range(n_pes)]
    b = [seeded_bf16(seed * 100 + 10 * pe + 1, (k, n), std_b) for pe in range(n_pes)]
    return a, b


def f32(t: torch.Tensor) -> np.ndarray:
    return np.ascontiguousarray(t.float().cpu().numpy())


class SinglePE:
    """Device buffers for one-PE calls of the bf16 path on cuda:0."""

    def __init__(self, problem: mb.Problem, device: int = 0):
        self.problem = problem
        self.device = device
        self.plan = mb.plan(problem, 1)
        ev_bytes = mb.events_bytes(problem, 1)
        self.events = torch.zeros(ev_bytes // 4, dtype=torch.int32, device=f"cuda:{device}")
        self.out = torch.empty(problem.m, problem.n, dtype=torch.bfloat16,
                               device=f"cuda:{device}")

    def run(self, a: torch.Tensor, b: torch.Tensor, trace=None, orchestrate=True):
        stream = torch.cuda.current_stream(self.device)
        mb.gemm_allreduce(a, b, self.out, workspace=None, events=self.events,
                          problem=self.problem, stream=stream, device=self.device, trace=trace,
                          orchestrate=orchestrate)
        mb.events_status(self.events, stream)
        return self.out

    def event_words(self) -> np.ndarray:
        return self.events[64:].cpu().numpy().view(np.uint32).copy()


def trace_records(trace: torch.Tensor):
    rec = trace.view(-1, 4).cpu().numpy().astype(np.uint64)
    rec = rec[rec[:, 3] != 0]
    kind = (rec[:, 0] & 0xFF).astype(np.int64)
    sub = ((rec[:, 0] >> 8) & 0xFF).astype(np.int64)
    cta = ((rec[:, 0] >> 16) & 0xFFFF).astype(np.int64)
    ticket = (rec[:, 0] >> 32).astype(np.int64)
    return dict(kind=kind, sub=sub, cta=cta, ticket=ticket, tile=rec[:, 1].astype(np.int64),
                t0=rec[:, 2], t1=rec[:, 3])


def same_process_team(devices, heap=1 << 30):
    """Teams for PEs on `devices`, one process driving them all (handles
    exchanged in-process)."""
    n = len(devices)
    handles = [None] * n
    teams = []
    import ctypes
    from megacu_b200 import _capi
    lib = _capi.load()
    raw = []
    for pe, dev in enumerate(devices):
        h = ctypes.c_void_p()
        mb.check(lib.megacu_b200_team_create(pe, n, dev, heap, ctypes.byref(h)))
        buf = ctypes.create_string_buffer(_capi.TEAM_HANDLE_BYTES)
        mb.check(lib.megacu_b200_team_export(h.value, buf))
        raw.append(h.value)
        handles[pe] = buf.raw
    blob = ctypes.create_string_buffer(b"".join(handles), n * _capi.TEAM_HANDLE_BYTES)
    for pe, dev in enumerate(devices):
        mb.check(lib.megacu_b200_team_connect(raw[pe], blob))
        t = mb.Team.__new__(mb.Team)
        t.my_pe, t.n_pes, t.device, t.handle = pe, n, dev, raw[pe]
        base, size = ctypes.c_void_p(), ctypes.c_int64()
        mb.check(lib.megacu_b200_team_info(raw[pe], None, None, ctypes.byref(base),
                                           ctypes.byref(size)))
        t.heap_base, t.heap_bytes = base.value, size.value
        t.multicast, t.multicast_error = False, None  # as a Team built without a region
        teams.append(t)
    return teams
