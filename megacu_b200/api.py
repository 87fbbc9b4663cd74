"""Python host mirror of megacu's GEMM + allreduce entry points.

Thin wrappers over the C ABI (``include/megacu_b200.h``): torch tensors are
only device-memory holders here, every byte of work runs in
``libmegacu_b200.so``. Names and argument meaning follow megacu:

* :func:`cuda_nvshmem_gemm_allreduce_phased_orchestrate` — megacu's fp32
  orchestrate entry (phased/megacu/gemm_allreduce_phased_orchestrate.cc:3-20);
* :func:`megacu_cuda_gemm_allreduce_phased_f32` — its native launcher
  (megacu_gemm_allreduce_phased.cu:157-232);
* :func:`gemm_allreduce` / :func:`gemm_reduce_scatter` — the bf16 fused
  megakernel (B200 path), orchestrated through the same phase API;
* :class:`Team` — the symmetric heap that replaces NVSHMEM's.

Errors come back as :class:`MegacuError` carrying megacu's status code and
per-site detail number.
"""
from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

from . import _capi
from ._capi import DriverView, GemmArProblem, GemmArProblemV2, Status


class MegacuError(RuntimeError):
    def __init__(self, status: Status):
        self.code = int(status.code)
        self.detail = int(status.detail)
        self.message = status.message.decode() if status.message else ""
        super().__init__(f"megacu {_capi.STATUS_NAMES[self.code]} (detail {self.detail}): "
                         f"{self.message}")


def check(status: Status) -> Status:
    if status.code != _capi.OK:
        raise MegacuError(status)
    return status


def lib() -> ctypes.CDLL:
    return _capi.load()


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream, named explicitly


def _stream_handle(stream) -> Optional[int]:
    """Raw cudaStream_t of ``stream``. None stays None (megacu: validate only);
    torch's default stream (handle 0) is passed as cudaStreamLegacy so that it
    is not mistaken for "no stream"."""
    if stream is None:
        return None
    handle = stream if isinstance(stream, int) else stream.cuda_stream
    return handle if handle != 0 else CUDA_STREAM_LEGACY


# ---- team ----------------------------------------------------------------------

class Team:
    """This PE's symmetric heap, mapped by every peer of the team.

    ``exchange`` maps this PE's handle (bytes) to the list of every PE's
    handle in PE order — e.g. :func:`torch_exchange` over torch.distributed.
    Every PE must create the team and allocate from it in the same order
    (as with ``nvshmem_init`` / ``nvshmem_malloc``).

    ``multicast_bytes > 0`` also sets up a multicast (NVLS) region of at least
    that size (one process per PE; rounded up to the multicast granularity).
    Where the device, driver or team shape cannot have one, the team works
    without it (``self.multicast`` is False); every PE reaches the same
    decision, since all see every PE's set-up blob.
    """

    def __init__(self, my_pe: int, n_pes: int, device: int, heap_bytes: int,
                 exchange: Optional[Callable[[bytes], Sequence[bytes]]] = None,
                 multicast_bytes: int = 0):
        self.my_pe, self.n_pes, self.device = my_pe, n_pes, device
        handle = ctypes.c_void_p()
        check(lib().megacu_b200_team_create(my_pe, n_pes, device, heap_bytes,
                                            ctypes.byref(handle)))
        self.handle = handle.value
        # A team still open when the interpreter exits (an exception on the
        # way) is destroyed then: a process must not end with its memory bound
        # to a multicast object while the other PEs still use it.
        self._finalizer = weakref.finalize(self, _destroy_team, self.handle)
        if n_pes > 1:
            if exchange is None:
                raise ValueError("a team of more than one PE needs an exchange function")
            mine = ctypes.create_string_buffer(_capi.TEAM_HANDLE_BYTES)
            check(lib().megacu_b200_team_export(self.handle, mine))
            handles = list(exchange(mine.raw))
            if len(handles) != n_pes or any(len(h) != _capi.TEAM_HANDLE_BYTES for h in handles):
                raise ValueError("exchange must return one 128-byte handle per PE")
            blob = ctypes.create_string_buffer(b"".join(handles), n_pes * _capi.TEAM_HANDLE_BYTES)
            check(lib().megacu_b200_team_connect(self.handle, blob))
        base = ctypes.c_void_p()
        size = ctypes.c_int64()
        check(lib().megacu_b200_team_info(self.handle, None, None, ctypes.byref(base),
                                          ctypes.byref(size)))
        self.heap_base, self.heap_bytes = base.value, size.value
        self.multicast = False
        self.multicast_error = None
        if multicast_bytes > 0 and n_pes > 1:
            self._connect_multicast(multicast_bytes, exchange)

    def _connect_multicast(self, nbytes: int, exchange) -> None:
        mine = ctypes.create_string_buffer(_capi.TEAM_HANDLE_BYTES)
        st = lib().megacu_b200_team_multicast_export(self.handle, nbytes, mine)
        if st.code != _capi.OK:
            self.multicast_error = MegacuError(st)
        handles = list(exchange(mine.raw if st.code == _capi.OK else
                                bytes(_capi.TEAM_HANDLE_BYTES)))
        # A PE that could not export sends zeros: then nobody connects.
        if any(not any(h[:4]) for h in handles):
            if self.multicast_error is None:
                self.multicast_error = RuntimeError("a peer cannot set up a multicast region")
            return
        blob = ctypes.create_string_buffer(b"".join(handles), self.n_pes * _capi.TEAM_HANDLE_BYTES)
        st = lib().megacu_b200_team_multicast_connect(self.handle, blob)
        if st.code != _capi.OK:
            self.multicast_error = MegacuError(st)
            return
        base = ctypes.c_void_p()
        size = ctypes.c_int64()
        check(lib().megacu_b200_team_multicast_info(self.handle, ctypes.byref(base),
                                                    ctypes.byref(size)))
        self.multicast = size.value > 0
        self.multicast_base, self.multicast_bytes = base.value, size.value

    def malloc(self, nbytes: int) -> int:
        ptr = ctypes.c_void_p()
        check(lib().megacu_b200_team_malloc(self.handle, nbytes, ctypes.byref(ptr)))
        return ptr.value

    def multicast_malloc(self, nbytes: int) -> int:
        ptr = ctypes.c_void_p()
        check(lib().megacu_b200_team_multicast_malloc(self.handle, nbytes, ctypes.byref(ptr)))
        return ptr.value

    def tensor(self, shape, dtype, multicast: bool = False):
        """A torch tensor over a fresh symmetric allocation (zero-filled), in
        the heap or, with ``multicast=True``, in the multicast region."""
        import torch
        numel = 1
        for s in shape:
            numel *= s
        itemsize = torch.empty((), dtype=dtype).element_size()
        nbytes = max(numel * itemsize, 16)
        ptr = self.multicast_malloc(nbytes) if multicast else self.malloc(nbytes)
        return tensor_from_pointer(ptr, shape, dtype, self.device, owner=self)

    def barrier(self, stream=None) -> None:
        check(lib().megacu_b200_team_barrier(self.handle, _stream_handle(stream)))

    def close(self) -> None:
        """Destroys the team; collective when it has a multicast region."""
        if self.handle is not None:
            finalizer = getattr(self, "_finalizer", None)
            if finalizer is not None:
                finalizer.detach()
            check(lib().megacu_b200_team_destroy(self.handle))
            self.handle = None

    def __enter__(self) -> "Team":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def view(self) -> _capi.TeamView:
        return _capi.TeamView(team=self.handle, team_my_pe=self.my_pe, team_n_pes=self.n_pes,
                              world_my_pe=self.my_pe, world_n_pes=self.n_pes,
                              cuda_device_ordinal=self.device)


def _destroy_team(handle) -> None:
    lib().megacu_b200_team_destroy(handle)


def torch_exchange(group=None) -> Callable[[bytes], Sequence[bytes]]:
    """Handle exchange over torch.distributed (any backend; gloo works)."""
    import torch.distributed as dist

    def exchange(mine: bytes) -> Sequence[bytes]:
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, mine, group=group)
        return out

    return exchange


def local_exchange(session: str, my_pe: int, n_pes: int,
                   timeout_ms: int = 60_000) -> Callable[[bytes], Sequence[bytes]]:
    """Handle exchange among the processes of one node without
    torch.distributed: every PE passes the same ``session`` string
    (megacu_b200_exchange_local, an abstract unix socket served by PE 0).
    Each call of the returned function is one collective exchange."""
    name = session.encode()

    def exchange(mine: bytes) -> Sequence[bytes]:
        size = len(mine)
        out = ctypes.create_string_buffer(size * n_pes)
        check(lib().megacu_b200_exchange_local(name, my_pe, n_pes, mine, size, out, timeout_ms))
        raw = out.raw
        return [raw[i * size:(i + 1) * size] for i in range(n_pes)]

    return exchange


def env_team(heap_bytes: int, multicast_bytes: int = 0, timeout_ms: int = 60_000) -> "Team":
    """A team of the processes torchrun (or any launcher setting LOCAL_RANK /
    LOCAL_WORLD_SIZE) started on this node, one per GPU, PE = local rank,
    built without torch.distributed. The session is MEGACU_B200_SESSION if
    set, else derived from MASTER_ADDR, MASTER_PORT and TORCHELASTIC_RUN_ID."""
    import os
    env = os.environ
    my_pe = int(env.get("LOCAL_RANK", env.get("RANK", "0")))
    n_pes = int(env.get("LOCAL_WORLD_SIZE", env.get("WORLD_SIZE", "1")))
    session = env.get("MEGACU_B200_SESSION") or "{}.{}.{}".format(
        env.get("MASTER_ADDR", "local"), env.get("MASTER_PORT", "0"),
        env.get("TORCHELASTIC_RUN_ID", "none"))
    return Team(my_pe, n_pes, my_pe, heap_bytes,
                local_exchange(session[:64], my_pe, n_pes, timeout_ms) if n_pes > 1 else None,
                multicast_bytes=multicast_bytes)


class _CudaArray:
    def __init__(self, ptr, shape, typestr, owner):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}
        self._owner = owner


def tensor_from_pointer(ptr: int, shape, dtype, device: int, owner=None):
    """Wraps device memory at ``ptr`` as a torch tensor (no copy, no ownership)."""
    import torch
    codes = {torch.bfloat16: ("<i2", torch.bfloat16), torch.float16: ("<f2", None),
             torch.float32: ("<f4", None), torch.int32: ("<i4", None),
             torch.uint8: ("|u1", None), torch.int64: ("<i8", None)}
    typestr, view_as = codes[dtype]
    with torch.cuda.device(device):
        t = torch.as_tensor(_CudaArray(ptr, shape, typestr, owner), device=f"cuda:{device}")
    return t.view(view_as) if view_as is not None else t


# ---- driver views ------------------------------------------------------------------

_VIEWS: dict = {}  # (stream handle, device) -> DriverView of a one-PE call


def _launch_view(stream, device: int, team: Optional[Team]) -> DriverView:
    """driver_view() for the launch wrappers below, built once per (stream,
    device) and team: the struct is passed by value, so the cached object is
    never changed by a call. (driver_view itself returns a fresh struct, which
    callers may modify.)"""
    key = (_stream_handle(stream), device)
    cache = _VIEWS if team is None else team.__dict__.setdefault("_views", {})
    d = cache.get(key)
    if d is None:
        d = cache[key] = driver_view(stream, device, team)
    return d


def driver_view(stream=None, device: int = 0, team: Optional[Team] = None) -> DriverView:
    """megacu's driver_view{launch_view, team_view} for this PE."""
    d = DriverView()
    d.launch.stream = _stream_handle(stream)
    d.launch.device_ordinal = device
    if team is not None:
        d.team = team.view()
    else:
        d.team.team_my_pe, d.team.team_n_pes = 0, 1
        d.team.world_my_pe, d.team.world_n_pes = 0, 1
        d.team.cuda_device_ordinal = device
    return d


# ---- bf16 fused megakernel ---------------------------------------------------------

@dataclass
class Problem:
    """megacu_gemm_ar_problem_v2: out[m, n] = sum over PEs of a[m, k] @ b[k, n]."""
    m: int
    n: int
    k: int
    mode: int = _capi.MODE_ALLREDUCE
    algo: int = _capi.ALGO_AUTO
    deterministic: bool = False
    tile_n: int = 0
    num_ctas: int = 0
    timeout_ns: int = 0
    cta_pairs: int = _capi.CTA_PAIRS_AUTO

    def __setattr__(self, name, value):
        object.__setattr__(self, name, value)
        self.__dict__.pop("_c", None)  # a changed field rebuilds the C struct

    def to_c(self, trace_ptr: Optional[int] = None, trace_capacity: int = 0) -> GemmArProblemV2:
        """The C struct (passed by value). Without a trace it is built once and
        reused until a field changes."""
        if trace_ptr is None and trace_capacity == 0:
            c = self.__dict__.get("_c")
            if c is not None:
                return c
        c = GemmArProblemV2(m=self.m, n=self.n, k=self.k, tile_m=0, tile_n=self.tile_n,
                            mode=self.mode, algo=self.algo,
                            deterministic=1 if self.deterministic else 0,
                            dtype=_capi.DTYPE_BF16, num_ctas=self.num_ctas,
                            cta_pairs=self.cta_pairs,
                            timeout_ns=self.timeout_ns, trace=trace_ptr,
                            trace_capacity=trace_capacity)
        if trace_ptr is None and trace_capacity == 0:
            self.__dict__["_c"] = c
        return c


def workspace_bytes(problem: Problem, n_pes: int) -> int:
    out = ctypes.c_int64()
    check(lib().megacu_b200_workspace_bytes(problem.to_c(), n_pes, ctypes.byref(out)))
    return out.value


def events_bytes(problem: Problem, n_pes: int) -> int:
    out = ctypes.c_int64()
    check(lib().megacu_b200_events_bytes(problem.to_c(), n_pes, ctypes.byref(out)))
    return out.value


@dataclass
class Plan:
    tile_m: int
    tile_n: int
    m_tiles: int
    n_tiles: int
    one_shot: bool
    slots_per_src: int
    group_m: int
    wire_bytes: int
    cta_pairs: bool = False  # 2-CTA clusters compute 256-row pair tiles
    gemm_units: int = 0      # GEMM tickets per call

    @property
    def tiles(self) -> int:
        return self.m_tiles * self.n_tiles


def plan(problem: Problem, n_pes: int) -> Plan:
    info = (ctypes.c_int32 * 10)()
    check(lib().megacu_b200_plan_info(problem.to_c(), n_pes, info))
    return Plan(info[0], info[1], info[2], info[3], bool(info[4]), info[5], info[6], info[7],
                bool(info[8]), info[9])


def plan_tile(problem: Problem, n_pes: int, r: int, pe: int = 0) -> tuple[int, int, int, int]:
    """(tile_row, tile_col, owner, local index) of raster index ``r`` on PE
    ``pe`` (the all-gather raster starts with the PE's own shard; the other
    modes' rasters are the same on every PE)."""
    out = (ctypes.c_int32 * 4)()
    check(lib().megacu_b200_plan_tile_on(problem.to_c(), n_pes, pe, r, out))
    return tuple(out)


def plan_pair(problem: Problem, n_pes: int, q: int) -> tuple[int, int]:
    """Raster indices of the two tiles a CTA pair computes for GEMM ticket ``q``."""
    out = (ctypes.c_int32 * 2)()
    check(lib().megacu_b200_plan_pair(problem.to_c(), n_pes, q, out))
    return tuple(out)


def gemm_allreduce(a, b, out, *, workspace, events, problem: Problem, stream=None,
                   device: int = 0, team: Optional[Team] = None, trace=None,
                   orchestrate: bool = True) -> None:
    """Launches the fused bf16 GEMM + allreduce / reduce-scatter (async).

    ``orchestrate=True`` goes through megacu's phase API (dispatcher +
    scheduler validation, then the launcher), as megacu's orchestrate entry
    does; ``False`` calls the launcher directly.
    """
    trace_ptr = _ptr(trace)
    cap = trace.numel() // 4 if trace is not None else 0
    d = _launch_view(stream, device, team)
    p = problem.to_c(trace_ptr, cap)
    args = (d, _ptr(a), _ptr(b), _ptr(workspace), _ptr(out), _ptr(events), p)
    if orchestrate:
        check(lib().megacu_cuda_gemm_allreduce_bf16_orchestrate(*args))
    elif problem.mode == _capi.MODE_REDUCE_SCATTER:
        check(lib().megacu_cuda_gemm_reduce_scatter_bf16(*args))
    else:
        check(lib().megacu_cuda_gemm_allreduce_bf16(*args))


def gemm_reduce_scatter(a, b, out, *, workspace, events, problem: Problem, **kw) -> None:
    problem.mode = _capi.MODE_REDUCE_SCATTER
    gemm_allreduce(a, b, out, workspace=workspace, events=events, problem=problem, **kw)


def allgather_gemm(a_shard, b, gathered, out, *, events, problem: Problem, stream=None,
                   device: int = 0, team: Optional[Team] = None, trace=None) -> None:
    """Launches the all-gather + GEMM (async): ``gathered`` [m, k] receives
    every PE's ``a_shard`` [m / tp, k] in PE order and ``out`` [m, n] =
    gathered @ b. ``a_shard`` and ``events`` lie in the team's heap when the
    team has more than one PE; ``problem.mode`` is set to MODE_ALLGATHER."""
    problem.mode = _capi.MODE_ALLGATHER
    trace_ptr = _ptr(trace)
    cap = trace.numel() // 4 if trace is not None else 0
    d = _launch_view(stream, device, team)
    check(lib().megacu_cuda_allgather_gemm_bf16(d, _ptr(a_shard), _ptr(b), _ptr(gathered),
                                                 _ptr(out), _ptr(events),
                                                 problem.to_c(trace_ptr, cap)))


# ---- tensor-parallel MLP blocks (benchmark config 5) ----------------------------------

def swiglu_events_bytes(problem: Problem) -> int:
    out = ctypes.c_int64()
    check(lib().megacu_b200_swiglu_events_bytes(problem.to_c(), ctypes.byref(out)))
    return out.value


def gemm_swiglu(x, w_gate, w_up, act, *, events, problem: Problem, stream=None,
                device: int = 0, trace=None) -> None:
    """act = silu(x @ w_gate) * (x @ w_up) (one PE, async). ``problem``: m =
    tokens, n = act columns, k = hidden."""
    trace_ptr = _ptr(trace)
    cap = trace.numel() // 4 if trace is not None else 0
    check(lib().megacu_cuda_gemm_swiglu_bf16(_launch_view(stream, device, None), _ptr(x),
                                             _ptr(w_gate), _ptr(w_up), _ptr(act), _ptr(events),
                                             problem.to_c(trace_ptr, cap)))


@dataclass
class MlpChainProblem:
    """megacu_mlp_chain_problem: ``layers`` blocks x -> allreduce(swiglu(x) @ w_down)."""
    tokens: int
    hidden: int
    inter: int          # this PE's slice of the intermediate size
    layers: int = 1
    algo: int = _capi.ALGO_AUTO
    deterministic: bool = False
    num_ctas: int = 0
    cta_pairs: int = _capi.CTA_PAIRS_AUTO
    timeout_ns: int = 0
    single_launch: bool = False  # all blocks (at most 6) in one persistent launch

    def to_c(self) -> "_capi.MlpChainProblem":
        return _capi.MlpChainProblem(tokens=self.tokens, hidden=self.hidden, inter=self.inter,
                                     layers=self.layers, algo=self.algo,
                                     deterministic=1 if self.deterministic else 0,
                                     num_ctas=self.num_ctas, cta_pairs=self.cta_pairs,
                                     single_launch=1 if self.single_launch else 0,
                                     timeout_ns=self.timeout_ns)


def mlp_chain_sizes(problem: MlpChainProblem, n_pes: int) -> dict:
    """Bytes of each buffer megacu_cuda_mlp_chain_bf16 needs on ``n_pes`` PEs."""
    out = (ctypes.c_int64 * 5)()
    check(lib().megacu_b200_mlp_chain_sizes(problem.to_c(), n_pes, out))
    return {"act": out[0], "workspace": out[1], "events_swiglu": out[2],
            "events_down": out[3], "x_work": out[4]}


def mlp_chain(x, w_gate, w_up, w_down, out, *, act, workspace, x_work, events_swiglu,
              events_down, problem: MlpChainProblem, stream=None, device: int = 0,
              team: Optional[Team] = None) -> None:
    """Runs ``problem.layers`` tensor-parallel MLP blocks (async); the last
    block's output lands in ``out``. ``w_gate``, ``w_up``, ``w_down``: one
    tensor per layer (this PE's slices)."""
    n = problem.layers
    if not (len(w_gate) == len(w_up) == len(w_down) == n):
        raise ValueError("one gate, up and down weight per layer")
    arr = lambda ws: (ctypes.c_void_p * n)(*[_ptr(w) for w in ws])
    check(lib().megacu_cuda_mlp_chain_bf16(_launch_view(stream, device, team), _ptr(x),
                                           arr(w_gate), arr(w_up), arr(w_down), _ptr(act),
                                           _ptr(workspace), _ptr(x_work), _ptr(out),
                                           _ptr(events_swiglu), _ptr(events_down),
                                           problem.to_c()))


def events_status(events, stream=None) -> list[int]:
    """Synchronises ``stream`` and raises MegacuError if a device wait failed."""
    info = (ctypes.c_int64 * 4)()
    check(lib().megacu_b200_events_status(_ptr(events), _stream_handle(stream), info))
    return list(info)


def events_counters(events, stream=None) -> list[int]:
    out = (ctypes.c_uint64 * 8)()
    check(lib().megacu_b200_events_counters(_ptr(events), _stream_handle(stream), out))
    return list(out)


# ---- megacu's fp32 phased entry points -------------------------------------------------

def megacu_cuda_gemm_allreduce_phased_f32(driver: DriverView, a, b, partial, out, events,
                                          m: int, n: int, k: int, tile_m: int,
                                          tile_n: int) -> Status:
    return lib().megacu_cuda_gemm_allreduce_phased_f32(
        driver, _ptr(a), _ptr(b), _ptr(partial), _ptr(out), _ptr(events),
        GemmArProblem(m=m, n=n, k=k, tile_m=tile_m, tile_n=tile_n))


def cuda_nvshmem_gemm_allreduce_phased_orchestrate(driver: DriverView, a, b, partial, out,
                                                   events, m: int, n: int, k: int,
                                                   tile_m: int, tile_n: int) -> Status:
    return lib().megacu_cuda_gemm_allreduce_f32_orchestrate(
        driver, _ptr(a), _ptr(b), _ptr(partial), _ptr(out), _ptr(events),
        GemmArProblem(m=m, n=n, k=k, tile_m=tile_m, tile_n=tile_n))


def co_resident_control_bytes() -> int:
    out = ctypes.c_int64()
    check(lib().megacu_b200_co_resident_control_bytes(ctypes.byref(out)))
    return out.value


def megacu_cuda_gemm_allreduce_f32_co_resident(driver: DriverView, a, b, partial, out, events,
                                               control, m: int, n: int, k: int, tile_m: int,
                                               tile_n: int) -> Status:
    """megacu's fp32 phase with co-resident persistent progress (one
    cooperative persistent launch; ``control`` holds
    :func:`co_resident_control_bytes` bytes of device memory)."""
    return lib().megacu_cuda_gemm_allreduce_f32_co_resident(
        driver, _ptr(a), _ptr(b), _ptr(partial), _ptr(out), _ptr(events), _ptr(control),
        GemmArProblem(m=m, n=n, k=k, tile_m=tile_m, tile_n=tile_n))


def co_resident_status(control, stream=None) -> list[int]:
    """Synchronises ``stream``; raises MegacuError (detail 40) if a wait of the
    last co-resident launch gave up; returns [node, tile] of that wait."""
    info = (ctypes.c_int64 * 2)()
    check(lib().megacu_b200_co_resident_status(_ptr(control), _stream_handle(stream), info))
    return list(info)
