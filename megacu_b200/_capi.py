"""ctypes binding of the C ABI declared in include/megacu_b200.h.

The structures below are byte-for-byte the C structs of that header (which
are themselves the layout of megacu's C++ types). Loading fails loudly when
the native library has not been built: there is no Python fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

from .build import CHECKED_LIB_PATH, LIB_PATH, ROOT

c_int32, c_int64, c_uint8, c_uint16, c_uint64 = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint8,
                                                 ctypes.c_uint16, ctypes.c_uint64)
c_void_p = ctypes.c_void_p

HEADER_PATH = os.path.join(ROOT, "include", "megacu_b200.h")
TEAM_HANDLE_BYTES = 128

# status codes (megacu::status_code)
OK, INVALID_ARGUMENT, UNSUPPORTED, BACKEND_ERROR, LAUNCH_ERROR = range(5)
STATUS_NAMES = ["ok", "invalid_argument", "unsupported", "backend_error", "launch_error"]
MODE_ALLREDUCE, MODE_REDUCE_SCATTER, MODE_ALLGATHER = 0, 1, 2
ALGO_AUTO, ALGO_ONE_SHOT, ALGO_TWO_SHOT = 0, 1, 2
CTA_PAIRS_AUTO, CTA_PAIRS_OFF, CTA_PAIRS_ON = 0, 1, 2
DTYPE_BF16 = 2


class Status(ctypes.Structure):
    _fields_ = [("code", c_uint8), ("detail", c_uint16), ("message", ctypes.c_char_p)]

    def __repr__(self) -> str:
        msg = self.message.decode() if self.message else ""
        return f"Status({STATUS_NAMES[self.code]}, detail={self.detail}, {msg!r})"


class LaunchView(ctypes.Structure):
    _fields_ = [("stream", c_void_p), ("device_ordinal", c_int32)]


class TeamView(ctypes.Structure):
    _fields_ = [("team", c_void_p), ("team_my_pe", c_int32), ("team_n_pes", c_int32),
                ("world_my_pe", c_int32), ("world_n_pes", c_int32),
                ("cuda_device_ordinal", c_int32), ("backend", c_uint16), ("session", c_uint64),
                ("owner", c_uint8)]


class DriverView(ctypes.Structure):
    _fields_ = [("launch", LaunchView), ("team", TeamView)]


class GemmArProblem(ctypes.Structure):
    _fields_ = [("m", c_int64), ("n", c_int64), ("k", c_int64), ("tile_m", c_int32),
                ("tile_n", c_int32)]


class GemmArProblemV2(ctypes.Structure):
    _fields_ = [("m", c_int64), ("n", c_int64), ("k", c_int64), ("tile_m", c_int32),
                ("tile_n", c_int32), ("mode", c_int32), ("algo", c_int32),
                ("deterministic", c_int32), ("dtype", c_int32), ("num_ctas", c_int32),
                ("cta_pairs", c_int32), ("timeout_ns", c_uint64), ("trace", c_void_p),
                ("trace_capacity", c_int64)]


class MlpChainProblem(ctypes.Structure):
    _fields_ = [("tokens", c_int64), ("hidden", c_int64), ("inter", c_int64),
                ("layers", c_int32), ("algo", c_int32), ("deterministic", c_int32),
                ("num_ctas", c_int32), ("cta_pairs", c_int32), ("single_launch", c_int32),
                ("timeout_ns", c_uint64)]


_PROTOTYPES = {
    # name: (restype, argtypes)
    "megacu_cuda_gemm_swiglu_bf16":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblemV2]),
    "megacu_b200_swiglu_events_bytes": (Status, [GemmArProblemV2, ctypes.POINTER(c_int64)]),
    "megacu_b200_mlp_chain_sizes":
        (Status, [MlpChainProblem, c_int32, ctypes.POINTER(c_int64)]),
    "megacu_cuda_mlp_chain_bf16":
        (Status, [DriverView, c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p),
                  ctypes.POINTER(c_void_p), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                  c_void_p, MlpChainProblem]),
    "megacu_cuda_gemm_allreduce_phased_f32":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblem]),
    "megacu_cuda_gemm_allreduce_f32_orchestrate":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblem]),
    "megacu_cuda_gemm_allreduce_f32_co_resident":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                  GemmArProblem]),
    "megacu_b200_co_resident_control_bytes": (Status, [ctypes.POINTER(c_int64)]),
    "megacu_b200_co_resident_status": (Status, [c_void_p, c_void_p, ctypes.POINTER(c_int64)]),
    "megacu_cuda_gemm_allreduce_bf16":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblemV2]),
    "megacu_cuda_gemm_reduce_scatter_bf16":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblemV2]),
    "megacu_cuda_allgather_gemm_bf16":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblemV2]),
    "megacu_cuda_gemm_allreduce_bf16_orchestrate":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, GemmArProblemV2]),
    "megacu_cuda_gemm_bf16_noalloc":
        (Status, [DriverView, c_void_p, c_void_p, c_void_p, GemmArProblemV2]),
    "megacu_b200_noalloc_scratch":
        (Status, [c_int32, ctypes.POINTER(c_void_p), ctypes.POINTER(c_int64)]),
    "megacu_b200_workspace_bytes":
        (Status, [GemmArProblemV2, c_int32, ctypes.POINTER(c_int64)]),
    "megacu_b200_events_bytes": (Status, [GemmArProblemV2, c_int32, ctypes.POINTER(c_int64)]),
    "megacu_b200_plan_info": (Status, [GemmArProblemV2, c_int32, ctypes.POINTER(c_int32)]),
    "megacu_b200_plan_tile":
        (Status, [GemmArProblemV2, c_int32, c_int32, ctypes.POINTER(c_int32)]),
    "megacu_b200_plan_tile_on":
        (Status, [GemmArProblemV2, c_int32, c_int32, c_int32, ctypes.POINTER(c_int32)]),
    "megacu_b200_plan_pair":
        (Status, [GemmArProblemV2, c_int32, c_int32, ctypes.POINTER(c_int32)]),
    "megacu_b200_events_status": (Status, [c_void_p, c_void_p, ctypes.POINTER(c_int64)]),
    "megacu_b200_events_counters": (Status, [c_void_p, c_void_p, ctypes.POINTER(c_uint64)]),
    "megacu_b200_team_create":
        (Status, [c_int32, c_int32, c_int32, c_int64, ctypes.POINTER(c_void_p)]),
    "megacu_b200_team_export": (Status, [c_void_p, c_void_p]),
    "megacu_b200_team_connect": (Status, [c_void_p, c_void_p]),
    "megacu_b200_team_malloc": (Status, [c_void_p, c_int64, ctypes.POINTER(c_void_p)]),
    "megacu_b200_team_info":
        (Status, [c_void_p, ctypes.POINTER(c_int32), ctypes.POINTER(c_int32),
                  ctypes.POINTER(c_void_p), ctypes.POINTER(c_int64)]),
    "megacu_b200_team_barrier": (Status, [c_void_p, c_void_p]),
    "megacu_b200_team_destroy": (Status, [c_void_p]),
    "megacu_b200_exchange_local":
        (Status, [ctypes.c_char_p, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_int64]),
    "megacu_b200_team_create_local":
        (Status, [ctypes.c_char_p, c_int32, c_int32, c_int32, c_int64, c_int64,
                  ctypes.POINTER(c_void_p)]),
    "megacu_b200_team_multicast_export": (Status, [c_void_p, c_int64, c_void_p]),
    "megacu_b200_team_multicast_connect": (Status, [c_void_p, c_void_p]),
    "megacu_b200_team_multicast_malloc": (Status, [c_void_p, c_int64, ctypes.POINTER(c_void_p)]),
    "megacu_b200_team_multicast_info":
        (Status, [c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_int64)]),
    "megacu_dispatcher_explicit_attrs_component": (ctypes.c_int, []),
    "megacu_scheduler_explicit_asap_component": (ctypes.c_int, []),
    "megacu_platform_cuda_component": (ctypes.c_int, []),
    "megacu_backend_nvshmem_component": (ctypes.c_int, []),
    "megacu_target_runtime_component": (ctypes.c_int, []),
    "megacu_b200_version": (ctypes.c_char_p, []),
}

_lib = None


def library_path() -> str:
    """libmegacu_b200.so, or its bounds-checked build when
    MEGACU_B200_LIBRARY=checked."""
    return CHECKED_LIB_PATH if os.environ.get("MEGACU_B200_LIBRARY") == "checked" else LIB_PATH


def load(path: str | None = None) -> ctypes.CDLL:
    """Loads the native library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or library_path()
    if not os.path.exists(path):
        raise ImportError(
            f"megacu_b200 native library missing at {path}: run "
            "`python -m megacu_b200.build` (nvcc, sm_100a) — there is no fallback path")
    lib = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
    for name, (res, args) in _PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declared_functions(header: str = HEADER_PATH) -> list[str]:
    """Names of every function include/megacu_b200.h declares."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(megacu_\w+)\s*\(", text)))
