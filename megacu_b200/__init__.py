"""megacu_b200: B200-native (sm_100a) fused GEMM + allreduce / reduce-scatter.

The product is the native library ``lib/libmegacu_b200.so`` behind the C ABI
in ``include/megacu_b200.h``; this package is its Python host mirror (ctypes)
plus the in-tree build. Importing it does not need a GPU; calling a launcher
does, and fails loudly if the native library is missing.
"""
from .api import (MegacuError, MlpChainProblem, Plan, Problem, Team, allgather_gemm, check,
                  co_resident_control_bytes, co_resident_status, env_team, local_exchange,
                  megacu_cuda_gemm_allreduce_f32_co_resident,
                  cuda_nvshmem_gemm_allreduce_phased_orchestrate, gemm_swiglu, mlp_chain,
                  mlp_chain_sizes, swiglu_events_bytes,
                  driver_view, events_bytes, events_counters, events_status, gemm_allreduce,
                  gemm_reduce_scatter, megacu_cuda_gemm_allreduce_phased_f32, plan, plan_pair, plan_tile,
                  tensor_from_pointer, torch_exchange, workspace_bytes)
from ._capi import (ALGO_AUTO, ALGO_ONE_SHOT, ALGO_TWO_SHOT, CTA_PAIRS_AUTO, CTA_PAIRS_OFF,
                    CTA_PAIRS_ON, MODE_ALLGATHER, MODE_ALLREDUCE, MODE_REDUCE_SCATTER, load)

__all__ = [
    "MegacuError", "MlpChainProblem", "Plan", "Problem", "Team", "allgather_gemm", "check",
    "co_resident_control_bytes", "co_resident_status", "env_team", "local_exchange",
    "megacu_cuda_gemm_allreduce_f32_co_resident",
    "cuda_nvshmem_gemm_allreduce_phased_orchestrate", "gemm_swiglu", "mlp_chain", "mlp_chain_sizes",
    "swiglu_events_bytes",
    "driver_view", "events_bytes", "events_counters", "events_status", "gemm_allreduce",
    "gemm_reduce_scatter", "megacu_cuda_gemm_allreduce_phased_f32", "plan", "plan_pair", "plan_tile", "tensor_from_pointer",
    "torch_exchange", "workspace_bytes", "ALGO_AUTO", "ALGO_ONE_SHOT", "ALGO_TWO_SHOT",
    "CTA_PAIRS_AUTO", "CTA_PAIRS_OFF", "CTA_PAIRS_ON", "MODE_ALLGATHER", "MODE_ALLREDUCE", "MODE_REDUCE_SCATTER", "load",
]
