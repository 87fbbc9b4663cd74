// GEMM + allreduce workload ABI (C++ side).
//
// Interface parity with megacu
// `examples/cuda_nvshmem/gemm_allreduce/common/gemm_allreduce.h:8-41`: the
// operator names, `gemm_ar_driver`, `gemm_ar_problem` and the orchestrate
// entry `cuda_nvshmem_gemm_allreduce_phased_orchestrate` (fp32, C++ linkage).
// Added for B200: the bf16 orchestrate entry with `megacu_gemm_ar_problem_v2`
// (one-shot / two-shot allreduce, reduce-scatter, fp32-wire deterministic
// mode), declared in megacu_b200.h.
#pragma once

#include <cstdint>

#include <megacu/runtime.h>
#include <megacu/views.h>
#include <megacu_b200.h>

namespace ops {

struct gemm_tile_produce {
  static constexpr auto name = "gemm_tile_produce";
};

struct allreduce_tile_consume {
  static constexpr auto name = "allreduce_tile_consume";
};

struct phased_megakernel {
  static constexpr auto name = "phased_megakernel";
};

}  // namespace ops

using gemm_ar_driver = megacu::cuda_nvshmem::driver_view;

struct gemm_ar_problem {
  std::int64_t m = 0;
  std::int64_t n = 0;
  std::int64_t k = 0;
  std::int32_t tile_m = 0;
  std::int32_t tile_n = 0;
};

// Builds megacu's three-task phase for the fp32 problem and runs it through
// `megacu_cuda_gemm_allreduce_phased_f32`.
megacu::status cuda_nvshmem_gemm_allreduce_phased_orchestrate(gemm_ar_driver driver,
                                                              float const *a, float const *b,
                                                              float *partial, float *out,
                                                              void *events,
                                                              gemm_ar_problem problem);
