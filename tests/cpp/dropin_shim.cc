// Test infrastructure: a C-linkage handle on megacu's own orchestration
// (examples/cuda_nvshmem/gemm_allreduce/phased/megacu/
// gemm_allreduce_phased_orchestrate.cc), which oracle/Makefile compiles,
// unchanged, against this repository's headers and links with
// libmegacu_b200.so into oracle/_ref/libref_orchestrate_on_b200.so. Linked
// with -Bsymbolic, so the call below reaches that reference-compiled
// definition, not the library's own one.
#include <cstring>

#include <megacu/gemm_allreduce.h>
#include <megacu_b200.h>

extern "C" megacu_status dropin_orchestrate(megacu_driver_view driver, float const *a,
                                            float const *b, float *partial, float *out,
                                            void *events, megacu_gemm_ar_problem problem) {
  gemm_ar_driver d;
  std::memcpy(&d, &driver, sizeof(d));
  gemm_ar_problem p;
  std::memcpy(&p, &problem, sizeof(p));
  megacu::status st = cuda_nvshmem_gemm_allreduce_phased_orchestrate(d, a, b, partial, out,
                                                                     events, p);
  megacu_status out_status;
  std::memcpy(&out_status, &st, sizeof(out_status));
  return out_status;
}
