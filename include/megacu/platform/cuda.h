// CUDA platform: launch view plus the device-side readiness primitives the
// event tensors are built from.
//
// Interface parity with megacu `include/megacu/platform/cuda.h:13-55`:
// `launch_view{stream, device_ordinal}`, `has_stream`, and
// `device::{fence_system, load_ready, signal_ready, wait_ready}`.
//
// B200 differences (behavioural, not in the names):
//  * `signal_ready` is a system-scope release store and `load_ready` a
//    system-scope acquire load (`st.release.sys` / `ld.acquire.sys`), so a
//    flag written by a peer GPU over NVLink orders the data written before it.
//    The reference uses `__threadfence_system` + `atomicExch` / `atomicAdd(p,0)`.
//  * `wait_ready` is bounded: it gives up after `timeout_ns` of
//    `%globaltimer` time and returns false, so a missing peer can never hang
//    a shared GPU. The reference spins forever (cuda.h:49-55).
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define MEGACU_CUDA_HOST_DEVICE __host__ __device__
#else
#define MEGACU_CUDA_HOST_DEVICE
#endif

namespace megacu::cuda {

struct launch_view {
  void *stream = nullptr;
  std::int32_t device_ordinal = 0;
};

// True when the launch carries a stream. A null stream means "validate only".
bool has_stream(launch_view launch) noexcept;

namespace device {

// Default bound of a readiness wait: two seconds of GPU wall time.
inline constexpr std::uint64_t default_wait_timeout_ns = 2000000000ull;

MEGACU_CUDA_HOST_DEVICE inline void fence_system() {
#if defined(__CUDA_ARCH__)
  asm volatile("fence.acq_rel.sys;" ::: "memory");
#endif
}

MEGACU_CUDA_HOST_DEVICE inline std::uint64_t global_time_ns() {
#if defined(__CUDA_ARCH__)
  std::uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
#else
  return 0;
#endif
}

MEGACU_CUDA_HOST_DEVICE inline int load_ready(int const *events,
                                              std::int64_t index) {
#if defined(__CUDA_ARCH__)
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];"
               : "=r"(v)
               : "l"(events + index)
               : "memory");
  return v;
#else
  return events[index];
#endif
}

MEGACU_CUDA_HOST_DEVICE inline void signal_ready(int *events,
                                                 std::int64_t index,
                                                 int value) {
#if defined(__CUDA_ARCH__)
  asm volatile("st.release.sys.global.b32 [%0], %1;"
               :
               : "l"(events + index), "r"(value)
               : "memory");
#else
  events[index] = value;
#endif
}

// Spins until `events[index] == value` or `timeout_ns` elapses. Returns
// whether the value was seen. On the host (no GPU) this is a single check.
MEGACU_CUDA_HOST_DEVICE inline bool wait_ready(
    int const *events, std::int64_t index, int value,
    std::uint64_t timeout_ns = default_wait_timeout_ns) {
#if defined(__CUDA_ARCH__)
  if (load_ready(events, index) == value) {
    return true;
  }
  std::uint64_t const start = global_time_ns();
  for (std::uint32_t spin = 1;; ++spin) {
    if (load_ready(events, index) == value) {
      return true;
    }
    if ((spin & 63u) == 0 && global_time_ns() - start > timeout_ns) {
      return false;
    }
  }
#else
  (void)timeout_ns;
  return events[index] == value;
#endif
}

}  // namespace device

}  // namespace megacu::cuda

#undef MEGACU_CUDA_HOST_DEVICE
