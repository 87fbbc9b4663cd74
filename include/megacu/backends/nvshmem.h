// Communication backend: team description plus device-side remote access.
//
// Interface parity with megacu `include/megacu/backends/nvshmem.h:19-64`:
// `ownership`, `team_view{team, team_my_pe, team_n_pes, world_my_pe,
// world_n_pes, cuda_device_ordinal, backend, session, owner}`, `team_size`,
// `has_remote_pes`, `device::remote_int`, `device::remote_float`.
//
// On B200 the backend is not NVSHMEM. It is a peer table over NVLink 5 /
// NVSwitch: every rank's symmetric heap is a plain `cudaMalloc` block that
// the other ranks map with CUDA IPC, so a symmetric address on rank `pe` is
// `peers.base[pe] + (ptr - peers.base[my_pe])`. `team_view.team` carries the
// `megacu_b200_team` handle (see megacu_b200.h) that owns that table. The
// three-argument `remote_*` forms keep the reference's single-rank behaviour
// (a local read); the four-argument forms take the peer table and issue a
// plain load from the peer's memory.
#pragma once

#include <cstdint>

#include <megacu/views.h>

#if defined(__CUDACC__)
#define MEGACU_NVSHMEM_HOST_DEVICE __host__ __device__
#else
#define MEGACU_NVSHMEM_HOST_DEVICE
#endif

namespace megacu::nvshmem {

enum class ownership : std::uint8_t { external, owned };

struct team_view {
  void *team = nullptr;
  std::int32_t team_my_pe = 0;
  std::int32_t team_n_pes = 1;
  std::int32_t world_my_pe = 0;
  std::int32_t world_n_pes = 1;
  std::int32_t cuda_device_ordinal = 0;
  megacu::backend_id backend;
  megacu::session_id session;
  ownership owner = ownership::external;
};

std::int32_t team_size(team_view team) noexcept;

bool has_remote_pes(team_view team) noexcept;

// Largest team one B200 node holds (8 GPUs on one NVSwitch fabric).
inline constexpr int max_team_pes = 8;

// Device view of every rank's symmetric heap base, indexed by team PE.
struct peer_table {
  char *base[max_team_pes] = {};
  std::int32_t my_pe = 0;
  std::int32_t n_pes = 1;

  template <class T>
  MEGACU_NVSHMEM_HOST_DEVICE T *translate(T const *local, int pe) const {
    auto offset = reinterpret_cast<char const *>(local) - base[my_pe];
    return reinterpret_cast<T *>(base[pe] + offset);
  }
};

namespace device {

MEGACU_NVSHMEM_HOST_DEVICE inline int remote_int(int const *value,
                                                 std::int64_t index, int pe) {
  (void)pe;
  return value[index];
}

MEGACU_NVSHMEM_HOST_DEVICE inline float remote_float(float const *value,
                                                     std::int64_t index,
                                                     int pe) {
  (void)pe;
  return value[index];
}

MEGACU_NVSHMEM_HOST_DEVICE inline int remote_int(int const *value,
                                                 std::int64_t index, int pe,
                                                 peer_table const &peers) {
  int const *remote = peers.translate(value, pe);
#if defined(__CUDA_ARCH__)
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];"
               : "=r"(v)
               : "l"(remote + index)
               : "memory");
  return v;
#else
  return remote[index];
#endif
}

MEGACU_NVSHMEM_HOST_DEVICE inline float remote_float(float const *value,
                                                     std::int64_t index,
                                                     int pe,
                                                     peer_table const &peers) {
  float const *remote = peers.translate(value, pe);
#if defined(__CUDA_ARCH__)
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(remote + index));
  return v;
#else
  return remote[index];
#endif
}

}  // namespace device

}  // namespace megacu::nvshmem

#undef MEGACU_NVSHMEM_HOST_DEVICE
