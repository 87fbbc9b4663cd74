// Team object behind `team_view.team`: this PE's symmetric heap plus the
// mapped heaps of its peers (CUDA IPC over NVLink / NVSwitch).
//
// It plays the role NVSHMEM plays for megacu (nvshmem_init / nvshmem_malloc
// / remote pointers, backends/nvshmem.h:19-64): a symmetric allocation has
// the same offset in every PE's heap, so a peer's copy is
// `peers.base[pe] + (ptr - heap)`.
#pragma once

#include <cstdint>
#include <mutex>

#include <megacu/backends/nvshmem.h>

namespace megacu_b200 {

inline constexpr std::uint32_t kTeamMagic = 0x6d636274u;
// The first bytes of every heap are reserved for host-driven team barriers.
inline constexpr std::int64_t kTeamReservedBytes = 4096;

struct team_impl {
  std::uint32_t magic = kTeamMagic;
  std::int32_t my_pe = 0;
  std::int32_t n_pes = 1;
  std::int32_t device = 0;
  char *heap = nullptr;
  std::int64_t heap_bytes = 0;
  std::int64_t used = kTeamReservedBytes;
  bool connected = false;
  bool opened[megacu::nvshmem::max_team_pes] = {};
  megacu::nvshmem::peer_table peers;
  std::uint32_t barrier_epoch = 0;  // team barriers issued so far
  std::mutex mu;

  bool contains(void const *p, std::int64_t bytes) const {
    auto const *c = static_cast<char const *>(p);
    return c >= heap && bytes >= 0 && c + bytes <= heap + heap_bytes;
  }
};

inline team_impl *as_team(void *handle) {
  auto *t = static_cast<team_impl *>(handle);
  return (t != nullptr && t->magic == kTeamMagic) ? t : nullptr;
}

}  // namespace megacu_b200
