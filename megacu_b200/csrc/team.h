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
#include <thread>

#include <megacu/backends/nvshmem.h>

namespace megacu_b200 {

inline constexpr std::uint32_t kTeamMagic = 0x6d636274u;
// The first bytes of every heap are reserved for host-driven team barriers.
inline constexpr std::int64_t kTeamReservedBytes = 4096;

// Optional multicast (NVLS) region: this PE's own device memory bound to a
// multicast object that every PE of the team bound its memory to. A store
// through `multi` (multimem.st) reaches every PE's copy; a multimem.ld_reduce
// through it returns the sum over all PEs' copies, reduced in the NVSwitch.
// Allocations are symmetric (same offset on every PE), like the heap's.
struct multicast_region {
  bool ready = false;                // bound and mapped on every PE
  std::int64_t bytes = 0;            // a multiple of the multicast granularity
  std::int64_t granularity = 0;
  std::int64_t used = 0;
  unsigned long long object = 0;     // the multicast object (CUmemGenericAllocationHandle)
  unsigned long long memory = 0;     // this PE's physical memory bound to it
  char *local = nullptr;             // unicast mapping of this PE's memory
  char *multi = nullptr;             // multicast mapping (multimem.* only)
  bool have_object = false, have_memory = false, bound = false;
  bool local_mapped = false, multi_mapped = false;
  int export_fd = -1;                // PE 0: the object's shareable file descriptor
  int listen_fd = -1;                // PE 0: socket that hands export_fd to the peers
  std::thread server;                // PE 0: serves export_fd during set-up
  char socket_name[64] = {};

  bool contains(void const *p, std::int64_t n) const {
    auto const *c = static_cast<char const *>(p);
    return ready && c >= local && n >= 0 && c + n <= local + bytes;
  }
  // The multicast address of a pointer into this PE's region.
  char *alias(void const *p) const { return multi + (static_cast<char const *>(p) - local); }
};

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
  multicast_region mc;
  std::mutex mu;

  bool contains(void const *p, std::int64_t bytes) const {
    auto const *c = static_cast<char const *>(p);
    return c >= heap && bytes >= 0 && c + bytes <= heap + heap_bytes;
  }
};

// Releases the multicast region (multicast.cu). Collective when the region
// is ready: it first meets every PE at a team barrier, so no PE unbinds its
// memory while another may still reach it through the multicast object.
void release_multicast(team_impl *t);

inline team_impl *as_team(void *handle) {
  auto *t = static_cast<team_impl *>(handle);
  return (t != nullptr && t->magic == kTeamMagic) ? t : nullptr;
}

}  // namespace megacu_b200
