// Multicast (NVLS) region of a team: the memory behind the in-switch
// reduction of the two-shot allreduce.
//
// Set-up, collective over the team (one process per PE):
//   1. export: every PE creates its physical memory; PE 0 also creates the
//      multicast object, exports it as a file descriptor and serves that
//      descriptor on an abstract unix socket (SCM_RIGHTS), whose name goes
//      into PE 0's handle blob;
//   2. the caller exchanges the blobs (as for megacu_b200_team_connect);
//   3. connect: the other PEs fetch the descriptor and import the object;
//      every PE adds its device; a team barrier (all devices added before any
//      memory is bound); every PE binds its memory and maps it twice, once
//      plain (unicast) and once through the multicast object; the memory is
//      zeroed; a second team barrier (nobody reaches a peer before it is
//      bound).
// The driver API is resolved at run time (cudaGetDriverEntryPoint), so the
// library does not link libcuda.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <random>

#include <megacu_b200.h>

#include "team.h"

namespace megacu_b200 {
namespace {

constexpr std::uint32_t kMulticastMagic = 0x6d636d63u;
constexpr int kSocketTimeoutMs = 60000;

struct multicast_blob {
  std::uint32_t magic;
  std::int32_t pe;
  std::int32_t n_pes;
  std::int32_t device;
  std::uint64_t pid;
  std::int64_t bytes;
  char socket_name[64];
};
static_assert(sizeof(multicast_blob) <= MEGACU_B200_TEAM_HANDLE_BYTES, "multicast blob");

struct driver_api {
  PFN_cuDeviceGet_v2000 device_get = nullptr;
  PFN_cuDeviceGetAttribute_v2000 device_attribute = nullptr;
  PFN_cuMulticastGetGranularity_v12010 mc_granularity = nullptr;
  PFN_cuMulticastCreate_v12010 mc_create = nullptr;
  PFN_cuMulticastAddDevice_v12010 mc_add_device = nullptr;
  PFN_cuMulticastBindMem_v12010 mc_bind = nullptr;
  PFN_cuMulticastUnbind_v12010 mc_unbind = nullptr;
  PFN_cuMemCreate_v10020 mem_create = nullptr;
  PFN_cuMemRelease_v10020 mem_release = nullptr;
  PFN_cuMemAddressReserve_v10020 va_reserve = nullptr;
  PFN_cuMemAddressFree_v10020 va_free = nullptr;
  PFN_cuMemMap_v10020 map = nullptr;
  PFN_cuMemUnmap_v10020 unmap = nullptr;
  PFN_cuMemSetAccess_v10020 set_access = nullptr;
  PFN_cuMemExportToShareableHandle_v10020 export_handle = nullptr;
  PFN_cuMemImportFromShareableHandle_v10020 import_handle = nullptr;
  bool ok = false;
};

template <class Fn>
bool resolve(char const *name, Fn &fn) {
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr) {
    return false;
  }
  fn = reinterpret_cast<Fn>(p);
  return true;
}

driver_api const &api() {
  static driver_api d;
  static std::once_flag once;
  std::call_once(once, [] {
    d.ok = resolve("cuDeviceGet", d.device_get) &&
           resolve("cuDeviceGetAttribute", d.device_attribute) &&
           resolve("cuMulticastGetGranularity", d.mc_granularity) &&
           resolve("cuMulticastCreate", d.mc_create) &&
           resolve("cuMulticastAddDevice", d.mc_add_device) &&
           resolve("cuMulticastBindMem", d.mc_bind) &&
           resolve("cuMulticastUnbind", d.mc_unbind) && resolve("cuMemCreate", d.mem_create) &&
           resolve("cuMemRelease", d.mem_release) &&
           resolve("cuMemAddressReserve", d.va_reserve) &&
           resolve("cuMemAddressFree", d.va_free) && resolve("cuMemMap", d.map) &&
           resolve("cuMemUnmap", d.unmap) && resolve("cuMemSetAccess", d.set_access) &&
           resolve("cuMemExportToShareableHandle", d.export_handle) &&
           resolve("cuMemImportFromShareableHandle", d.import_handle);
  });
  return d;
}

megacu_status ok_status() { return {MEGACU_OK, 0, nullptr}; }

megacu_status fail(megacu_status_code code, std::uint16_t detail, char const *msg) {
  return {static_cast<std::uint8_t>(code), detail, msg};
}

// The message names the failed call and its CUresult; it lives in a
// per-thread buffer (never freed; the thread's next failure overwrites it).
megacu_status driver_fail(std::uint16_t detail, char const *call, CUresult r) {
  static thread_local char message[160];
  std::snprintf(message, sizeof(message), "%s failed (CUresult %d) in the multicast set-up", call,
                static_cast<int>(r));
  return fail(MEGACU_BACKEND_ERROR, detail, message);
}

// ---- the file descriptor hand-over ---------------------------------------------

bool abstract_address(char const *name, sockaddr_un &addr, socklen_t &len) {
  std::memset(&addr, 0, sizeof(addr));
  addr.sun_family = AF_UNIX;
  std::size_t const n = std::strlen(name);
  if (n == 0 || n + 1 > sizeof(addr.sun_path)) return false;
  std::memcpy(addr.sun_path + 1, name, n);  // sun_path[0] = 0: abstract namespace
  len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
  return true;
}

// PE 0: hands `fd` to `clients` connections; gives up at the deadline (the
// peers then report a failed fetch).
void serve_descriptor(int listen_fd, int fd, int clients) {
  auto const deadline =
      std::chrono::steady_clock::now() + std::chrono::milliseconds(kSocketTimeoutMs);
  for (int served = 0; served < clients;) {
    auto const left = std::chrono::duration_cast<std::chrono::milliseconds>(
        deadline - std::chrono::steady_clock::now());
    if (left.count() <= 0) return;
    pollfd pfd{listen_fd, POLLIN, 0};
    if (poll(&pfd, 1, static_cast<int>(left.count())) <= 0) return;
    int const c = accept(listen_fd, nullptr, nullptr);
    if (c < 0) continue;
    char byte = 'm';
    iovec iov{&byte, 1};
    alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int))] = {};
    msghdr msg{};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    msg.msg_control = control;
    msg.msg_controllen = sizeof(control);
    cmsghdr *cm = CMSG_FIRSTHDR(&msg);
    cm->cmsg_level = SOL_SOCKET;
    cm->cmsg_type = SCM_RIGHTS;
    cm->cmsg_len = CMSG_LEN(sizeof(int));
    std::memcpy(CMSG_DATA(cm), &fd, sizeof(int));
    if (sendmsg(c, &msg, 0) == 1) ++served;
    close(c);
  }
}

// Other PEs: fetch the descriptor from PE 0's socket; -1 on failure.
int fetch_descriptor(char const *name) {
  sockaddr_un addr;
  socklen_t len;
  if (!abstract_address(name, addr, len)) return -1;
  auto const deadline =
      std::chrono::steady_clock::now() + std::chrono::milliseconds(kSocketTimeoutMs);
  int s = -1;
  for (;;) {
    s = socket(AF_UNIX, SOCK_STREAM, 0);
    if (s < 0) return -1;
    if (connect(s, reinterpret_cast<sockaddr *>(&addr), len) == 0) break;
    close(s);
    s = -1;
    if (std::chrono::steady_clock::now() > deadline) return -1;
    usleep(10000);
  }
  pollfd pfd{s, POLLIN, 0};
  if (poll(&pfd, 1, kSocketTimeoutMs) <= 0) {
    close(s);
    return -1;
  }
  char byte = 0;
  iovec iov{&byte, 1};
  alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int))] = {};
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = control;
  msg.msg_controllen = sizeof(control);
  int fd = -1;
  if (recvmsg(s, &msg, 0) == 1) {
    cmsghdr *cm = CMSG_FIRSTHDR(&msg);
    if (cm != nullptr && cm->cmsg_level == SOL_SOCKET && cm->cmsg_type == SCM_RIGHTS) {
      std::memcpy(&fd, CMSG_DATA(cm), sizeof(int));
    }
  }
  close(s);
  return fd;
}

// Team barrier run to completion on a private stream; fails if a PE did not
// arrive within the barrier's bound.
megacu_status barrier_now(team_impl *t) {
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return fail(MEGACU_BACKEND_ERROR, 12, cudaGetErrorString(e));
  megacu_status st = megacu_b200_team_barrier(t, s);
  e = cudaStreamSynchronize(s);
  cudaStreamDestroy(s);
  if (st.code != MEGACU_OK) return st;
  if (e != cudaSuccess) return fail(MEGACU_BACKEND_ERROR, 12, cudaGetErrorString(e));
  std::uint32_t word = 0;
  auto *flag = reinterpret_cast<std::uint32_t *>(t->heap) + 32;
  e = cudaMemcpy(&word, flag, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(MEGACU_BACKEND_ERROR, 12, cudaGetErrorString(e));
  if (word != 0) {
    cudaMemset(flag, 0, sizeof(word));
    return fail(MEGACU_BACKEND_ERROR, 12, "a PE did not reach the team barrier in time");
  }
  return ok_status();
}

CUmulticastObjectProp object_prop(team_impl const *t, std::int64_t bytes) {
  CUmulticastObjectProp prop{};
  prop.numDevices = static_cast<unsigned int>(t->n_pes);
  prop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  prop.size = static_cast<std::size_t>(bytes);
  return prop;
}

}  // namespace

void release_multicast(team_impl *t) {
  multicast_region &r = t->mc;
  driver_api const &d = api();
  cudaSetDevice(t->device);
  cudaDeviceSynchronize();
  if (r.ready && t->n_pes > 1) {
    barrier_now(t);  // bounded; a missing PE only delays the release
  }
  if (d.ok) {
    auto const bytes = static_cast<std::size_t>(r.bytes);
    if (r.multi_mapped) d.unmap(reinterpret_cast<CUdeviceptr>(r.multi), bytes);
    if (r.multi != nullptr) d.va_free(reinterpret_cast<CUdeviceptr>(r.multi), bytes);
    if (r.local_mapped) d.unmap(reinterpret_cast<CUdeviceptr>(r.local), bytes);
    if (r.local != nullptr) d.va_free(reinterpret_cast<CUdeviceptr>(r.local), bytes);
    if (r.bound) {
      CUdevice dev;
      if (d.device_get(&dev, t->device) == CUDA_SUCCESS) d.mc_unbind(r.object, dev, 0, bytes);
    }
    if (r.have_memory) d.mem_release(r.memory);
    if (r.have_object) d.mem_release(r.object);
  }
  if (r.server.joinable()) r.server.join();
  if (r.export_fd >= 0) close(r.export_fd);
  if (r.listen_fd >= 0) close(r.listen_fd);
  r.ready = r.bound = r.have_memory = r.have_object = false;
  r.local_mapped = r.multi_mapped = false;
  r.local = r.multi = nullptr;
  r.export_fd = r.listen_fd = -1;
  r.bytes = r.used = r.granularity = 0;
}

}  // namespace megacu_b200

using namespace megacu_b200;

extern "C" megacu_status megacu_b200_team_multicast_export(void *team, std::int64_t bytes,
                                                           void *handle) {
  team_impl *t = as_team(team);
  if (t == nullptr || handle == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  if (!t->connected) return fail(MEGACU_INVALID_ARGUMENT, 24, "team is not connected");
  if (t->n_pes < 2) return fail(MEGACU_UNSUPPORTED, 35, "a multicast region needs 2 or more PEs");
  if (bytes <= 0) return fail(MEGACU_INVALID_ARGUMENT, 1, "invalid multicast region size");
  multicast_region &r = t->mc;
  if (r.have_memory || r.have_object || r.ready) {
    return fail(MEGACU_INVALID_ARGUMENT, 36, "the team already has a multicast region");
  }
  driver_api const &d = api();
  if (!d.ok) return fail(MEGACU_UNSUPPORTED, 35, "CUDA driver without multicast objects");
  cudaError_t e = cudaSetDevice(t->device);
  if (e == cudaSuccess) e = cudaFree(nullptr);  // the device's primary context is current
  if (e != cudaSuccess) return fail(MEGACU_LAUNCH_ERROR, 10, cudaGetErrorString(e));
  CUdevice dev;
  CUresult res = d.device_get(&dev, t->device);
  if (res != CUDA_SUCCESS) return driver_fail(37, "cuDeviceGet", res);
  int supported = 0;
  if (d.device_attribute(&supported, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev) !=
          CUDA_SUCCESS ||
      !supported) {
    return fail(MEGACU_UNSUPPORTED, 35, "this device does not support multicast objects");
  }
  CUmulticastObjectProp prop = object_prop(t, bytes);
  std::size_t granularity = 0;
  res = d.mc_granularity(&granularity, &prop, CU_MULTICAST_GRANULARITY_RECOMMENDED);
  if (res != CUDA_SUCCESS || granularity == 0) {
    return driver_fail(37, "cuMulticastGetGranularity", res);
  }
  std::int64_t const size =
      (bytes + static_cast<std::int64_t>(granularity) - 1) / granularity * granularity;
  prop.size = static_cast<std::size_t>(size);

  CUmemAllocationProp mp{};
  mp.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  mp.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  mp.location.id = t->device;
  mp.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  CUmemGenericAllocationHandle memory;
  res = d.mem_create(&memory, static_cast<std::size_t>(size), &mp, 0);
  if (res != CUDA_SUCCESS) return driver_fail(37, "cuMemCreate", res);
  r.memory = memory;
  r.have_memory = true;
  r.bytes = size;
  r.granularity = static_cast<std::int64_t>(granularity);

  multicast_blob blob{};
  blob.magic = kMulticastMagic;
  blob.pe = t->my_pe;
  blob.n_pes = t->n_pes;
  blob.device = t->device;
  blob.pid = static_cast<std::uint64_t>(getpid());
  blob.bytes = size;
  if (t->my_pe == 0) {
    CUmemGenericAllocationHandle object;
    res = d.mc_create(&object, &prop);
    if (res != CUDA_SUCCESS) {
      release_multicast(t);
      return driver_fail(37, "cuMulticastCreate", res);
    }
    r.object = object;
    r.have_object = true;
    int fd = -1;
    res = d.export_handle(&fd, object, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
    if (res != CUDA_SUCCESS || fd < 0) {
      release_multicast(t);
      return driver_fail(38, "cuMemExportToShareableHandle", res);
    }
    r.export_fd = fd;
    std::random_device rd;
    std::snprintf(r.socket_name, sizeof(r.socket_name), "megacu_b200.mc.%llu.%08x%08x",
                  static_cast<unsigned long long>(getpid()), rd(), rd());
    sockaddr_un addr;
    socklen_t len;
    int const s = socket(AF_UNIX, SOCK_STREAM, 0);
    if (s < 0 || !abstract_address(r.socket_name, addr, len) ||
        bind(s, reinterpret_cast<sockaddr *>(&addr), len) != 0 || listen(s, t->n_pes) != 0) {
      if (s >= 0) close(s);
      release_multicast(t);
      return fail(MEGACU_BACKEND_ERROR, 38, "cannot open the multicast hand-over socket");
    }
    r.listen_fd = s;
    r.server = std::thread(serve_descriptor, s, fd, t->n_pes - 1);
    std::memcpy(blob.socket_name, r.socket_name, sizeof(blob.socket_name));
  }
  std::memset(handle, 0, MEGACU_B200_TEAM_HANDLE_BYTES);
  std::memcpy(handle, &blob, sizeof(blob));
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_multicast_connect(void *team, void const *handles) {
  team_impl *t = as_team(team);
  if (t == nullptr || handles == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  multicast_region &r = t->mc;
  if (r.ready) return ok_status();
  if (!r.have_memory) {
    return fail(MEGACU_INVALID_ARGUMENT, 36, "call megacu_b200_team_multicast_export first");
  }
  driver_api const &d = api();
  auto const *bytes = static_cast<unsigned char const *>(handles);
  multicast_blob first{};
  for (int pe = 0; pe < t->n_pes; ++pe) {
    multicast_blob blob;
    std::memcpy(&blob, bytes + pe * MEGACU_B200_TEAM_HANDLE_BYTES, sizeof(blob));
    if (blob.magic != kMulticastMagic || blob.pe != pe || blob.n_pes != t->n_pes ||
        blob.bytes != r.bytes) {
      release_multicast(t);
      return fail(MEGACU_INVALID_ARGUMENT, 32, "multicast handle does not match this team");
    }
    for (int q = 0; q < pe; ++q) {
      multicast_blob other;
      std::memcpy(&other, bytes + q * MEGACU_B200_TEAM_HANDLE_BYTES, sizeof(other));
      if (other.pid == blob.pid) {
        release_multicast(t);
        return fail(MEGACU_UNSUPPORTED, 35, "a multicast region needs one process per PE");
      }
    }
    if (pe == 0) first = blob;
  }
  cudaError_t e = cudaSetDevice(t->device);
  if (e != cudaSuccess) {
    release_multicast(t);
    return fail(MEGACU_LAUNCH_ERROR, 10, cudaGetErrorString(e));
  }
  if (t->my_pe != 0) {
    first.socket_name[sizeof(first.socket_name) - 1] = 0;
    int const fd = fetch_descriptor(first.socket_name);
    if (fd < 0) {
      release_multicast(t);
      return fail(MEGACU_BACKEND_ERROR, 38, "cannot fetch the multicast object from PE 0");
    }
    CUmemGenericAllocationHandle object;
    CUresult const res = d.import_handle(
        &object, reinterpret_cast<void *>(static_cast<std::intptr_t>(fd)),
        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    close(fd);
    if (res != CUDA_SUCCESS) {
      release_multicast(t);
      return driver_fail(38, "cuMemImportFromShareableHandle", res);
    }
    r.object = object;
    r.have_object = true;
  }
  CUdevice dev;
  CUresult res = d.device_get(&dev, t->device);
  if (res == CUDA_SUCCESS) res = d.mc_add_device(r.object, dev);
  if (res != CUDA_SUCCESS) {
    release_multicast(t);
    return driver_fail(37, "cuMulticastAddDevice", res);
  }
  // Every device must be added before any memory is bound.
  megacu_status st = barrier_now(t);
  if (st.code != MEGACU_OK) {
    release_multicast(t);
    return st;
  }
  auto const size = static_cast<std::size_t>(r.bytes);
  res = d.mc_bind(r.object, 0, r.memory, 0, size, 0);
  if (res != CUDA_SUCCESS) {
    release_multicast(t);
    return driver_fail(37, "cuMulticastBindMem", res);
  }
  r.bound = true;
  CUmemAccessDesc access{};
  access.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  access.location.id = t->device;
  access.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  CUdeviceptr local = 0, multi = 0;
  auto const align = static_cast<std::size_t>(r.granularity);
  char const *step = "cuMemAddressReserve";
  res = d.va_reserve(&local, size, align, 0, 0);
  if (res == CUDA_SUCCESS) {
    r.local = reinterpret_cast<char *>(local);
    step = "cuMemMap";
    res = d.map(local, size, 0, r.memory, 0);
  }
  if (res == CUDA_SUCCESS) {
    r.local_mapped = true;
    step = "cuMemSetAccess";
    res = d.set_access(local, size, &access, 1);
  }
  if (res == CUDA_SUCCESS) {
    step = "cuMemAddressReserve (multicast)";
    res = d.va_reserve(&multi, size, align, 0, 0);
  }
  if (res == CUDA_SUCCESS) {
    r.multi = reinterpret_cast<char *>(multi);
    step = "cuMemMap (multicast)";
    res = d.map(multi, size, 0, r.object, 0);
  }
  if (res == CUDA_SUCCESS) {
    r.multi_mapped = true;
    step = "cuMemSetAccess (multicast)";
    res = d.set_access(multi, size, &access, 1);
  }
  if (res != CUDA_SUCCESS) {
    release_multicast(t);
    return driver_fail(37, step, res);
  }
  e = cudaMemset(r.local, 0, size);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    release_multicast(t);
    return fail(MEGACU_LAUNCH_ERROR, 11, cudaGetErrorString(e));
  }
  // Nobody reaches a peer's memory through the object before it is bound.
  st = barrier_now(t);
  if (st.code != MEGACU_OK) {
    release_multicast(t);
    return st;
  }
  if (r.server.joinable()) r.server.join();
  if (r.export_fd >= 0) {
    close(r.export_fd);
    r.export_fd = -1;
  }
  if (r.listen_fd >= 0) {
    close(r.listen_fd);
    r.listen_fd = -1;
  }
  r.used = 0;
  r.ready = true;
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_multicast_malloc(void *team, std::int64_t bytes,
                                                           void **ptr) {
  team_impl *t = as_team(team);
  if (t == nullptr || ptr == nullptr || bytes < 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  }
  std::lock_guard<std::mutex> lock(t->mu);
  multicast_region &r = t->mc;
  if (!r.ready) return fail(MEGACU_INVALID_ARGUMENT, 36, "the team has no multicast region");
  std::int64_t const size = (bytes + 255) / 256 * 256;
  if (r.used + size > r.bytes) {
    return fail(MEGACU_INVALID_ARGUMENT, 34, "multicast region exhausted");
  }
  *ptr = r.local + r.used;
  r.used += size;
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_multicast_info(void *team, void **base,
                                                         std::int64_t *bytes) {
  team_impl *t = as_team(team);
  if (t == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  if (base) *base = t->mc.ready ? t->mc.local : nullptr;
  if (bytes) *bytes = t->mc.ready ? t->mc.bytes : 0;
  return ok_status();
}
