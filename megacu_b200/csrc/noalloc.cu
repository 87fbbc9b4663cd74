// Allocation-free entry point of the single-PE bf16 megakernel.
//
// Some callers cannot allocate device memory for us: a plugin host that
// hands an operator only its input and output buffers (the host owns every
// byte of device memory and exposes no workspace), a process whose device
// memory is entirely managed by another allocator, or a latency-critical
// serving loop where a cudaMalloc call (which may synchronise the device) is
// not acceptable. For them, `megacu_cuda_gemm_bf16_noalloc` runs the same
// kernel as `megacu_cuda_gemm_allreduce_bf16` on one PE, with the kernel's
// scratch (the control block with the device task-queue tickets, and the
// event tensor) in a fixed array compiled into this library.
//
// Limits and sharing rules:
//  * scratch is `kNoAllocScratchBytes` (256 KiB) per GPU, held by every GPU
//    that loads the library until the process exits; problems whose tile
//    grid needs more (more than 8183 output tiles) are rejected;
//  * every call on a GPU shares that one array: calls that overlap on the
//    GPU (on different streams, or from different threads) race and must
//    not be issued; calls in stream order are fine;
//  * each call clears the array's queue tickets and its error word before
//    the kernel runs, so an error (a timed-out wait, or a failed bounds
//    check in the checked build) is reported for the call that met it and
//    never stops a later call; `megacu_b200_noalloc_scratch` gives the
//    array's device address, which `megacu_b200_events_status` (the last
//    call's error, read and cleared) and `megacu_b200_events_counters`
//    (completion counters summed over every call on the GPU, errors
//    included) accept like any events buffer;
//  * the first call on a device (and the first after that device's context
//    was reset) looks up the array's device address with that device
//    current; make that first call before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include <megacu_b200.h>

#include "kernels/gemm_ar_kernel.cuh"
#include "kernels/launch.cuh"
#include "tma_map.h"

namespace {

using namespace megacu_b200;

constexpr std::int64_t kNoAllocScratchBytes = 256 * 1024;
constexpr int kNoAllocMaxDevices = 64;

// The scratch itself. In host code this name is only a handle for the
// runtime: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
// Per device: the array's address and the id of the context it was looked up
// in. A device reset (cudaDeviceReset, or another library resetting the
// primary context) reloads this module and may move the array, so the
// address is looked up again whenever the current context's id differs.
void *g_noalloc_addr[kNoAllocMaxDevices] = {};
unsigned long long g_noalloc_ctx[kNoAllocMaxDevices] = {};

megacu_status na_ok() { return {MEGACU_OK, 0, nullptr}; }

megacu_status na_fail(megacu_status_code code, std::uint16_t detail, char const *msg) {
  return {static_cast<std::uint8_t>(code), detail, msg};
}

megacu_status na_cuda(cudaError_t e, std::uint16_t detail) {
  return {MEGACU_LAUNCH_ERROR, detail, cudaGetErrorString(e)};
}

// Unique id of the calling thread's current context (0 if the driver cannot
// say). Resolved through cudaGetDriverEntryPoint, so the library does not
// link libcuda.
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
    }
    ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(ptr);
    }
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of this GPU's scratch, with `device` current: looked up
// once per device and context (every call when the context id is unknown).
megacu_status scratch_address(int device, void **out) {
  if (device < 0 || device >= kNoAllocMaxDevices) {
    return na_fail(MEGACU_INVALID_ARGUMENT, 10, "device ordinal out of range");
  }
  // Since CUDA 12.0 cudaSetDevice also initialises the device's primary
  // context and makes it current, so its id can be asked for right after.
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return na_cuda(e, 10);
  unsigned long long const ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[device] == nullptr || ctx == 0 || g_noalloc_ctx[device] != ctx) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return na_cuda(e, 50);
    g_noalloc_addr[device] = ptr;
    g_noalloc_ctx[device] = ctx;
  }
  *out = g_noalloc_addr[device];
  return na_ok();
}

}  // namespace

extern "C" megacu_status megacu_cuda_gemm_bf16_noalloc(megacu_driver_view driver, void const *a,
                                                       void const *b, void *out,
                                                       megacu_gemm_ar_problem_v2 problem) {
  if (driver.team.team_n_pes != 1) {
    return na_fail(MEGACU_UNSUPPORTED, 51,
                   "the allocation-free entry runs on one PE only (team_n_pes must be 1)");
  }
  problem.mode = MEGACU_MODE_ALLREDUCE;
  std::int32_t info[10];
  megacu_status st = megacu_b200_plan_info(problem, 1, info);
  if (st.code != MEGACU_OK) return st;
  if (a == nullptr || b == nullptr || out == nullptr) {
    return na_fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  auto aligned = [](void const *p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; };
  if (!aligned(a) || !aligned(b) || !aligned(out)) {
    return na_fail(MEGACU_INVALID_ARGUMENT, 21, "buffers must be 16-byte aligned");
  }
  std::int32_t const tile_n = info[1], m_tiles = info[2], n_tiles = info[3];
  std::int64_t const tiles = static_cast<std::int64_t>(m_tiles) * n_tiles;
  if (events_bytes_for(1, static_cast<std::int32_t>(tiles)) > kNoAllocScratchBytes) {
    return na_fail(MEGACU_INVALID_ARGUMENT, 52,
                   "problem too large for the allocation-free entry: its tile grid needs more "
                   "than the 256 KiB of built-in scratch (at most 8183 output tiles)");
  }
  if (driver.launch.stream == nullptr) {
    return na_ok();
  }
  int const device = driver.launch.device_ordinal;
  void *scratch = nullptr;
  st = scratch_address(device, &scratch);  // also makes `device` current
  if (st.code != MEGACU_OK) return st;

  CUtensorMap map_a, map_b;
  if (!encode_bf16_map(&map_a, a, problem.m, problem.k, kBlockM) ||
      !encode_bf16_map(&map_b, b, problem.k, problem.n, kBlockK)) {
    return na_fail(MEGACU_BACKEND_ERROR, 30, "cuTensorMapEncodeTiled failed");
  }
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);
  // The array keeps whatever the previous call left. The queue tickets and
  // the CTA count must start at zero, and so must the error word and its
  // info (the kernel abandons its waits once the error word is set): clear
  // both ranges. The launch counter between them stays, since every flag is
  // tagged with the epoch it gives.
  static_assert(offsetof(control_block, gemm_ticket) == 0 &&
                    offsetof(control_block, done_ctas) == 8 &&
                    offsetof(control_block, launch_count) == 12 &&
                    offsetof(control_block, error_code) == 16 &&
                    offsetof(control_block, error_info) == 20,
                "control block words cleared per call");
  cudaError_t e = cudaMemsetAsync(scratch, 0, 3 * sizeof(std::uint32_t), stream);
  if (e != cudaSuccess) return na_cuda(e, 11);
  e = cudaMemsetAsync(static_cast<unsigned char *>(scratch) + offsetof(control_block, error_code),
                      0, 4 * sizeof(std::uint32_t), stream);
  if (e != cudaSuccess) return na_cuda(e, 11);

  gemm_ar_params prm{};
  prm.m = static_cast<std::int32_t>(problem.m);
  prm.n = static_cast<std::int32_t>(problem.n);
  prm.k = static_cast<std::int32_t>(problem.k);
  prm.m_tiles = m_tiles;
  prm.n_tiles = n_tiles;
  prm.tiles = static_cast<std::int32_t>(tiles);
  prm.n_pes = 1;
  prm.my_pe = 0;
  prm.mode = mode_allreduce;
  prm.group_m = info[6];
  prm.comm_warps = kWorkerWarps;  // unused with one PE
  prm.rows_per_pe = prm.m;
  prm.timeout_ns = problem.timeout_ns != 0 ? problem.timeout_ns : 10000000000ull;
  prm.out = static_cast<__nv_bfloat16 *>(out);
  prm.events = static_cast<std::uint32_t *>(scratch);
  prm.peers.n_pes = 1;
  prm.trace = reinterpret_cast<unsigned long long *>(problem.trace);
  prm.trace_capacity = problem.trace != nullptr ? problem.trace_capacity : 0;

  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return na_cuda(e, 10);
  int const grid = problem.num_ctas > 0 ? problem.num_ctas : sms;
  e = launch_bf16_plan(false, tile_n, info[8] != 0, device, grid, stream, map_a, map_b, prm);
  if (e != cudaSuccess) return na_cuda(e, 14);
  return na_ok();
}

extern "C" megacu_status megacu_b200_noalloc_scratch(std::int32_t device, void **events,
                                                    std::int64_t *bytes) {
  if (events == nullptr) return na_fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  void *scratch = nullptr;
  megacu_status const st = scratch_address(device, &scratch);
  if (st.code != MEGACU_OK) return st;
  *events = scratch;
  if (bytes != nullptr) *bytes = kNoAllocScratchBytes;
  return na_ok();
}
