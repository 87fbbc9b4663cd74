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
//  * the first call on a device looks up the array's device address (with
//    that device current); make that first call before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

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
void *g_noalloc_addr[kNoAllocMaxDevices] = {};

megacu_status na_ok() { return {MEGACU_OK, 0, nullptr}; }

megacu_status na_fail(megacu_status_code code, std::uint16_t detail, char const *msg) {
  return {static_cast<std::uint8_t>(code), detail, msg};
}

megacu_status na_cuda(cudaError_t e, std::uint16_t detail) {
  return {MEGACU_LAUNCH_ERROR, detail, cudaGetErrorString(e)};
}

// Device address of this GPU's scratch; looked up once per device with that
// device current.
megacu_status scratch_address(int device, void **out) {
  if (device < 0 || device >= kNoAllocMaxDevices) {
    return na_fail(MEGACU_INVALID_ARGUMENT, 10, "device ordinal out of range");
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[device] == nullptr) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return na_cuda(e, 50);
    g_noalloc_addr[device] = ptr;
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
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return na_cuda(e, 10);
  void *scratch = nullptr;
  st = scratch_address(device, &scratch);
  if (st.code != MEGACU_OK) return st;

  CUtensorMap map_a, map_b;
  if (!encode_bf16_map(&map_a, a, problem.m, problem.k, kBlockM) ||
      !encode_bf16_map(&map_b, b, problem.k, problem.n, kBlockK)) {
    return na_fail(MEGACU_BACKEND_ERROR, 30, "cuTensorMapEncodeTiled failed");
  }
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);
  // The device task-queue words must start at zero: clear them (the array
  // keeps whatever the previous call left).
  e = cudaMemsetAsync(scratch, 0, 3 * sizeof(std::uint32_t), stream);
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
