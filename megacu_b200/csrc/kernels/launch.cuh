// Host-side launch of the megakernel variants: one CTA per SM, or 2-CTA
// clusters (CTA pairs) for the cta_group::2 GEMM.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "gemm_ar_kernel.cuh"

namespace megacu_b200 {

inline constexpr int kLaunchMaxDevices = 64;

// Persistent launch of `Kernel` (one CTA per SM, or 2-CTA clusters with
// kPair): sets its dynamic shared memory once per device and, for clusters,
// caps the grid at the pairs that fit on the device at once.
template <auto Kernel, bool kPair, int kSmem, class... Args>
cudaError_t launch_persistent(int device, int grid, cudaStream_t stream, Args const &...args) {
  // Per device, set once; host threads may race here harmlessly (the
  // attribute and the cluster count are the same whoever sets them).
  static std::atomic<bool> configured[kLaunchMaxDevices] = {};
  static std::atomic<int> max_pairs[kLaunchMaxDevices] = {};
  bool const known = device >= 0 && device < kLaunchMaxDevices;
  if (!known || !configured[device].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (known) configured[device].store(true, std::memory_order_release);
  }
  if constexpr (!kPair) {
    Kernel<<<grid, kThreads, kSmem, stream>>>(args...);
    return cudaGetLastError();
  } else {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int pairs = known ? max_pairs[device].load(std::memory_order_acquire) : 0;
    if (pairs == 0) {
      cfg.gridDim = dim3(2, 1, 1);
      cudaError_t e = cudaOccupancyMaxActiveClusters(&pairs, Kernel, &cfg);
      if (e != cudaSuccess) return e;
      if (pairs < 1) return cudaErrorInvalidConfiguration;
      if (known) max_pairs[device].store(pairs, std::memory_order_release);
    }
    int const g = std::max(2, std::min(grid / 2, pairs) * 2);
    cfg.gridDim = dim3(static_cast<unsigned>(g), 1, 1);
    return cudaLaunchKernelEx(&cfg, Kernel, args...);
  }
}

// K split (gemm_ar_params::k_split > 1, one CTA per tile otherwise): clusters
// of k_split CTAs, one cluster per GEMM tile. Falls back to one CTA per tile
// (k_split = 1 on the usual persistent grid) when the device cannot hold
// that many clusters at once, since a cluster computes one tile only.
template <auto Kernel, int kSmem>
cudaError_t launch_split(int device, int grid, cudaStream_t stream, CUtensorMap const &ma,
                         CUtensorMap const &mb, CUtensorMap const &mb2, gemm_ar_params prm) {
  static std::atomic<int> max_clusters[kLaunchMaxDevices][5] = {};
  bool const known = device >= 0 && device < kLaunchMaxDevices;
  int const ks = prm.k_split;
  cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = known ? max_clusters[device][ks].load(std::memory_order_acquire) : 0;
  if (clusters == 0) {
    cfg.gridDim = dim3(static_cast<unsigned>(ks), 1, 1);
    e = cudaOccupancyMaxActiveClusters(&clusters, Kernel, &cfg);
    if (e != cudaSuccess) return e;
    if (known) max_clusters[device][ks].store(clusters, std::memory_order_release);
  }
  if (clusters < prm.tiles) {
    prm.k_split = 1;
    return launch_persistent<Kernel, false, kSmem>(device, grid, stream, ma, mb, mb2, prm);
  }
  cfg.gridDim = dim3(static_cast<unsigned>(prm.tiles * ks), 1, 1);
  return cudaLaunchKernelEx(&cfg, Kernel, ma, mb, mb2, prm);
}

template <int BN, bool kWireF32, bool kPair, bool kSwiGLU = false, bool kGather = false>
cudaError_t launch_variant(int device, int grid, cudaStream_t stream, CUtensorMap const &ma,
                           CUtensorMap const &mb, CUtensorMap const &mb2,
                           gemm_ar_params const &prm) {
  constexpr auto kKernel = &gemm_ar_megakernel<BN, kWireF32, kPair, kSwiGLU, kGather>;
  constexpr int kSmem = gemm_config<BN, kPair>::smem_bytes;
  if constexpr (!kPair && !kSwiGLU && !kGather) {
    if (prm.k_split > 1) {
      return launch_split<kKernel, kSmem>(device, grid, stream, ma, mb, mb2, prm);
    }
  }
  return launch_persistent<kKernel, kPair, kSmem>(device, grid, stream, ma, mb, mb2, prm);
}

// Launches the variant a plan picked: tile_n 64 / 128 / 256, CTA pairs
// (tile_n >= 128 only) or not.
template <bool kWireF32>
cudaError_t launch_gemm_ar(int tile_n, bool pairs, int device, int grid, cudaStream_t stream,
                           CUtensorMap const &ma, CUtensorMap const &mb,
                           gemm_ar_params const &prm) {
  switch (tile_n) {
    case 256:
      return pairs ? launch_variant<256, kWireF32, true>(device, grid, stream, ma, mb, mb, prm)
                   : launch_variant<256, kWireF32, false>(device, grid, stream, ma, mb, mb, prm);
    case 128:
      return pairs ? launch_variant<128, kWireF32, true>(device, grid, stream, ma, mb, mb, prm)
                   : launch_variant<128, kWireF32, false>(device, grid, stream, ma, mb, mb, prm);
    default:
      return launch_variant<64, kWireF32, false>(device, grid, stream, ma, mb, mb, prm);
  }
}

// Launches of the bf16 plans, defined once in capi.cu (so that the kernel
// variants are compiled in one translation unit only).
cudaError_t launch_bf16_plan(bool wire_f32, int tile_n, bool pairs, int device, int grid,
                             cudaStream_t stream, CUtensorMap const &ma, CUtensorMap const &mb,
                             gemm_ar_params const &prm);

}  // namespace megacu_b200
