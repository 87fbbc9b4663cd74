// CUDA platform shell of the generic megakernel.
//
// Interface parity with megacu `include/megacu/platform/cuda/megakernel.cuh:
// 7-33` (device_context, launch_config, megakernel_entry, launch_megakernel).
// B200 addition: `launch_config::cooperative` launches through
// cudaLaunchCooperativeKernel, which guarantees every CTA is co-resident —
// required when CTAs of different GPUs wait on one another's tiles.
#pragma once

#include <cuda_runtime.h>

namespace megacu::platform::cuda {

struct device_context {
  __device__ int block_id() const { return blockIdx.x; }

  __device__ int grid_blocks() const { return gridDim.x; }

  __device__ int thread_id() const { return threadIdx.x; }

  __device__ int block_threads() const { return blockDim.x; }

  __device__ void sync_block() const { __syncthreads(); }
};

struct launch_config {
  int blocks = 1;
  int threads = 1;
  bool cooperative = false;
};

template <class Program>
__global__ void megakernel_entry(Program program) {
  program(device_context{});
}

template <class Program>
cudaError_t launch_megakernel(cudaStream_t stream, launch_config config, Program program) {
  if (config.cooperative) {
    void *args[] = {&program};
    return cudaLaunchCooperativeKernel(reinterpret_cast<void const *>(&megakernel_entry<Program>),
                                       dim3(config.blocks), dim3(config.threads), args, 0, stream);
  }
  megakernel_entry<<<config.blocks, config.threads, 0, stream>>>(program);
  return cudaGetLastError();
}

}  // namespace megacu::platform::cuda
