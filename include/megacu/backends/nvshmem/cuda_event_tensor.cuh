// Event tensor over the NVLink peer table.
//
// Interface parity with megacu
// `include/megacu/backends/nvshmem/cuda_event_tensor.cuh:13-59`:
// event_tensor_i32{events, tiles, my_pe, n_pes} with publish(tile, value) /
// acquire(tile, value) over int32 [n_pes][tiles] (slot = pe * tiles + tile),
// and task_event_tensor_i32{event_tensor, publish_task, acquire_task} whose
// before/after hooks acquire before `acquire_task` and publish after
// `publish_task` with ready value tile + 1.
//
// B200 differences: publish is a sys-scope fence followed by a release store
// into every PE's slot through the peer table (megacu: __threadfence_system,
// atomicExch, nvshmem_int_p); acquire is a bounded ld.acquire.sys spin that
// reports failure instead of hanging, and the hooks return that result.
#pragma once

#include <cstdint>

#include <megacu/backends/nvshmem.h>
#include <megacu/platform/cuda.h>

namespace megacu::backend::nvshmem::cuda {

struct event_tensor_i32 {
  int *events = nullptr;
  std::int64_t tiles = 0;
  int my_pe = 0;
  int n_pes = 1;
  megacu::nvshmem::peer_table const *peers = nullptr;  // required when n_pes > 1
  std::uint64_t timeout_ns = megacu::cuda::device::default_wait_timeout_ns;
  unsigned int *error_word = nullptr;  // optional: set to 1 on a timed-out acquire

  __device__ void publish(std::int64_t tile_id, int ready_value) const {
    megacu::cuda::device::fence_system();
    std::int64_t const slot = static_cast<std::int64_t>(my_pe) * tiles + tile_id;
    for (int pe = 0; pe < n_pes; ++pe) {
      int *target = pe == my_pe ? events : peers->translate(events, pe);
      megacu::cuda::device::signal_ready(target, slot, ready_value);
    }
  }

  __device__ bool acquire(std::int64_t tile_id, int ready_value) const {
    for (int pe = 0; pe < n_pes; ++pe) {
      std::int64_t const slot = static_cast<std::int64_t>(pe) * tiles + tile_id;
      if (!megacu::cuda::device::wait_ready(events, slot, ready_value, timeout_ns)) {
        if (error_word != nullptr) atomicExch(error_word, 1u);
        return false;
      }
    }
    return true;
  }
};

struct task_event_tensor_i32 {
  event_tensor_i32 event_tensor;
  int publish_task = -1;
  int acquire_task = -1;

  template <class Context, class Task, class Work>
  __device__ bool before(Context ctx, Task task, Work work) const {
    if (task.value == acquire_task && ctx.thread_id() == 0) {
      return event_tensor.acquire(work.tile_id, static_cast<int>(work.tile_id + 1));
    }
    return true;
  }

  template <class Context, class Task, class Work>
  __device__ bool after(Context ctx, Task task, Work work) const {
    if (task.value == publish_task && ctx.thread_id() == 0) {
      event_tensor.publish(work.tile_id, static_cast<int>(work.tile_id + 1));
    }
    return true;
  }
};

}  // namespace megacu::backend::nvshmem::cuda
