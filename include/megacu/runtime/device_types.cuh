// Device-side task and work-item types of the generic megakernel loop.
//
// Interface parity with megacu `include/megacu/runtime/device_types.cuh:7-16`.
#pragma once

#include <cstdint>

namespace megacu::runtime::device {

struct task_ref {
  int value = -1;

  __device__ bool valid() const { return value >= 0; }
};

struct work_item {
  bool active = false;
  std::int64_t tile_id = 0;
  // B200 addition: the task this work item belongs to, for dispatchers that
  // hand out (task, tile) units (co-resident progress); -1 where every task
  // runs on every tile.
  int task = -1;
};

}  // namespace megacu::runtime::device
