// Device scheduler: tasks 0 .. task_count-1 in order for every work item.
//
// Interface parity with megacu
// `include/megacu/scheduler/explicit_asap_device.cuh:7-31`.
#pragma once

#include <megacu/runtime/device_types.cuh>

namespace megacu::scheduler::device {

struct explicit_asap {
  int task_count = 0;

  template <class Context, class Work>
  __device__ megacu::runtime::device::task_ref first(Context, Work) const {
    megacu::runtime::device::task_ref t;
    t.value = task_count > 0 ? 0 : -1;
    return t;
  }

  template <class Context, class Work>
  __device__ megacu::runtime::device::task_ref next(
      Context, Work, megacu::runtime::device::task_ref current) const {
    megacu::runtime::device::task_ref t;
    t.value = current.value + 1 < task_count ? current.value + 1 : -1;
    return t;
  }

  template <class Context, class Work>
  __device__ void complete(Context, megacu::runtime::device::task_ref, Work) const {}
};

}  // namespace megacu::scheduler::device
