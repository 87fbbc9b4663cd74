// Generic persistent device loop: for every work item the dispatcher hands
// this CTA, run the scheduler's tasks in order with the backend's
// before/after hooks around each operator body.
//
// Interface parity with megacu `include/megacu/runtime/device_entry.cuh:12-29`
// (entry<Scheduler, Dispatcher, Backend, Operators>, before -> sync ->
// invoke -> sync -> after -> sync -> complete). B200 difference: a backend
// hook may return bool; `false` (a bounded wait that gave up) ends this CTA's
// loop instead of running the body on data that never arrived. The decision
// is made block-uniform through shared memory so no CTA barrier is skipped
// by some threads only.
#pragma once

#include <type_traits>

#include <megacu/runtime/device_types.cuh>

namespace megacu::runtime::device {

namespace detail {

template <class Hook>
__device__ __forceinline__ bool hook_ok(Hook &&hook) {
  if constexpr (std::is_same_v<decltype(hook()), bool>) {
    return hook();
  } else {
    hook();
    return true;
  }
}

}  // namespace detail

template <class Scheduler, class Dispatcher, class Backend, class Operators>
struct entry {
  Scheduler scheduler;
  Dispatcher dispatcher;
  Backend backend;
  Operators operators;

  template <class Context>
  __device__ void operator()(Context ctx) const {
    __shared__ int failed;
    if (ctx.thread_id() == 0) failed = 0;
    ctx.sync_block();
    for (auto work = dispatcher.first(ctx); work.active; work = dispatcher.next(ctx, work)) {
      for (auto task = scheduler.first(ctx, work); task.valid();
           task = scheduler.next(ctx, work, task)) {
        if (!detail::hook_ok([&] { return backend.before(ctx, task, work); })) {
          failed = 1;
        }
        ctx.sync_block();
        if (failed) return;

        operators.invoke(ctx, task, work);
        ctx.sync_block();

        if (!detail::hook_ok([&] { return backend.after(ctx, task, work); })) {
          failed = 1;
        }
        ctx.sync_block();
        if (failed) return;

        scheduler.complete(ctx, task, work);
      }
    }
  }
};

}  // namespace megacu::runtime::device
