// Host ASAP scheduler.
//
// Behaviour follows megacu `src/scheduler/explicit_asap.cc:29-111`: at every
// step the lowest-index task whose `depends_on` tasks have all completed runs
// next (submission order breaks ties); sync-only tasks complete without a
// body; no runnable task left -> invalid_argument/2 (cycle or dangling
// dependency); a missing callable -> invalid_argument/3; any progress model
// other than ASAP -> unsupported/1. `validate_*` walks the same order without
// invoking operator bodies.
#include <cstdint>
#include <vector>

#include <megacu/runtime.h>

namespace megacu::runtime::scheduler {
namespace {

bool ready_to_run(linked_task const &task, std::vector<bool> const &done) {
  for (attr const &a : task.attributes.entries()) {
    if (a.kind != attr_kind::dependency) {
      continue;
    }
    if (a.task.value >= done.size() || !done[a.task.value]) {
      return false;
    }
  }
  return true;
}

status walk_asap(std::span<linked_task const> tasks,
                 dispatcher::dispatch_state const & /*dispatch*/,
                 progress_model progress, bool invoke_bodies) {
  if (progress != progress_model::asap) {
    return {status_code::unsupported, 1,
            "explicit ASAP scheduler only supports ASAP progress"};
  }
  std::vector<bool> done(tasks.size(), false);
  for (std::size_t step = 0; step < tasks.size(); ++step) {
    std::size_t pick = tasks.size();
    for (std::size_t i = 0; i < tasks.size(); ++i) {
      if (!done[i] && ready_to_run(tasks[i], done)) {
        pick = i;
        break;
      }
    }
    if (pick == tasks.size()) {
      return {status_code::invalid_argument, 2,
              "task dependency cycle or invalid dependency"};
    }
    linked_task const &task = tasks[pick];
    if (task.kind == task_kind::operator_body && invoke_bodies) {
      if (!task.invoke) {
        return {status_code::invalid_argument, 3, "missing task callable"};
      }
      status st = task.invoke();
      if (st.code != status_code::ok) {
        return st;
      }
    }
    done[pick] = true;
  }
  return {};
}

}  // namespace

status run_explicit_asap(std::span<linked_task const> tasks,
                         dispatcher::dispatch_state const &dispatch,
                         progress_model progress) {
  return walk_asap(tasks, dispatch, progress, true);
}

status validate_explicit_asap(std::span<linked_task const> tasks,
                              dispatcher::dispatch_state const &dispatch,
                              progress_model progress) {
  return walk_asap(tasks, dispatch, progress, false);
}

}  // namespace megacu::runtime::scheduler

extern "C" int megacu_scheduler_explicit_asap_component() { return 1; }
