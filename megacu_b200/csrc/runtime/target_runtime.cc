// Target runtime: dispatcher first, then the scheduler.
//
// Behaviour follows megacu `src/target/runtime.cc:5-27`.
#include <megacu/runtime.h>

namespace megacu::runtime::target {
namespace {

template <class Next>
status dispatch_then(std::span<linked_task const> tasks,
                     std::span<linked_event_tensor const> events,
                     Next next) {
  dispatcher::dispatch_state counts;
  status st = dispatcher::map_explicit_attrs(counts, tasks, events);
  if (st.code != status_code::ok) {
    return st;
  }
  return next(counts);
}

}  // namespace

status run_phase(std::span<linked_task const> tasks,
                 std::span<linked_event_tensor const> events,
                 progress_model progress) {
  return dispatch_then(tasks, events, [&](auto const &counts) {
    return scheduler::run_explicit_asap(tasks, counts, progress);
  });
}

status validate_phase(std::span<linked_task const> tasks,
                      std::span<linked_event_tensor const> events,
                      progress_model progress) {
  return dispatch_then(tasks, events, [&](auto const &counts) {
    return scheduler::validate_explicit_asap(tasks, counts, progress);
  });
}

}  // namespace megacu::runtime::target

extern "C" int megacu_target_runtime_component() { return 1; }
