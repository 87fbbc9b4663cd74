// Host dispatcher: folds the attributes of a phase into dispatch counts.
//
// Behaviour follows megacu `src/dispatcher/explicit_attrs.cc:5-40`:
// tile_grid(m, n) adds m*n tiles, an event tensor shape(a, b) adds a*b sync
// events, and every publish / acquire / join attribute is counted once. The
// counts are the host half of the dispatcher; the device half is the tile
// queue inside the megakernel.
#include <megacu/runtime.h>

namespace megacu::runtime::dispatcher {

status map_explicit_attrs(dispatch_state &out,
                          std::span<linked_task const> tasks,
                          std::span<linked_event_tensor const> events) {
  dispatch_state s;
  s.task_count = tasks.size();
  s.event_tensor_count = events.size();

  for (linked_event_tensor const &ev : events) {
    for (attr const &a : ev.attributes.entries()) {
      if (a.kind == attr_kind::event_tensor_shape) {
        s.sync_event_count += a.first * a.second;
      }
    }
  }

  for (linked_task const &task : tasks) {
    s.sync_task_count += task.kind == task_kind::sync_only ? 1 : 0;
    for (attr const &a : task.attributes.entries()) {
      switch (a.kind) {
        case attr_kind::dispatch_tile_grid:
          s.tile_grid_attrs += 1;
          s.total_tile_count += a.first * a.second;
          break;
        case attr_kind::event_publish:
          s.event_publish_attrs += 1;
          break;
        case attr_kind::event_acquire:
          s.event_acquire_attrs += 1;
          break;
        case attr_kind::event_join:
          s.event_join_attrs += 1;
          break;
        default:
          break;
      }
    }
  }

  out = s;
  return {};
}

}  // namespace megacu::runtime::dispatcher

extern "C" int megacu_dispatcher_explicit_attrs_component() { return 1; }
