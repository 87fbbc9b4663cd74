// Lowering of a phase for co-resident persistent progress (the unit graph of
// include/megacu/runtime/co_resident.h).
#include <megacu/runtime/co_resident.h>

#include <cstdint>
#include <vector>

namespace megacu::runtime::co_resident {
namespace {

constexpr std::int64_t kMaxUnits = (std::int64_t(1) << 31) - 1;  // device tickets are 32-bit

status fail(status_code code, std::uint16_t detail, char const *msg) { return {code, detail, msg}; }

// Event tensors a task joins, as a bit mask.
std::uint32_t join_mask(linked_task const &t) {
  std::uint32_t mask = 0;
  for (attr const &a : t.attributes.entries()) {
    if (a.kind == attr_kind::event_join && a.event.value < static_cast<std::uint32_t>(max_events)) {
      mask |= 1u << a.event.value;
    }
  }
  return mask;
}

// The phase's ASAP order (lowest-index ready task first), as the explicit
// ASAP scheduler walks it; false on a cycle or a dangling dependency.
bool asap_order(std::span<linked_task const> tasks, std::vector<std::int32_t> &order) {
  std::vector<bool> done(tasks.size(), false);
  order.clear();
  for (std::size_t step = 0; step < tasks.size(); ++step) {
    std::size_t pick = tasks.size();
    for (std::size_t i = 0; i < tasks.size() && pick == tasks.size(); ++i) {
      if (done[i]) continue;
      bool ready = true;
      for (attr const &a : tasks[i].attributes.entries()) {
        if (a.kind == attr_kind::dependency && (a.task.value >= tasks.size() || !done[a.task.value])) {
          ready = false;
        }
      }
      if (ready) pick = i;
    }
    if (pick == tasks.size()) return false;
    done[pick] = true;
    order.push_back(static_cast<std::int32_t>(pick));
  }
  return true;
}

struct lowering {
  std::span<linked_task const> tasks;
  std::vector<std::int32_t> node_of;  // phase task -> node, -1 for sync tasks
  graph const *g;

  // Adds to `wait` the nodes that `x` stands for as a dependency of a node:
  // an operator task is itself, a sync task its own dependencies. `joined`
  // holds the acquiring node's event tensors that every sync on the way so
  // far joins; a publisher of one of them is waited for tile by tile, so it
  // is left out.
  void expand(std::int32_t x, std::uint32_t joined, std::uint32_t &wait,
              std::vector<std::vector<std::uint32_t>> &seen) const {
    for (std::uint32_t m : seen[x]) {
      if (m == joined) return;
    }
    seen[x].push_back(joined);
    linked_task const &t = tasks[x];
    if (t.kind == task_kind::operator_body) {
      std::int32_t const n = node_of[x];
      if ((g->nodes[n].publish & joined) == 0) wait |= 1u << n;
      return;
    }
    std::uint32_t const still = joined & join_mask(t);
    for (attr const &a : t.attributes.entries()) {
      if (a.kind == attr_kind::dependency) {
        expand(static_cast<std::int32_t>(a.task.value), still, wait, seen);
      }
    }
  }
};

}  // namespace

status lower(graph &out, std::span<linked_task const> tasks,
             std::span<linked_event_tensor const> events,
             dispatcher::dispatch_state const &dispatch, progress_model progress) {
  if (progress != progress_model::co_resident_persistent) {
    return fail(status_code::unsupported, 1, "co-resident lowering needs co_resident_persistent progress");
  }
  if (dispatch.task_count != tasks.size() || dispatch.event_tensor_count != events.size()) {
    return fail(status_code::invalid_argument, 6, "dispatch counts do not describe this phase");
  }
  if (events.size() > static_cast<std::size_t>(max_events)) {
    return fail(status_code::unsupported, 9, "too many event tensors for one co-resident graph");
  }
  graph g{};
  lowering low{tasks, std::vector<std::int32_t>(tasks.size(), -1), &g};

  // Event tensors: slots, storage, scope.
  g.event_count = static_cast<std::int32_t>(events.size());
  std::int64_t slots_total = 0;
  for (std::size_t e = 0; e < events.size(); ++e) {
    for (attr const &a : events[e].attributes.entries()) {
      if (a.kind == attr_kind::event_tensor_shape) {
        if (a.first < 0 || a.second < 0) {
          return fail(status_code::invalid_argument, 6, "negative event tensor shape");
        }
        g.events[e].slots += a.first * a.second;
      } else if (a.kind == attr_kind::event_tensor_storage) {
        g.events[e].storage = a.pointer;
      } else if (a.kind == attr_kind::event_tensor_scope) {
        g.events[e].team_scope = 1;
      }
    }
    slots_total += g.events[e].slots;
  }
  if (slots_total != dispatch.sync_event_count) {
    return fail(status_code::invalid_argument, 6, "dispatch counts do not describe this phase");
  }

  // Nodes: one per operator task, in submission order.
  std::int64_t grid_tiles = 0;
  for (std::size_t i = 0; i < tasks.size(); ++i) {
    linked_task const &t = tasks[i];
    std::int64_t tiles = 0;
    bool has_grid = false;
    std::uint32_t publish = 0, acquire = 0;
    for (attr const &a : t.attributes.entries()) {
      if (a.kind == attr_kind::dispatch_tile_grid) {
        if (a.first < 0 || a.second < 0) {
          return fail(status_code::invalid_argument, 6, "negative tile grid");
        }
        has_grid = true;
        tiles += a.first * a.second;
      } else if (a.kind == attr_kind::event_publish || a.kind == attr_kind::event_acquire) {
        if (a.event.value >= events.size()) {
          return fail(status_code::invalid_argument, 6, "event tensor reference out of range");
        }
        (a.kind == attr_kind::event_publish ? publish : acquire) |= 1u << a.event.value;
      }
    }
    grid_tiles += tiles;
    if (t.kind != task_kind::operator_body) continue;
    if (g.node_count == max_nodes) {
      return fail(status_code::unsupported, 8, "too many operator tasks for one co-resident graph");
    }
    std::int32_t const n = g.node_count++;
    low.node_of[i] = n;
    node &nd = g.nodes[n];
    nd.phase_task = static_cast<std::int32_t>(i);
    nd.publish = publish;
    nd.acquire = acquire;
    // Without a tile grid, a task that acquires event tensors has one unit
    // per slot (it consumes each tile as it is published); else one unit.
    std::int32_t first_acquired = -1;
    for (std::int32_t e = 0; e < g.event_count && first_acquired < 0; ++e) {
      if ((acquire >> e) & 1u) first_acquired = e;
    }
    nd.units = has_grid ? tiles : (first_acquired >= 0 ? g.events[first_acquired].slots : 1);
    if (nd.units > kMaxUnits) {
      return fail(status_code::unsupported, 10, "too many work units");
    }
    for (std::int32_t e = 0; e < g.event_count; ++e) {
      if (((publish >> e) & 1u) == 0) continue;
      if (g.events[e].publisher >= 0) {
        return fail(status_code::unsupported, 9, "an event tensor is published by two tasks");
      }
      g.events[e].publisher = n;
    }
  }
  if (grid_tiles != dispatch.total_tile_count) {
    return fail(status_code::invalid_argument, 6, "dispatch counts do not describe this phase");
  }

  // Queue order: the phase's ASAP order.
  std::vector<std::int32_t> order;
  if (!asap_order(tasks, order)) {
    return fail(status_code::invalid_argument, 2, "task dependency cycle or invalid dependency");
  }
  std::vector<std::int32_t> position(static_cast<std::size_t>(g.node_count), 0);
  std::int32_t placed = 0;
  for (std::int32_t x : order) {
    std::int32_t const n = low.node_of[x];
    if (n < 0) continue;
    position[n] = placed;
    g.order[placed++] = n;
    g.nodes[n].first_unit = g.units;
    g.units += g.nodes[n].units;
    if (g.units > kMaxUnits) {
      return fail(status_code::unsupported, 10, "too many work units");
    }
  }

  // Every tensor a node publishes or acquires has one slot per unit (tile t
  // uses slot t), storage, and for an acquire an earlier publisher.
  for (std::int32_t n = 0; n < g.node_count; ++n) {
    node const &nd = g.nodes[n];
    for (std::int32_t e = 0; e < g.event_count; ++e) {
      bool const pub = (nd.publish >> e) & 1u, acq = (nd.acquire >> e) & 1u;
      if (!pub && !acq) continue;
      event const &ev = g.events[e];
      if (ev.slots != nd.units) {
        return fail(status_code::invalid_argument, 6,
                    "a published or acquired event tensor needs one slot per tile of the task");
      }
      if (ev.storage == nullptr) {
        return fail(status_code::invalid_argument, 6,
                    "an event tensor used on the device needs symmetric_i32_storage");
      }
      if (acq && (ev.publisher < 0 || ev.publisher == n || position[ev.publisher] > position[n])) {
        return fail(status_code::invalid_argument, 6,
                    "an acquired event tensor needs a publisher earlier in the queue");
      }
    }
  }

  // Waits: per tile for the acquired tensors, per node for the rest.
  for (std::int32_t n = 0; n < g.node_count; ++n) {
    node &nd = g.nodes[n];
    std::vector<std::vector<std::uint32_t>> seen(tasks.size());
    std::uint32_t wait = 0;
    for (attr const &a : tasks[nd.phase_task].attributes.entries()) {
      if (a.kind == attr_kind::dependency) {
        low.expand(static_cast<std::int32_t>(a.task.value), nd.acquire, wait, seen);
      }
    }
    nd.wait_nodes = wait;
  }
  out = g;
  return {};
}

status lower_phase(graph &out, std::span<linked_task const> tasks,
                   std::span<linked_event_tensor const> events, progress_model progress) {
  dispatcher::dispatch_state counts;
  status st = dispatcher::map_explicit_attrs(counts, tasks, events);
  if (st.code != status_code::ok) return st;
  return lower(out, tasks, events, counts, progress);
}

}  // namespace megacu::runtime::co_resident
