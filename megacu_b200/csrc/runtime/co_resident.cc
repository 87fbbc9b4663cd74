// Lowering of a phase for co-resident persistent progress (the unit graph of
// include/megacu/runtime/co_resident.h).
#include <megacu/runtime/co_resident.h>

#include <cstdint>
#include <vector>

namespace megacu::runtime::co_resident {
namespace {

constexpr std::int64_t kMaxUnits = (std::int64_t(1) << 31) - 1;  // device tickets are 32-bit

status fail(status_code code, std::uint16_t detail, char const *msg) { return {code, detail, msg}; }

bool joins(linked_task const &t, std::int32_t ev) {
  if (ev == no_event) return false;
  for (attr const &a : t.attributes.entries()) {
    if (a.kind == attr_kind::event_join && static_cast<std::int32_t>(a.event.value) == ev) {
      return true;
    }
  }
  return false;
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
  graph *g;

  // Adds to `wait` the nodes that `x` stands for as a dependency of a node
  // that acquires `ev` (published by node `pub`): an operator task is itself,
  // a sync task its own dependencies. The publisher is left out when every
  // sync on the way joins `ev` (its tiles are waited for one by one).
  void expand(std::int32_t x, bool joined, std::int32_t ev, std::int32_t pub,
              std::uint32_t &wait, std::vector<std::uint8_t> &seen) const {
    std::uint8_t const mark = joined ? 2 : 1;
    if (seen[x] & mark) return;
    seen[x] |= mark;
    linked_task const &t = tasks[x];
    if (t.kind == task_kind::operator_body) {
      std::int32_t const n = node_of[x];
      if (!(joined && n == pub)) wait |= 1u << n;
      return;
    }
    bool const still = joined && joins(t, ev);
    for (attr const &a : t.attributes.entries()) {
      if (a.kind == attr_kind::dependency) {
        expand(static_cast<std::int32_t>(a.task.value), still, ev, pub, wait, seen);
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
    std::int32_t publish = no_event, acquire = no_event;
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
        std::int32_t &slot = a.kind == attr_kind::event_publish ? publish : acquire;
        std::int32_t const ev = static_cast<std::int32_t>(a.event.value);
        if (slot != no_event && slot != ev) {
          return fail(status_code::unsupported, 9,
                      "a co-resident task publishes / acquires at most one event tensor");
        }
        slot = ev;
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
    // Without a tile grid, a task that acquires an event tensor has one unit
    // per slot (it consumes each tile as it is published); else one unit.
    nd.units = has_grid ? tiles : (acquire != no_event ? g.events[acquire].slots : 1);
    if (nd.units > kMaxUnits) {
      return fail(status_code::unsupported, 10, "too many work units");
    }
    if (publish != no_event) {
      if (g.events[publish].publisher >= 0) {
        return fail(status_code::unsupported, 9, "an event tensor is published by two tasks");
      }
      g.events[publish].publisher = n;
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

  // A tensor that is published or acquired on the device needs its storage.
  for (std::int32_t e = 0; e < g.event_count; ++e) {
    bool used = g.events[e].publisher >= 0;
    for (std::int32_t n = 0; n < g.node_count; ++n) used = used || g.nodes[n].acquire == e;
    if (used && g.events[e].storage == nullptr) {
      return fail(status_code::invalid_argument, 6,
                  "an event tensor used on the device needs symmetric_i32_storage");
    }
  }

  // Waits: per tile for the acquired tensor, per node for the rest.
  for (std::int32_t n = 0; n < g.node_count; ++n) {
    node &nd = g.nodes[n];
    std::int32_t pub = -1;
    if (nd.acquire != no_event) {
      event const &ev = g.events[nd.acquire];
      pub = ev.publisher;
      if (pub < 0 || pub == n || position[pub] > position[n] || ev.slots != nd.units ||
          ev.slots != g.nodes[pub].units) {
        return fail(status_code::invalid_argument, 6,
                    "an acquired event tensor needs an earlier publisher with one tile per slot");
      }
    }
    std::vector<std::uint8_t> seen(tasks.size(), 0);
    std::uint32_t wait = 0;
    for (attr const &a : tasks[nd.phase_task].attributes.entries()) {
      if (a.kind == attr_kind::dependency) {
        low.expand(static_cast<std::int32_t>(a.task.value), true, nd.acquire, pub, wait, seen);
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
