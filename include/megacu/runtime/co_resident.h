// Co-resident persistent progress: a phase lowered to ONE persistent launch
// whose CTAs pull work units from a device queue (a B200 extension).
//
// megacu declares progress_model::co_resident_persistent
// (include/megacu/runtime.h:18) but its only scheduler rejects it
// (src/scheduler/explicit_asap.cc:34-39, unsupported/1), and a phase's
// attributes are only counted by its dispatcher, never consumed. Here they
// are: lower() reads the phase's tasks, tile grids, event tensors and
// dependencies and builds the unit graph that the device side
// (megacu/scheduler/co_resident_device.cuh) executes:
//
//  * every operator task is a node with `units` work units: the tiles of its
//    dispatcher::tile_grid, or without a grid one per slot of the event
//    tensors it acquires, or one; sync tasks have none;
//  * the device queue hands out the units node by node in the phase's ASAP
//    order (lowest ready task index first), tile by tile within a node;
//  * a node that acquires event tensors published by other nodes waits per
//    tile: its tile t starts once each publisher's tile t has published (on
//    every PE for a team-scope tensor). A sync task joining such a tensor,
//    and a direct dependency on its publisher, are covered by this per-tile
//    wait: the phase's barrier becomes tile-level dataflow;
//  * every other dependency waits for the whole node: its units start once
//    every unit of the node it depends on has completed (dependencies on a
//    sync task stand for that task's own dependencies).
// Every wait targets units handed out earlier, so a launch whose CTAs are
// all resident at once (cooperative launch) cannot deadlock.
//
// Errors: progress other than co_resident_persistent -> unsupported/1; a
// dependency cycle or dangling dependency -> invalid_argument/2 (as the ASAP
// scheduler); more than `max_nodes` operator tasks -> unsupported/8; more
// than `max_events` event tensors, or an event tensor published by two
// tasks -> unsupported/9; an acquired event tensor that no task publishes,
// is published later in the queue or by the acquiring task itself, a
// published or acquired tensor whose slots differ from the task's tiles, or
// one without storage -> invalid_argument/6; unit count overflow ->
// unsupported/10.
#pragma once

#include <cstdint>
#include <span>

#include <megacu/runtime.h>

namespace megacu::runtime::co_resident {

inline constexpr int max_nodes = 16;
inline constexpr int max_events = 16;

// One operator task of the phase. Nodes are indexed by the task's position
// among the phase's operator tasks (its slot in the device operator table).
struct node {
  std::int32_t phase_task = -1;   // index of the task in the phase
  std::uint32_t publish = 0;      // bit e: tile t publishes slot t of event tensor e
  std::uint32_t acquire = 0;      // bit e: tile t waits for slot t of event tensor e
  std::uint32_t wait_nodes = 0;   // bit j: every unit of node j completes first
  std::int64_t units = 0;
  std::int64_t first_unit = 0;    // queue index of the node's first unit
};

struct event {
  std::int64_t slots = 0;         // shape(a, b): a * b
  void *storage = nullptr;        // symmetric_i32_storage, if given
  std::int32_t team_scope = 0;    // 1 with cuda_nvshmem::events::team_scope()
  std::int32_t publisher = -1;    // node that publishes it
};

// The lowered graph; trivially copyable, so it can be copied to the device.
struct graph {
  std::int32_t node_count = 0;
  std::int32_t event_count = 0;
  std::int64_t units = 0;                 // total work units of the launch
  std::int32_t order[max_nodes] = {};     // node indices in queue order
  node nodes[max_nodes] = {};
  event events[max_events] = {};
};

// Lowers `tasks` / `events` (a phase's, with `dispatch` from
// dispatcher::map_explicit_attrs) for co-resident persistent progress.
status lower(graph &out, std::span<linked_task const> tasks,
             std::span<linked_event_tensor const> events,
             dispatcher::dispatch_state const &dispatch, progress_model progress);

// map_explicit_attrs, then lower(): the co-resident counterpart of
// target::validate_phase.
status lower_phase(graph &out, std::span<linked_task const> tasks,
                   std::span<linked_event_tensor const> events, progress_model progress);

}  // namespace megacu::runtime::co_resident
