// Test harness for the co-resident lowering (megacu/runtime/co_resident.h), a
// B200 extension with no counterpart in megacu: built only against this
// repository's headers, into tests/_build/libhost_harness.so.
#include <cstdint>

#include <megacu/runtime.h>
#include <megacu/runtime/co_resident.h>

namespace {

struct fake_driver {
  megacu::cuda::launch_view launch;
  megacu::nvshmem::team_view team;
};

megacu::status nothing(int) { return {}; }

}  // namespace

extern "C" {

// Builds a phase of `n` tasks like harness_phase (kinds[i]: 0 operator task,
// 1 sync task; deps: 8 per task, -1 = none; tile_grid[i * 2 + {0,1}] when
// > 0 in the first entry) with `n_events` event tensors of shape
// event_shape[e * 2 + {0, 1}]; ev[i * 3 + {0, 1, 2}]: the event tensor task
// i publishes / acquires / joins, -1 = none; bit e of storage_mask gives
// event tensor e a (never dereferenced) storage attribute. progress 0 asap, 1
// co_resident_persistent. Lowers it; outputs the status (code, detail), the
// graph header (node_count, units, event_count) and per node (8 int64 each):
// phase task, publish mask, acquire mask, wait mask, units, first unit, queue
// position, and per event (2 int64): slots, publisher. ev[i * 3 + 1] may name
// a second acquired tensor through ev2[i] (-1 = none).
int harness_co_resident(int n, const std::int32_t *kinds, const std::int32_t *deps,
                        const std::int64_t *tile_grid, const std::int32_t *ev,
                        const std::int32_t *ev2, int n_events,
                        const std::int64_t *event_shape, std::uint32_t storage_mask,
                        int progress, std::int32_t status_out[2],
                        std::int64_t header[3], std::int64_t *nodes, std::int64_t *events) {
  namespace rt = megacu::runtime;
  namespace co = megacu::runtime::co_resident;
  fake_driver driver{};
  auto phase = rt::make_phase(driver, progress == 0 ? rt::progress_model::asap
                                                    : rt::progress_model::co_resident_persistent);
  static int storage[1];
  rt::event_tensor_ref evs[16];
  for (int e = 0; e < n_events && e < 16; ++e) {
    auto set = rt::attrs(rt::events::shape(event_shape[2 * e], event_shape[2 * e + 1]));
    if ((storage_mask >> e) & 1u) {
      set.push(megacu::cuda_nvshmem::events::symmetric_i32_storage(storage));
    }
    evs[e] = phase.event_tensor(set);
  }
  for (int i = 0; i < n; ++i) {
    rt::attr_set set;
    for (int j = 0; j < 8; ++j) {
      std::int32_t d = deps[i * 8 + j];
      if (d >= 0) set.push(rt::scheduler::depends_on(rt::task_ref{static_cast<std::uint32_t>(d)}));
    }
    if (tile_grid[2 * i] > 0) set.push(rt::dispatcher::tile_grid(tile_grid[2 * i], tile_grid[2 * i + 1]));
    if (ev[3 * i + 0] >= 0) set.push(rt::events::publish(evs[ev[3 * i + 0]]));
    if (ev[3 * i + 1] >= 0) set.push(rt::events::acquire(evs[ev[3 * i + 1]]));
    if (ev2[i] >= 0) set.push(rt::events::acquire(evs[ev2[i]]));
    if (ev[3 * i + 2] >= 0) set.push(rt::events::join(evs[ev[3 * i + 2]]));
    if (kinds[i] == 1) {
      phase.sync(set);
    } else {
      phase.submit(rt::op("nothing", &nothing), i, set);
    }
  }
  co::graph g;
  megacu::status st = co::lower_phase(g, phase.tasks(), phase.event_tensors(), phase.progress());
  status_out[0] = static_cast<std::int32_t>(st.code);
  status_out[1] = st.detail;
  header[0] = g.node_count;
  header[1] = g.units;
  header[2] = g.event_count;
  if (st.code != megacu::status_code::ok) return 0;
  for (int k = 0; k < g.node_count; ++k) {
    co::node const &nd = g.nodes[k];
    std::int64_t *row = nodes + 8 * k;
    row[0] = nd.phase_task;
    row[1] = nd.publish;
    row[2] = nd.acquire;
    row[3] = nd.wait_nodes;
    row[4] = nd.units;
    row[5] = nd.first_unit;
    row[6] = -1;
    for (int q = 0; q < g.node_count; ++q) {
      if (g.order[q] == k) row[6] = q;
    }
    row[7] = 0;
  }
  for (int e = 0; e < g.event_count; ++e) {
    events[2 * e] = g.events[e].slots;
    events[2 * e + 1] = g.events[e].publisher;
  }
  return 0;
}

}  // extern "C"
