// Test harness for the host runtime (phase / dispatcher / ASAP scheduler).
//
// The same source is compiled twice:
//   * against this repository's include/ and megacu_b200/csrc/runtime/*.cc
//     (tests/_build/libhost_harness.so), and
//   * against the reference's own include/ and src/*.cc, by oracle/Makefile
//     (oracle/_ref/libref_host_harness.so),
// and tests/golden/make_golden.py records the reference build's answers so
// tests/test_host_runtime.py can compare ours against them anywhere.
//
// Only the public API of megacu/runtime.h is used here, so both builds see
// the same calls.
#include <cstdint>
#include <cstring>
#include <vector>

#include <megacu/runtime.h>

namespace {

struct fake_driver {
  megacu::cuda::launch_view launch;
  megacu::nvshmem::team_view team;
};

struct order_log {
  std::vector<int> order;
  int fail_at = -1;
};

struct task_tag {
  order_log *log;
  int index;
};

megacu::status record(task_tag *tag) {
  tag->log->order.push_back(tag->index);
  if (tag->index == tag->log->fail_at) {
    return {megacu::status_code::backend_error, 77, "planted failure"};
  }
  return {};
}

void write_status(megacu::status s, std::int32_t out[2]) {
  out[0] = static_cast<std::int32_t>(s.code);
  out[1] = s.detail;
}

}  // namespace

extern "C" {

// Builds a phase of `n` tasks. kinds[i]: 0 operator task, 1 sync task.
// deps: up to 8 dependency indices per task (deps[i * 8 + j], -1 = none;
// an index >= n is a dangling dependency). tile_grid[i * 2 + {0,1}]: a
// dispatcher::tile_grid(m, n) attribute when m > 0. ev_attr[i]: bit 0
// publish, bit 1 acquire, bit 2 join of event tensor 0 (if any exists).
// n_events event tensors get shape(event_shape[e*2], event_shape[e*2+1]).
// mode 0: run(); 1: validate through run(launcher) (launcher records -2);
// progress 0 asap, 1 co_resident_persistent. fail_at: index of a task whose
// body returns an error. Outputs: order of executed bodies, dispatch counts
// (9 int64) and the returned status (code, detail).
int harness_phase(int n, const std::int32_t *kinds, const std::int32_t *deps,
                  const std::int64_t *tile_grid, const std::int32_t *ev_attr, int n_events,
                  const std::int64_t *event_shape, int mode, int progress, int fail_at,
                  std::int32_t *order_out, std::int32_t *order_len, std::int64_t counts[9],
                  std::int32_t status_out[2]) {
  namespace rt = megacu::runtime;
  fake_driver driver{};
  auto phase = rt::make_phase(driver, progress == 0 ? rt::progress_model::asap
                                                    : rt::progress_model::co_resident_persistent);
  order_log log;
  log.fail_at = fail_at;
  std::vector<task_tag> tags(static_cast<std::size_t>(n) + 1);
  std::vector<rt::event_tensor_ref> evs;
  for (int e = 0; e < n_events; ++e) {
    evs.push_back(phase.event_tensor(
        rt::attrs(rt::events::shape(event_shape[2 * e], event_shape[2 * e + 1]))));
  }
  for (int i = 0; i < n; ++i) {
    rt::attr_set set;
    for (int j = 0; j < 8; ++j) {
      std::int32_t d = deps[i * 8 + j];
      if (d >= 0) set.push(rt::scheduler::depends_on(rt::task_ref{static_cast<std::uint32_t>(d)}));
    }
    if (tile_grid[2 * i] > 0) set.push(rt::dispatcher::tile_grid(tile_grid[2 * i], tile_grid[2 * i + 1]));
    if (!evs.empty()) {
      if (ev_attr[i] & 1) set.push(rt::events::publish(evs[0]));
      if (ev_attr[i] & 2) set.push(rt::events::acquire(evs[0]));
      if (ev_attr[i] & 4) set.push(rt::events::join(evs[0]));
    }
    tags[i] = {&log, i};
    if (kinds[i] == 1) {
      phase.sync(set);
    } else {
      phase.submit(rt::op("record", &record), &tags[i], set);
    }
  }
  rt::dispatcher::dispatch_state ds;
  rt::dispatcher::map_explicit_attrs(ds, phase.tasks(), phase.event_tensors());
  counts[0] = static_cast<std::int64_t>(ds.task_count);
  counts[1] = static_cast<std::int64_t>(ds.event_tensor_count);
  counts[2] = ds.tile_grid_attrs;
  counts[3] = ds.total_tile_count;
  counts[4] = ds.sync_task_count;
  counts[5] = ds.sync_event_count;
  counts[6] = ds.event_publish_attrs;
  counts[7] = ds.event_acquire_attrs;
  counts[8] = ds.event_join_attrs;
  megacu::status st;
  if (mode == 0) {
    st = phase.run();
  } else {
    tags[n] = {&log, -2};
    st = phase.run(rt::op("launcher", &record), &tags[n]);
  }
  write_status(st, status_out);
  *order_len = static_cast<std::int32_t>(log.order.size());
  for (std::size_t i = 0; i < log.order.size(); ++i) order_out[i] = log.order[i];
  return 0;
}

// Capacity and latching behaviour: a phase<driver, max_tasks, max_events>
// with `tasks` submits and `events` event tensors, then run().
// Returns the status and whether the overflowing refs were invalid.
int harness_capacity(int tasks, int events, std::int32_t status_out[2],
                     std::int32_t *last_task_invalid, std::int32_t *last_event_invalid) {
  namespace rt = megacu::runtime;
  fake_driver driver{};
  rt::phase<fake_driver, 2, 1> phase(driver, rt::progress_model::asap);
  order_log log;
  task_tag tag{&log, 0};
  rt::task_ref last{};
  rt::event_tensor_ref last_ev{};
  for (int e = 0; e < events; ++e) last_ev = phase.event_tensor();
  for (int t = 0; t < tasks; ++t) last = phase.submit(rt::op("record", &record), &tag);
  *last_task_invalid = last == rt::invalid_task_ref() ? 1 : 0;
  *last_event_invalid = last_ev == rt::invalid_event_tensor_ref() ? 1 : 0;
  write_status(phase.run(), status_out);
  return 0;
}

// A task submitted with a null entry, then run().
int harness_missing_entry(std::int32_t status_out[2]) {
  namespace rt = megacu::runtime;
  fake_driver driver{};
  auto phase = rt::make_phase(driver, rt::progress_model::asap);
  phase.submit(rt::op<megacu::status(task_tag *)>("nothing"), static_cast<task_tag *>(nullptr));
  write_status(phase.run(), status_out);
  return 0;
}

// attr_set capacity: number of successful pushes out of `tries`.
int harness_attr_capacity(int tries) {
  megacu::runtime::attr_set set;
  int ok = 0;
  for (int i = 0; i < tries; ++i) {
    ok += set.push(megacu::runtime::scheduler::depends_on(
              megacu::runtime::task_ref{static_cast<std::uint32_t>(i)}))
              ? 1
              : 0;
  }
  return ok;
}

// Link anchors and the platform / backend helpers.
int harness_components(std::int32_t out[8]) {
  fake_driver d{};
  out[0] = megacu::cuda::has_stream(d.launch) ? 1 : 0;
  d.launch.stream = &d;
  out[1] = megacu::cuda::has_stream(d.launch) ? 1 : 0;
  out[2] = megacu::nvshmem::team_size(d.team);
  out[3] = megacu::nvshmem::has_remote_pes(d.team) ? 1 : 0;
  d.team.team_n_pes = 2;
  out[4] = megacu::nvshmem::team_size(d.team);
  out[5] = megacu::nvshmem::has_remote_pes(d.team) ? 1 : 0;
  int ready[1] = {0};
  megacu::cuda::device::signal_ready(ready, 0, 7);
  out[6] = megacu::cuda::device::load_ready(ready, 0);
  out[7] = megacu::nvshmem::device::remote_int(ready, 0, 0);
  return 0;
}

}  // extern "C"
