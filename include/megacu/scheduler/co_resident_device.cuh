// Device half of co-resident persistent progress (a B200 extension): the
// dispatcher, scheduler and backend hooks that run a lowered unit graph
// (megacu/runtime/co_resident.h) inside the generic persistent loop
// (megacu/runtime/device_entry.cuh) as one launch.
//
//  * co_resident_queue (dispatcher): every CTA draws unit tickets from one
//    device counter; unit u is tile u - first_unit of the node whose range
//    holds it (work_item.task = that node);
//  * co_resident (scheduler): one task per unit, the unit's node;
//  * co_resident_events (backend): before a unit, thread 0 waits until every
//    node it depends on has completed all its units and, for each event
//    tensor the node acquires, until slot `tile` holds tile + 1 on every PE
//    of the tensor's scope (megacu's ready value,
//    backends/nvshmem/cuda_event_tensor.cuh:41-59); after it, it publishes
//    slot `tile` of each tensor the node publishes and counts the unit
//    done. Every
//    wait is bounded: one that gives up sets the state's error word and
//    ends the CTA's loop.
// The launcher copies the graph into `co_resident_state` and zeroes the
// counters before every launch, and launches cooperatively so that all CTAs
// are resident at once (every wait targets units handed out earlier).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include <megacu/backends/nvshmem.h>
#include <megacu/backends/nvshmem/cuda_event_tensor.cuh>
#include <megacu/platform/cuda.h>
#include <megacu/platform/cuda/megakernel.cuh>
#include <megacu/runtime/co_resident.h>
#include <megacu/runtime/device_entry.cuh>
#include <megacu/runtime/device_types.cuh>

namespace megacu::scheduler::device {

namespace co = megacu::runtime::co_resident;

// Device memory of one co-resident launch.
struct co_resident_state {
  co::graph graph;
  unsigned int ticket;         // next unit to hand out
  unsigned int error;          // 0, or 1 once a wait gave up
  unsigned int error_info[2];  // node, tile of the first wait that gave up
  unsigned int done[co::max_nodes];  // completed units per node
};

struct co_resident_queue {
  co_resident_state *state = nullptr;

  template <class Context>
  __device__ megacu::runtime::device::work_item draw(Context ctx) const {
    __shared__ unsigned int drawn;
    if (ctx.thread_id() == 0) drawn = atomicAdd(&state->ticket, 1u);
    ctx.sync_block();
    unsigned int const u = drawn;
    ctx.sync_block();
    megacu::runtime::device::work_item w;
    co::graph const &g = state->graph;
    w.active = static_cast<std::int64_t>(u) < g.units;
    if (w.active) {
      for (int n = 0; n < g.node_count; ++n) {
        co::node const &nd = g.nodes[n];
        if (static_cast<std::int64_t>(u) >= nd.first_unit &&
            static_cast<std::int64_t>(u) < nd.first_unit + nd.units) {
          w.task = n;
          w.tile_id = static_cast<std::int64_t>(u) - nd.first_unit;
        }
      }
    }
    return w;
  }

  template <class Context>
  __device__ megacu::runtime::device::work_item first(Context ctx) const {
    return draw(ctx);
  }

  template <class Context>
  __device__ megacu::runtime::device::work_item next(
      Context ctx, megacu::runtime::device::work_item) const {
    return draw(ctx);
  }
};

struct co_resident {
  template <class Context, class Work>
  __device__ megacu::runtime::device::task_ref first(Context, Work work) const {
    megacu::runtime::device::task_ref t;
    t.value = work.task;
    return t;
  }

  template <class Context, class Work>
  __device__ megacu::runtime::device::task_ref next(Context, Work,
                                                    megacu::runtime::device::task_ref) const {
    return {};
  }

  template <class Context, class Work>
  __device__ void complete(Context, megacu::runtime::device::task_ref, Work) const {}
};

struct co_resident_events {
  co_resident_state *state = nullptr;
  megacu::nvshmem::peer_table peers;  // team of the team-scope event tensors
  std::uint64_t timeout_ns = megacu::cuda::device::default_wait_timeout_ns;

  __device__ megacu::backend::nvshmem::cuda::event_tensor_i32 tensor(std::int32_t e) const {
    co::event const &ev = state->graph.events[e];
    megacu::backend::nvshmem::cuda::event_tensor_i32 t;
    t.events = static_cast<int *>(ev.storage);
    t.tiles = ev.slots;
    t.my_pe = ev.team_scope ? peers.my_pe : 0;
    t.n_pes = ev.team_scope ? peers.n_pes : 1;
    t.peers = &peers;
    t.timeout_ns = timeout_ns;
    return t;
  }

  __device__ void give_up(int node, std::int64_t tile) const {
    if (atomicCAS(&state->error, 0u, 1u) == 0u) {
      state->error_info[0] = static_cast<unsigned int>(node);
      state->error_info[1] = static_cast<unsigned int>(tile);
    }
  }

  template <class Context, class Task, class Work>
  __device__ bool before(Context ctx, Task task, Work work) const {
    if (ctx.thread_id() != 0) return true;
    co::graph const &g = state->graph;
    co::node const &nd = g.nodes[task.value];
    std::uint64_t const start = megacu::cuda::device::global_time_ns();
    for (int j = 0; j < g.node_count; ++j) {
      if (((nd.wait_nodes >> j) & 1u) == 0) continue;
      unsigned int const want = static_cast<unsigned int>(g.nodes[j].units);
      for (std::uint32_t spin = 0;; ++spin) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];"
                     : "=r"(v)
                     : "l"(&state->done[j])
                     : "memory");
        if (v >= want) break;
        bool const gave_up = *static_cast<unsigned int volatile *>(&state->error) != 0u;
        if (gave_up || megacu::cuda::device::global_time_ns() - start > timeout_ns) {
          give_up(task.value, work.tile_id);
          return false;
        }
        __nanosleep(spin < 64 ? 64 : 256);
      }
    }
    for (int e = 0; e < g.event_count; ++e) {
      if (((nd.acquire >> e) & 1u) != 0 &&
          !tensor(e).acquire(work.tile_id, static_cast<int>(work.tile_id + 1))) {
        give_up(task.value, work.tile_id);
        return false;
      }
    }
    return true;
  }

  template <class Context, class Task, class Work>
  __device__ bool after(Context ctx, Task task, Work work) const {
    if (ctx.thread_id() != 0) return true;
    co::graph const &g = state->graph;
    co::node const &nd = g.nodes[task.value];
    for (int e = 0; e < g.event_count; ++e) {
      if (((nd.publish >> e) & 1u) != 0) {
        tensor(e).publish(work.tile_id, static_cast<int>(work.tile_id + 1));
      }
    }
    __threadfence();  // the CTA's writes of this unit (ordered by the block barrier) first
    atomicAdd(&state->done[task.value], 1u);
    return true;
  }
};

// The generic persistent loop over a co-resident graph with the caller's
// operator table: `Operators::invoke(ctx, task, work)` runs tile
// `work.tile_id` of node `task.value` (nodes are numbered in the phase's
// submission order of operator tasks).
template <class Operators>
using co_resident_program =
    megacu::runtime::device::entry<co_resident, co_resident_queue, co_resident_events, Operators>;

// Launches `ops` over `g`: copies the graph into `state` (device memory) with
// every counter zeroed, then one cooperative launch of as many CTAs of
// `threads` threads as are resident at once, at most one per unit. The event
// tensors' storage must be reset by the caller (megacu's launcher zeroes its
// events before every call).
template <class Operators>
cudaError_t launch_co_resident(co::graph const &g, co_resident_state *state, Operators const &ops,
                               megacu::nvshmem::peer_table const &peers, std::uint64_t timeout_ns,
                               int device, int threads, cudaStream_t stream) {
  co_resident_state init{};
  init.graph = g;
  cudaError_t e = cudaMemcpyAsync(state, &init, sizeof(init), cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  using program = co_resident_program<Operators>;
  program prog{co_resident{}, co_resident_queue{state}, co_resident_events{state, peers, timeout_ns},
               ops};
  int per_sm = 0, sms = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &per_sm, megacu::platform::cuda::megakernel_entry<program>, threads, 0);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  std::int64_t const resident = static_cast<std::int64_t>(std::max(per_sm, 1)) * sms;
  megacu::platform::cuda::launch_config cfg;
  cfg.blocks = static_cast<int>(std::max<std::int64_t>(1, std::min(g.units, resident)));
  cfg.threads = threads;
  cfg.cooperative = true;
  return megacu::platform::cuda::launch_megakernel(stream, cfg, prog);
}

}  // namespace megacu::scheduler::device
