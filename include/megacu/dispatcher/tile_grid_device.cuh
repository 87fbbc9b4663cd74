// Device dispatchers.
//
// `tile_grid` keeps megacu's static round-robin assignment (tile =
// blockIdx + i * gridDim; `include/megacu/dispatcher/tile_grid_device.cuh:9-24`).
// `task_queue` is the B200 dispatcher: CTAs pull tiles from a device ticket
// counter, so a CTA that finishes early takes the next tile instead of
// idling. The counter must be zero at launch; `tiles + gridDim.x` tickets are
// drawn per launch (each CTA draws one past the end).
#pragma once

#include <cstdint>

#include <megacu/runtime/device_types.cuh>

namespace megacu::dispatcher::device {

struct tile_grid {
  std::int64_t tiles = 0;

  template <class Context>
  __device__ megacu::runtime::device::work_item first(Context ctx) const {
    megacu::runtime::device::work_item w;
    w.tile_id = ctx.block_id();
    w.active = w.tile_id < tiles;
    return w;
  }

  template <class Context>
  __device__ megacu::runtime::device::work_item next(
      Context ctx, megacu::runtime::device::work_item current) const {
    megacu::runtime::device::work_item w;
    w.tile_id = current.tile_id + ctx.grid_blocks();
    w.active = w.tile_id < tiles;
    return w;
  }
};

struct task_queue {
  std::int64_t tiles = 0;
  unsigned int *ticket = nullptr;  // device counter, zero at launch

  template <class Context>
  __device__ megacu::runtime::device::work_item draw(Context ctx) const {
    __shared__ unsigned int drawn;
    if (ctx.thread_id() == 0) drawn = atomicAdd(ticket, 1u);
    ctx.sync_block();
    megacu::runtime::device::work_item w;
    w.tile_id = drawn;
    w.active = w.tile_id < tiles;
    ctx.sync_block();
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

}  // namespace megacu::dispatcher::device
