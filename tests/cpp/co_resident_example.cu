// A phase of three operator tasks with per-tile dataflow, run with
// co-resident persistent progress through the public API only (test
// infrastructure; also the worked example of that API):
//
//   fill   tile_grid(1, T), publishes E0:   x[t][i] = t + i / 1024
//   scale  acquires E0, publishes E1:       y[t][i] = 2 x[t][i]
//   sum    acquires E0 and E1:              z[t][i] = x[t][i] + y[t][i]
//
// The phase is built with megacu's authoring API (make_phase, event_tensor,
// submit, attrs), lowered by co_resident::lower_phase and launched with
// launch_co_resident and this file's own device operator table; one
// persistent launch runs all 3 T units, each tile of `scale` and `sum`
// starting as soon as its inputs' tiles are published. Prints "ok" and exits
// 0 when z matches on the host; exits 1 on a mismatch, 2 on an API error.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <vector>

#include <megacu/runtime.h>
#include <megacu/runtime/co_resident.h>
#include <megacu/scheduler/co_resident_device.cuh>

namespace {

constexpr int kTiles = 300;
constexpr int kTileElems = 1024;

struct fake_driver {
  megacu::cuda::launch_view launch;
  megacu::nvshmem::team_view team;
};

// Host-side stand-ins for the operators' signatures (the phase records them;
// the device table below is what runs).
megacu::status op_fill(float *) { return {}; }
megacu::status op_scale(float const *, float *) { return {}; }
megacu::status op_sum(float const *, float const *, float *) { return {}; }

struct operators {
  float *x, *y, *z;

  template <class Context, class Task, class Work>
  __device__ void invoke(Context ctx, Task task, Work work) const {
    std::int64_t const base = work.tile_id * kTileElems;
    for (int i = ctx.thread_id(); i < kTileElems; i += ctx.block_threads()) {
      std::int64_t const at = base + i;
      if (task.value == 0) {
        x[at] = static_cast<float>(work.tile_id) + static_cast<float>(i) / 1024.0f;
      } else if (task.value == 1) {
        y[at] = 2.0f * x[at];
      } else if (task.value == 2) {
        z[at] = x[at] + y[at];
      }
    }
  }
};

int check(cudaError_t e, char const *what) {
  if (e != cudaSuccess) {
    std::printf("%s: %s\n", what, cudaGetErrorString(e));
    return 2;
  }
  return 0;
}

}  // namespace

int main() {
  namespace rt = megacu::runtime;
  namespace co = megacu::runtime::co_resident;
  namespace dev = megacu::scheduler::device;
  std::size_t const elems = static_cast<std::size_t>(kTiles) * kTileElems;
  float *x = nullptr, *y = nullptr, *z = nullptr;
  int *e0 = nullptr, *e1 = nullptr;
  dev::co_resident_state *state = nullptr;
  if (check(cudaMalloc(&x, elems * 4), "malloc") || check(cudaMalloc(&y, elems * 4), "malloc") ||
      check(cudaMalloc(&z, elems * 4), "malloc") || check(cudaMalloc(&e0, kTiles * 4), "malloc") ||
      check(cudaMalloc(&e1, kTiles * 4), "malloc") ||
      check(cudaMalloc(&state, sizeof(dev::co_resident_state)), "malloc")) {
    return 2;
  }
  cudaMemset(e0, 0, kTiles * 4);
  cudaMemset(e1, 0, kTiles * 4);

  fake_driver driver{};
  auto phase = rt::make_phase(driver, rt::progress_model::co_resident_persistent);
  auto ready_x = phase.event_tensor(rt::attrs(
      rt::events::shape(1, kTiles), megacu::cuda_nvshmem::events::symmetric_i32_storage(e0)));
  auto ready_y = phase.event_tensor(rt::attrs(
      rt::events::shape(1, kTiles), megacu::cuda_nvshmem::events::symmetric_i32_storage(e1)));
  auto fill = phase.submit(rt::op("fill", &op_fill), x,
                           rt::attrs(rt::dispatcher::tile_grid(1, kTiles),
                                     rt::events::publish(ready_x)));
  auto scale = phase.submit(rt::op("scale", &op_scale), static_cast<float const *>(x), y,
                            rt::attrs(rt::scheduler::depends_on(fill),
                                      rt::events::acquire(ready_x),
                                      rt::events::publish(ready_y)));
  phase.submit(rt::op("sum", &op_sum), static_cast<float const *>(x),
               static_cast<float const *>(y), z,
               rt::attrs(rt::scheduler::depends_on(fill), rt::scheduler::depends_on(scale),
                         rt::events::acquire(ready_x), rt::events::acquire(ready_y)));
  co::graph g;
  megacu::status st = co::lower_phase(g, phase.tasks(), phase.event_tensors(), phase.progress());
  if (st.code != megacu::status_code::ok) {
    std::printf("lowering: %d/%d %s\n", static_cast<int>(st.code), st.detail,
                st.message ? st.message : "");
    return 2;
  }
  if (g.units != 3 * kTiles || g.nodes[1].wait_nodes != 0 || g.nodes[2].wait_nodes != 0) {
    std::printf("unexpected graph: %lld units\n", static_cast<long long>(g.units));
    return 1;
  }
  megacu::nvshmem::peer_table peers{};
  peers.n_pes = 1;
  peers.my_pe = 0;
  if (check(dev::launch_co_resident(g, state, operators{x, y, z}, peers, 5000000000ull, 0, 256,
                                    nullptr),
            "launch") ||
      check(cudaDeviceSynchronize(), "kernel")) {
    return 2;
  }
  unsigned int error = 1;
  cudaMemcpy(&error, &state->error, 4, cudaMemcpyDeviceToHost);
  std::vector<float> host(elems);
  cudaMemcpy(host.data(), z, elems * 4, cudaMemcpyDeviceToHost);
  for (int t = 0; t < kTiles; ++t) {
    for (int i = 0; i < kTileElems; ++i) {
      float const want = 3.0f * (static_cast<float>(t) + static_cast<float>(i) / 1024.0f);
      float const got = host[static_cast<std::size_t>(t) * kTileElems + i];
      if (std::fabs(got - want) > 1e-4f * std::fabs(want) + 1e-6f) {
        std::printf("z[%d][%d] = %g, want %g\n", t, i, got, want);
        return 1;
      }
    }
  }
  if (error != 0) {
    std::printf("a wait gave up\n");
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
