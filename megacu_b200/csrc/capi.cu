// C ABI of megacu_b200: validation, tile planning, TMA descriptors, team
// (symmetric heap) management and the launchers of the sm_100a megakernels.
//
// Error convention follows megacu's native launcher
// (megacu_gemm_allreduce_phased.cu:34-49,157-232): status by value, detail
// codes per site (1 invalid problem, 2 missing storage, 10 cudaSetDevice,
// 11 memset, 12 team barrier, 13 remote PEs without a team backend,
// 14 launch), a null stream validates only. Detail codes 20+ are B200
// additions and are listed in megacu_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <mutex>

#include <megacu/backends/nvshmem.h>
#include <megacu/backends/nvshmem/cuda_event_tensor.cuh>
#include <megacu/dispatcher/tile_grid_device.cuh>
#include <megacu/gemm_allreduce.h>
#include <megacu/platform/cuda/megakernel.cuh>
#include <megacu/runtime.h>
#include <megacu/runtime/co_resident.h>
#include <megacu/runtime/device_entry.cuh>
#include <megacu/scheduler/co_resident_device.cuh>
#include <megacu/scheduler/explicit_asap_device.cuh>
#include <megacu/views.h>
#include <megacu_b200.h>

#include "kernels/gemm_ar_kernel.cuh"
#include "kernels/launch.cuh"
#include "team.h"
#include "tma_map.h"

// ---- the C structs are the C++ types, byte for byte --------------------------
static_assert(sizeof(megacu_status) == sizeof(megacu::status), "status layout");
static_assert(offsetof(megacu_status, detail) == offsetof(megacu::status, detail), "status");
static_assert(offsetof(megacu_status, message) == offsetof(megacu::status, message), "status");
static_assert(sizeof(megacu_driver_view) == sizeof(megacu::cuda_nvshmem::driver_view), "driver");
static_assert(offsetof(megacu_driver_view, team) == offsetof(megacu::cuda_nvshmem::driver_view, team),
              "driver");
static_assert(offsetof(megacu_team_view, session) == offsetof(megacu::nvshmem::team_view, session),
              "team_view");
static_assert(offsetof(megacu_team_view, owner) == offsetof(megacu::nvshmem::team_view, owner),
              "team_view");
static_assert(sizeof(megacu_gemm_ar_problem) == sizeof(gemm_ar_problem), "problem");

namespace {

using namespace megacu_b200;

constexpr int kMaxDevices = 64;

megacu_status ok_status() { return {MEGACU_OK, 0, nullptr}; }

megacu_status fail(megacu_status_code code, std::uint16_t detail, char const *msg) {
  return {static_cast<std::uint8_t>(code), detail, msg};
}

megacu_status cuda_fail(cudaError_t e, std::uint16_t detail) {
  return {MEGACU_LAUNCH_ERROR, detail, cudaGetErrorString(e)};
}

megacu::status to_cpp(megacu_status s) {
  megacu::status out;
  std::memcpy(&out, &s, sizeof(out));
  return out;
}

megacu_status to_c(megacu::status s) {
  megacu_status out;
  std::memcpy(&out, &s, sizeof(out));
  return out;
}

megacu::cuda_nvshmem::driver_view to_cpp(megacu_driver_view d) {
  megacu::cuda_nvshmem::driver_view out;
  std::memcpy(&out, &d, sizeof(out));
  return out;
}

megacu_driver_view to_c(megacu::cuda_nvshmem::driver_view d) {
  megacu_driver_view out;
  std::memcpy(&out, &d, sizeof(out));
  return out;
}

int sm_count(int device) {
  // Host threads may race here harmlessly: all store the same value.
  static std::atomic<int> cached[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) return 148;
  int n = cached[device].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) {
      n = 148;
    }
    cached[device].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace

namespace megacu_b200 {

cudaError_t launch_bf16_plan(bool wire_f32, int tile_n, bool pairs, int device, int grid,
                             cudaStream_t stream, CUtensorMap const &ma, CUtensorMap const &mb,
                             gemm_ar_params const &prm) {
  return wire_f32 ? launch_gemm_ar<true>(tile_n, pairs, device, grid, stream, ma, mb, prm)
                  : launch_gemm_ar<false>(tile_n, pairs, device, grid, stream, ma, mb, prm);
}

}  // namespace megacu_b200

namespace {

using namespace megacu_b200;

// ---- plan of one bf16 call ---------------------------------------------------

struct bf16_plan {
  std::int32_t tile_n = 256;
  std::int32_t m_tiles = 0, n_tiles = 0, tiles = 0;
  std::int32_t one_shot = 0;
  std::int32_t slots_per_src = 0;
  std::int32_t group_m = 16;
  std::int32_t wire_bytes = 2;
  std::int32_t pairs = 0;       // 1: 2-CTA clusters compute 256-row pair tiles
  std::int32_t gemm_units = 0;  // GEMM tickets per call (tiles, or pair tiles)
  std::int32_t chunk_rows = 0;  // all-gather: rows per copy chunk
  std::int32_t chunks_per_block = 0;
  std::int64_t workspace_bytes = 0;
  std::int64_t events_bytes = 0;
};

// The device schedule's mode of a problem's mode.
std::int32_t sched_mode(std::int32_t mode) {
  return mode == MEGACU_MODE_REDUCE_SCATTER ? mode_reduce_scatter
         : mode == MEGACU_MODE_ALLGATHER    ? mode_allgather
                                            : mode_allreduce;
}



constexpr std::int32_t kPlanSms = 148;  // plans must not depend on the local device
constexpr std::int32_t kSwitchCommWarps = 1;

// One tile row (m <= 128, e.g. decode shapes): every CTA runs all of K for
// its tile, and a tcgen05.mma of a narrow tile costs about as much as a wide
// one, so the time goes with the k-blocks per CTA. The tile width and K split
// (gemm_ar_params::k_split: 1 or 2 CTAs per tile, a cluster) chosen here
// keep the most of `sms` SMs busy, then split K. A split needs two k-blocks
// per CTA at least, and the other rank's accumulator rows (active 32-row
// quarters x tile_n fp32) must fit rank 0's stage ring. (Measured on one
// B200 at M 16-128, N 8192, K 3584, CUDA-graph replays: tile_n 128 split in
// two 28.8-30.7 us, tile_n 64 unsplit 30.7 us, tile_n 256 split in four
// 32.8-36.9 us: the four-way reduction and the HBM contention of four CTAs
// streaming one column panel cost more than they save.)
struct row_split {
  std::int32_t tile_n;
  std::int32_t k_split;
};

row_split one_row_split(std::int64_t m, std::int64_t n, std::int64_t k, std::int32_t sms,
                        std::int32_t tile_n) {
  std::int64_t const rows = m < kBlockM ? m : kBlockM;
  std::int64_t const quarters = (rows + 31) / 32;
  std::int64_t const k_blocks = (k + kBlockK - 1) / kBlockK;
  row_split best{tile_n != 0 ? tile_n : 64, 1};
  std::int64_t best_ctas = -1;
  for (std::int32_t tn : {256, 128, 64}) {
    if (tile_n != 0 && tn != tile_n) continue;
    std::int64_t const tiles = (n + tn - 1) / tn;
    for (std::int32_t ks : {2, 1}) {
      bool const fits =
          ks == 1 || (tiles * ks <= sms && k_blocks >= 2 * ks &&
                      (ks - 1) * quarters * 32 * tn * 4 <= gemm_config<64>::ring_bytes);
      if (!fits) continue;
      std::int64_t const ctas = (tiles < sms ? tiles : sms) * ks;
      if (ctas > best_ctas || (ctas == best_ctas && ks > best.k_split)) {
        best = {tn, ks};
        best_ctas = ctas;
      }
      break;  // the largest split that fits this width
    }
  }
  return best;
}

megacu_status make_plan(megacu_gemm_ar_problem_v2 const &p, std::int32_t n_pes, bf16_plan &out) {
  if (p.m <= 0 || p.n <= 0 || p.k <= 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "invalid problem");
  }
  if (p.dtype != MEGACU_DTYPE_BF16) {
    return fail(MEGACU_UNSUPPORTED, 20, "bf16 megakernel needs dtype bf16");
  }
  if (p.n % 8 != 0 || p.k % 8 != 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 21, "n and k must be multiples of 8 (16-byte rows)");
  }
  if (p.m > (1ll << 30) || p.n > (1ll << 30) || p.k > (1ll << 30)) {
    return fail(MEGACU_UNSUPPORTED, 22, "dimension too large");
  }
  if (n_pes < 1 || n_pes > megacu::nvshmem::max_team_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "team size must be 1..8");
  }
  if (p.tile_m != 0 && p.tile_m != kBlockM) {
    return fail(MEGACU_UNSUPPORTED, 22, "tile_m must be 0 or 128");
  }
  if (p.mode != MEGACU_MODE_ALLREDUCE && p.mode != MEGACU_MODE_REDUCE_SCATTER &&
      p.mode != MEGACU_MODE_ALLGATHER) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "unknown mode");
  }
  if (p.algo < MEGACU_ALGO_AUTO || p.algo > MEGACU_ALGO_TWO_SHOT) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "unknown algo");
  }
  if (p.cta_pairs < MEGACU_CTA_PAIRS_AUTO || p.cta_pairs > MEGACU_CTA_PAIRS_ON) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "unknown cta_pairs");
  }
  bf16_plan pl;
  pl.m_tiles = static_cast<std::int32_t>((p.m + kBlockM - 1) / kBlockM);
  if (p.tile_n != 0) {
    if (p.tile_n != 64 && p.tile_n != 128 && p.tile_n != 256) {
      return fail(MEGACU_UNSUPPORTED, 22, "tile_n must be 0, 64, 128 or 256");
    }
    pl.tile_n = p.tile_n;
  } else if (pl.m_tiles == 1 && p.mode != MEGACU_MODE_ALLGATHER) {
    pl.tile_n = one_row_split(p.m, p.n, p.k, kPlanSms, 0).tile_n;
  } else {
    pl.tile_n = 64;
    for (std::int32_t cand : {256, 128}) {
      std::int64_t const t = pl.m_tiles * ((p.n + cand - 1) / cand);
      if (t >= kPlanSms) {
        pl.tile_n = cand;
        break;
      }
    }
  }
  pl.n_tiles = static_cast<std::int32_t>((p.n + pl.tile_n - 1) / pl.tile_n);
  std::int64_t const tiles = static_cast<std::int64_t>(pl.m_tiles) * pl.n_tiles;
  if (tiles > (1 << 24)) {
    return fail(MEGACU_UNSUPPORTED, 22, "too many tiles");
  }
  pl.tiles = static_cast<std::int32_t>(tiles);
  if (p.mode == MEGACU_MODE_REDUCE_SCATTER || p.mode == MEGACU_MODE_ALLGATHER) {
    if (p.m % (static_cast<std::int64_t>(n_pes) * kBlockM) != 0) {
      return fail(MEGACU_UNSUPPORTED, 26,
                  "reduce-scatter and all-gather need m divisible by tp * 128");
    }
    pl.one_shot = 0;
  } else if (n_pes == 1) {
    pl.one_shot = 0;
  } else if (p.algo == MEGACU_ALGO_ONE_SHOT) {
    pl.one_shot = 1;
  } else if (p.algo == MEGACU_ALGO_TWO_SHOT) {
    pl.one_shot = 0;
  } else {
    // One hop for latency-bound shapes (one tile row) and for two PEs, where
    // one-shot moves the same NVLink bytes as two-shot without the gather.
    pl.one_shot = (pl.m_tiles == 1 || n_pes == 2) ? 1 : 0;
  }
  // All-gather reduces nothing: its output has one rounding whatever the flag.
  pl.wire_bytes = (p.deterministic && p.mode != MEGACU_MODE_ALLGATHER) ? 4 : 2;
  // CTA pairs halve each SM's shared-memory operand traffic per MMA (256-row
  // MMAs, B split across the pair); they need pair tiles the grid can hold.
  {
    tile_schedule const sched{pl.m_tiles, pl.n_tiles, n_pes, sched_mode(p.mode), pl.group_m};
    bool const can_pair = pl.tile_n >= 128 && pairs_fit(sched);
    if (p.cta_pairs == MEGACU_CTA_PAIRS_ON && !can_pair) {
      return fail(MEGACU_UNSUPPORTED, 27,
                  "CTA pairs need tile_n >= 128 and an even number of tile rows (per PE block)");
    }
    pl.pairs = (can_pair && p.cta_pairs != MEGACU_CTA_PAIRS_OFF) ? 1 : 0;
    pl.gemm_units = pl.pairs ? pl.tiles / 2 : pl.tiles;
  }
  if (p.mode == MEGACU_MODE_ALLGATHER) {
    // No partials: the gathered A is the caller's buffer. Events: one PE's
    // arrive plane plus the gather flags and counters.
    pl.slots_per_src = 0;
    pl.workspace_bytes = 0;
    pl.chunk_rows = gather_chunk_rows(p.k);
    pl.chunks_per_block = kBlockM / pl.chunk_rows;
    pl.events_bytes = events_bytes_for_gather(n_pes, pl.tiles, pl.m_tiles / n_pes);
    out = pl;
    return ok_status();
  }
  // Each PE keeps its own partial of every tile (two parity planes); the
  // tile's reducers read it over NVLink.
  pl.slots_per_src = n_pes == 1 ? 0 : pl.tiles;
  pl.workspace_bytes =
      static_cast<std::int64_t>(2) * pl.slots_per_src * kBlockM * pl.tile_n * pl.wire_bytes;
  pl.events_bytes = events_bytes_for(n_pes, pl.tiles);
  out = pl;
  return ok_status();
}

bool aligned16(void const *p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// All-gather + GEMM: `ma` is this PE's A shard, `mg` the gathered A (both
// with 128-row boxes), `mb` the B operand.
cudaError_t launch_allgather(int tile_n, bool pairs, int device, int grid, cudaStream_t stream,
                             CUtensorMap const &ma, CUtensorMap const &mb, CUtensorMap const &mg,
                             gemm_ar_params const &prm) {
  switch (tile_n) {
    case 256:
      return pairs ? launch_variant<256, false, true, false, true>(device, grid, stream, ma, mb,
                                                                   mg, prm)
                   : launch_variant<256, false, false, false, true>(device, grid, stream, ma, mb,
                                                                    mg, prm);
    case 128:
      return pairs ? launch_variant<128, false, true, false, true>(device, grid, stream, ma, mb,
                                                                   mg, prm)
                   : launch_variant<128, false, false, false, true>(device, grid, stream, ma, mb,
                                                                    mg, prm);
    default:
      return launch_variant<64, false, false, false, true>(device, grid, stream, ma, mb, mg, prm);
  }
}

megacu_status run_bf16(megacu_driver_view driver, void const *a, void const *b, void *workspace,
                       void *out, void *events, megacu_gemm_ar_problem_v2 problem) {
  std::int32_t const n_pes = driver.team.team_n_pes;
  if (problem.mode == MEGACU_MODE_ALLGATHER) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "all-gather runs through megacu_cuda_allgather_gemm_bf16");
  }
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code != MEGACU_OK) return st;
  if (a == nullptr || b == nullptr || out == nullptr || events == nullptr ||
      (n_pes > 1 && workspace == nullptr)) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  if (!aligned16(a) || !aligned16(b) || !aligned16(out) || !aligned16(events) ||
      (workspace != nullptr && !aligned16(workspace))) {
    return fail(MEGACU_INVALID_ARGUMENT, 21, "buffers must be 16-byte aligned");
  }
  std::int32_t const my_pe = driver.team.team_my_pe;
  if (my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "team_my_pe out of range");
  }
  team_impl *team = nullptr;
  bool via_switch = false;
  // Two-shot allreduce: every owner stores its sums into every PE's out.
  bool const out_symmetric = n_pes > 1 && problem.mode == MEGACU_MODE_ALLREDUCE && !pl.one_shot;
  if (n_pes > 1) {
    team = as_team(driver.team.team);
    if (team == nullptr) {
      return fail(MEGACU_UNSUPPORTED, 13, "remote PEs need a megacu_b200 team in team_view.team");
    }
    if (!team->connected || team->n_pes != n_pes || team->my_pe != my_pe) {
      return fail(MEGACU_INVALID_ARGUMENT, 24, "team handle does not match team_view");
    }
    std::int64_t const out_bytes = problem.m * problem.n * 2;
    // A workspace in the multicast region selects the in-switch reduction
    // (bf16 wire): a reducer reads every PE's partial of a block with one
    // load, summed by the NVSwitch. A two-shot allreduce also stores each
    // sum through the switch into every PE's out, so its out must lie in the
    // region too; one-shot and reduce-scatter store into this PE's own out.
    bool const ws_mc = team->mc.contains(workspace, pl.workspace_bytes);
    bool const out_mc = team->mc.contains(out, out_bytes);
    if (ws_mc || (out_symmetric && out_mc)) {
      if (!ws_mc || pl.wire_bytes != 2 || (out_symmetric && !out_mc)) {
        return fail(MEGACU_UNSUPPORTED, 28,
                    "in-switch reduction needs the bf16 wire and the workspace (for a two-shot "
                    "allreduce also out) in the multicast region");
      }
      via_switch = true;
    }
    if (!(ws_mc || team->contains(workspace, pl.workspace_bytes)) ||
        !team->contains(events, pl.events_bytes) ||
        (out_symmetric && !(out_mc || team->contains(out, out_bytes)))) {
      return fail(MEGACU_INVALID_ARGUMENT, 25,
                  "workspace, events (and two-shot out) must lie in the team's symmetric heap "
                  "(workspace and out may lie in its multicast region)");
    }
  }
  if (!megacu::cuda::has_stream(megacu::cuda::launch_view{driver.launch.stream,
                                                          driver.launch.device_ordinal})) {
    return ok_status();
  }
  int const device = driver.launch.device_ordinal;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  if (team != nullptr && team->device != device) {
    return fail(MEGACU_INVALID_ARGUMENT, 24, "team was created on another device");
  }

  // One tile row (m < 128, decode shapes): each load brings only the rows of
  // A that exist (rounded up to 8), so the ring holds more, smaller stages.
  std::int32_t const a_box_rows =
      (problem.m < kBlockM && !pl.pairs) ? static_cast<std::int32_t>((problem.m + 7) / 8 * 8)
                                         : kBlockM;
  CUtensorMap map_a, map_b;
  if (!encode_bf16_map(&map_a, a, problem.m, problem.k, static_cast<std::uint32_t>(a_box_rows)) ||
      !encode_bf16_map(&map_b, b, problem.k, problem.n, kBlockK)) {
    return fail(MEGACU_BACKEND_ERROR, 30, "cuTensorMapEncodeTiled failed");
  }

  gemm_ar_params prm{};
  prm.a_box_rows = a_box_rows;
  prm.m = static_cast<std::int32_t>(problem.m);
  prm.n = static_cast<std::int32_t>(problem.n);
  prm.k = static_cast<std::int32_t>(problem.k);
  prm.m_tiles = pl.m_tiles;
  prm.n_tiles = pl.n_tiles;
  prm.tiles = pl.tiles;
  prm.n_pes = n_pes;
  prm.my_pe = my_pe;
  prm.mode = problem.mode == MEGACU_MODE_REDUCE_SCATTER ? mode_reduce_scatter : mode_allreduce;
  prm.one_shot = pl.one_shot;
  prm.group_m = pl.group_m;
  // The reduce queue: every (reduced tile, 32-row quarter, 64-column block),
  // the reduced tiles being this PE's own (two-shot, reduce-scatter) or all
  // tiles (one-shot), in raster order. The in-switch reduction hands out
  // (tile, quarter) tickets and reduces their blocks in order.
  tile_schedule const sched{pl.m_tiles, pl.n_tiles, n_pes, prm.mode, pl.group_m};
  std::int32_t const reduced_tiles =
      n_pes == 1 ? 0 : (pl.one_shot ? pl.tiles : owned_tiles(sched, my_pe));
  prm.n_comm = reduced_tiles * kQuarters * (via_switch ? 1 : pl.tile_n / 64);
  // One-shot peer exchange of one tile row, bf16 wire: 16-column slices.
  prm.comm_slices = (pl.one_shot && pl.m_tiles == 1 && !via_switch && pl.wire_bytes == 2 &&
                     prm.mode == mode_allreduce)
                        ? 1
                        : 0;
  if (prm.comm_slices) prm.n_comm *= 4;
  // Warps per CTA running exchange sub-tasks. The in-switch reduction
  // saturates the fabric with one per SM; more only lengthen its queues and
  // with them every sub-task's latency and the drain at the end (tp = 8, C2:
  // 184.3 us with 1, 195.0 with 2, 201.7 with 3, 209.9 with 4, 223.7 with
  // 8). Peer loads and stores need more in flight (240.6 us with 4 or 6,
  // 244.7 with 8, 279.5 with 2).
  prm.comm_warps = via_switch ? kSwitchCommWarps : kWorkerWarps;
  prm.rows_per_pe = static_cast<std::int32_t>(problem.m / n_pes);
  prm.timeout_ns = problem.timeout_ns != 0 ? problem.timeout_ns : 10000000000ull;
  prm.out = static_cast<__nv_bfloat16 *>(out);
  prm.workspace = static_cast<char *>(workspace);
  prm.events = static_cast<std::uint32_t *>(events);
  if (via_switch) {
    prm.mc_workspace = team->mc.alias(workspace);
    if (out_symmetric) prm.mc_out = reinterpret_cast<__nv_bfloat16 *>(team->mc.alias(out));
  }
  if (team != nullptr) {
    prm.peers = team->peers;
  } else {
    prm.peers.n_pes = 1;
    prm.peers.my_pe = 0;
  }
  prm.trace = reinterpret_cast<unsigned long long *>(problem.trace);
  prm.trace_capacity = problem.trace != nullptr ? problem.trace_capacity : 0;

  int grid = problem.num_ctas > 0 ? problem.num_ctas : sm_count(device);
  if (pl.m_tiles == 1 && !pl.pairs && problem.num_ctas <= 0) {
    prm.k_split = one_row_split(problem.m, problem.n, problem.k, grid, pl.tile_n).k_split;
  }
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);
  bool const f32 = pl.wire_bytes == 4;
  e = launch_bf16_plan(f32, pl.tile_n, pl.pairs != 0, device, grid, stream, map_a, map_b, prm);
  if (e != cudaSuccess) return cuda_fail(e, 14);
  return ok_status();
}

// All-gather + GEMM: gathered = every PE's a_shard in PE order, out =
// gathered @ b (this PE's columns). Validation and launch as run_bf16.
megacu_status run_allgather(megacu_driver_view driver, void const *a_shard, void const *b,
                            void *gathered, void *out, void *events,
                            megacu_gemm_ar_problem_v2 problem) {
  std::int32_t const n_pes = driver.team.team_n_pes;
  problem.mode = MEGACU_MODE_ALLGATHER;
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code != MEGACU_OK) return st;
  if (a_shard == nullptr || b == nullptr || gathered == nullptr || out == nullptr ||
      events == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  if (!aligned16(a_shard) || !aligned16(b) || !aligned16(gathered) || !aligned16(out) ||
      !aligned16(events)) {
    return fail(MEGACU_INVALID_ARGUMENT, 21, "buffers must be 16-byte aligned");
  }
  std::int32_t const my_pe = driver.team.team_my_pe;
  if (my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "team_my_pe out of range");
  }
  std::int64_t const rows_per_pe = problem.m / n_pes;
  team_impl *team = nullptr;
  if (n_pes > 1) {
    team = as_team(driver.team.team);
    if (team == nullptr) {
      return fail(MEGACU_UNSUPPORTED, 13, "remote PEs need a megacu_b200 team in team_view.team");
    }
    if (!team->connected || team->n_pes != n_pes || team->my_pe != my_pe) {
      return fail(MEGACU_INVALID_ARGUMENT, 24, "team handle does not match team_view");
    }
    if (!team->contains(a_shard, rows_per_pe * problem.k * 2) ||
        !team->contains(events, pl.events_bytes)) {
      return fail(MEGACU_INVALID_ARGUMENT, 25,
                  "a_shard and events must lie in the team's symmetric heap");
    }
  }
  if (!megacu::cuda::has_stream(megacu::cuda::launch_view{driver.launch.stream,
                                                          driver.launch.device_ordinal})) {
    return ok_status();
  }
  int const device = driver.launch.device_ordinal;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  if (team != nullptr && team->device != device) {
    return fail(MEGACU_INVALID_ARGUMENT, 24, "team was created on another device");
  }

  CUtensorMap map_a, map_b, map_g;
  if (!encode_bf16_map(&map_a, a_shard, rows_per_pe, problem.k, kBlockM) ||
      !encode_bf16_map(&map_b, b, problem.k, problem.n, kBlockK) ||
      !encode_bf16_map(&map_g, gathered, problem.m, problem.k, kBlockM)) {
    return fail(MEGACU_BACKEND_ERROR, 30, "cuTensorMapEncodeTiled failed");
  }

  gemm_ar_params prm{};
  prm.m = static_cast<std::int32_t>(problem.m);
  prm.n = static_cast<std::int32_t>(problem.n);
  prm.k = static_cast<std::int32_t>(problem.k);
  prm.m_tiles = pl.m_tiles;
  prm.n_tiles = pl.n_tiles;
  prm.tiles = pl.tiles;
  prm.n_pes = n_pes;
  prm.my_pe = my_pe;
  prm.mode = mode_allgather;
  prm.one_shot = 0;
  prm.group_m = pl.group_m;
  // The copy queue: every chunk of every shard (this PE's own last).
  prm.n_comm = n_pes * (pl.m_tiles / n_pes) * pl.chunks_per_block;
  // The dedicated worker warps copy from the start; the GEMM needs the rows
  // well before the epilogue warps would be free to help.
  prm.comm_warps = kReduceWarps;
  prm.rows_per_pe = static_cast<std::int32_t>(rows_per_pe);
  prm.timeout_ns = problem.timeout_ns != 0 ? problem.timeout_ns : 10000000000ull;
  prm.out = static_cast<__nv_bfloat16 *>(out);
  prm.workspace = nullptr;
  prm.events = static_cast<std::uint32_t *>(events);
  if (team != nullptr) {
    prm.peers = team->peers;
  } else {
    prm.peers.n_pes = 1;
    prm.peers.my_pe = 0;
  }
  prm.trace = reinterpret_cast<unsigned long long *>(problem.trace);
  prm.trace_capacity = problem.trace != nullptr ? problem.trace_capacity : 0;
  prm.a_shard = static_cast<__nv_bfloat16 const *>(a_shard);
  prm.gathered = static_cast<__nv_bfloat16 *>(gathered);
  prm.chunk_rows = pl.chunk_rows;
  prm.chunks_per_block = pl.chunks_per_block;

  int grid = problem.num_ctas > 0 ? problem.num_ctas : sm_count(device);
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);
  e = launch_allgather(pl.tile_n, pl.pairs != 0, device, grid, stream, map_a, map_b, map_g, prm);
  if (e != cudaSuccess) return cuda_fail(e, 14);
  return ok_status();
}

// ---- team barrier (host-ordered, device-executed) -----------------------------

// Every PE writes `epoch` into every peer's slot for it, then waits until
// all peers' slots for it reached `epoch`. Bounded; a timeout sets the
// team's error word (reserved heap word 32) instead of hanging.
__global__ void team_barrier_kernel(megacu::nvshmem::peer_table peers, std::uint32_t epoch,
                                    std::uint64_t timeout_ns) {
  auto *mine = reinterpret_cast<std::uint32_t *>(peers.base[peers.my_pe]);
  int const lane = threadIdx.x;
  ptx::fence_acq_rel_sys();
  if (lane < peers.n_pes) {
    auto *theirs = reinterpret_cast<std::uint32_t *>(peers.base[lane]);
    ptx::st_release_sys(theirs + peers.my_pe, epoch);
    std::uint64_t const start = ptx::now_ns();
    for (std::uint32_t spin = 0;; ++spin) {
      std::uint32_t const v = ptx::ld_acquire_sys(mine + lane);
      if (static_cast<std::int32_t>(v - epoch) >= 0) break;
      __nanosleep(64);
      if ((spin & 15u) == 0 && ptx::now_ns() - start > timeout_ns) {
        atomicExch(mine + 32, 1u);
        break;
      }
    }
  }
}

megacu_status team_barrier(team_impl *team, cudaStream_t stream) {
  std::uint32_t epoch;
  {
    std::lock_guard<std::mutex> lock(team->mu);
    epoch = ++team->barrier_epoch;
  }
  team_barrier_kernel<<<1, 32, 0, stream>>>(team->peers, epoch, 10000000000ull);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ok_status() : cuda_fail(e, 12);
}

// ---- fp32 phased path (megacu's launcher, on the generic device loop) -------

struct f32_gemm_tile_task {
  float const *a;
  float const *b;
  float *partial;
  gemm_ar_problem problem;

  // partial[r, c] = sum_k a[r, k] * b[k, c], k ascending, one fp32 FMA per
  // step: the order of megacu_gemm_allreduce_phased.cu:83-85.
  template <class Context>
  __device__ void operator()(Context ctx, std::int64_t tile_id) const {
    std::int64_t const n_tiles = (problem.n + problem.tile_n - 1) / problem.tile_n;
    std::int64_t const row0 = (tile_id / n_tiles) * problem.tile_m;
    std::int64_t const col0 = (tile_id % n_tiles) * problem.tile_n;
    std::int64_t const elems = static_cast<std::int64_t>(problem.tile_m) * problem.tile_n;
    for (std::int64_t e = ctx.thread_id(); e < elems; e += ctx.block_threads()) {
      std::int64_t const row = row0 + e / problem.tile_n;
      std::int64_t const col = col0 + e % problem.tile_n;
      if (row >= problem.m || col >= problem.n) continue;
      float acc = 0.0f;
      for (std::int64_t kk = 0; kk < problem.k; ++kk) {
        acc = fmaf(a[row * problem.k + kk], b[kk * problem.n + col], acc);
      }
      partial[row * problem.n + col] = acc;
    }
  }
};

struct f32_allreduce_tile_task {
  float *partial;
  float *out;
  gemm_ar_problem problem;
  megacu::nvshmem::peer_table peers;

  // out[i] = sum over PEs in PE order of partial_pe[i]
  // (megacu_gemm_allreduce_phased.cu:118-130); peers' partials are read
  // over NVLink with plain loads.
  template <class Context>
  __device__ void operator()(Context ctx, std::int64_t tile_id) const {
    std::int64_t const n_tiles = (problem.n + problem.tile_n - 1) / problem.tile_n;
    std::int64_t const row0 = (tile_id / n_tiles) * problem.tile_m;
    std::int64_t const col0 = (tile_id % n_tiles) * problem.tile_n;
    std::int64_t const elems = static_cast<std::int64_t>(problem.tile_m) * problem.tile_n;
    for (std::int64_t e = ctx.thread_id(); e < elems; e += ctx.block_threads()) {
      std::int64_t const row = row0 + e / problem.tile_n;
      std::int64_t const col = col0 + e % problem.tile_n;
      if (row >= problem.m || col >= problem.n) continue;
      std::int64_t const idx = row * problem.n + col;
      float sum = 0.0f;
      for (int pe = 0; pe < peers.n_pes; ++pe) {
        sum += pe == peers.my_pe ? *reinterpret_cast<float volatile *>(partial + idx)
                                 : megacu::nvshmem::device::remote_float(partial, idx, pe, peers);
      }
      out[idx] = sum;
    }
  }
};

struct f32_operators {
  f32_gemm_tile_task producer;
  f32_allreduce_tile_task consumer;

  template <class Context, class Task, class Work>
  __device__ void invoke(Context ctx, Task task, Work work) const {
    if (task.value == 0) {
      producer(ctx, work.tile_id);
    } else if (task.value == 2) {
      consumer(ctx, work.tile_id);
    }
  }
};

struct f32_program {
  megacu::nvshmem::peer_table peers;
  megacu::runtime::device::entry<megacu::scheduler::device::explicit_asap,
                                 megacu::dispatcher::device::tile_grid,
                                 megacu::backend::nvshmem::cuda::task_event_tensor_i32,
                                 f32_operators>
      entry;

  template <class Context>
  __device__ void operator()(Context ctx) const {
    // The event tensor keeps a pointer to the peer table; give it this
    // kernel's own copy (kernel parameters live in constant space).
    auto local = entry;
    local.backend.event_tensor.peers = &peers;
    local(ctx);
  }
};

// The operator table of the co-resident fp32 graph: node 0 is the GEMM tile
// producer, node 1 the allreduce tile consumer (the phase's operator tasks
// in submission order; the sync task is no node).
struct f32_graph_operators {
  f32_gemm_tile_task producer;
  f32_allreduce_tile_task consumer;

  template <class Context, class Task, class Work>
  __device__ void invoke(Context ctx, Task task, Work work) const {
    if (task.value == 0) {
      producer(ctx, work.tile_id);
    } else if (task.value == 1) {
      consumer(ctx, work.tile_id);
    }
  }
};

}  // namespace

// ============================================================================
// extern "C" entry points
// ============================================================================

extern "C" megacu_status megacu_cuda_gemm_allreduce_phased_f32(megacu_driver_view driver,
                                                               float const *a, float const *b,
                                                               float *partial, float *out,
                                                               void *events,
                                                               megacu_gemm_ar_problem problem) {
  if (problem.m <= 0 || problem.n <= 0 || problem.k <= 0 || problem.tile_m <= 0 ||
      problem.tile_n <= 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "invalid problem");
  }
  if (a == nullptr || b == nullptr || partial == nullptr || out == nullptr || events == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  std::int32_t const n_pes = driver.team.team_n_pes;
  std::int32_t const my_pe = driver.team.team_my_pe;
  if (n_pes < 1 || n_pes > megacu::nvshmem::max_team_pes || my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "invalid team shape");
  }
  if (driver.launch.stream == nullptr) {
    return ok_status();
  }
  std::int64_t const tiles = ((problem.m + problem.tile_m - 1) / problem.tile_m) *
                             ((problem.n + problem.tile_n - 1) / problem.tile_n);
  team_impl *team = nullptr;
  if (n_pes > 1) {
    team = as_team(driver.team.team);
    if (team == nullptr || !team->connected) {
      return fail(MEGACU_UNSUPPORTED, 13, "device-side remote path needs a megacu_b200 team");
    }
    if (team->n_pes != n_pes || team->my_pe != my_pe) {
      return fail(MEGACU_INVALID_ARGUMENT, 24, "team handle does not match team_view");
    }
    if (!team->contains(partial, problem.m * problem.n * 4) ||
        !team->contains(events, tiles * n_pes * 4)) {
      return fail(MEGACU_INVALID_ARGUMENT, 25, "partial and events must be symmetric");
    }
  }
  int const device = driver.launch.device_ordinal;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);

  e = cudaMemsetAsync(events, 0, tiles * n_pes * sizeof(int), stream);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  if (team != nullptr) {
    megacu_status st = team_barrier(team, stream);
    if (st.code != MEGACU_OK) return st;
  }

  f32_program program{};
  if (team != nullptr) {
    program.peers = team->peers;
  } else {
    program.peers.n_pes = 1;
    program.peers.my_pe = 0;
  }
  gemm_ar_problem prob;
  std::memcpy(&prob, &problem, sizeof(prob));
  program.entry.scheduler.task_count = 3;
  program.entry.dispatcher.tiles = tiles;
  auto &ev = program.entry.backend;
  ev.event_tensor.events = static_cast<int *>(events);
  ev.event_tensor.tiles = tiles;
  ev.event_tensor.my_pe = my_pe;
  ev.event_tensor.n_pes = n_pes;
  ev.publish_task = 0;
  ev.acquire_task = 2;
  program.entry.operators.producer = {a, b, partial, prob};
  program.entry.operators.consumer = {partial, out, prob, program.peers};

  int blocks = static_cast<int>(std::min<std::int64_t>(tiles, sm_count(device)));
  megacu::platform::cuda::launch_config cfg;
  cfg.blocks = blocks;
  cfg.threads = 256;
  cfg.cooperative = n_pes > 1;
  e = megacu::platform::cuda::launch_megakernel(stream, cfg, program);
  if (e != cudaSuccess) return cuda_fail(e, 14);
  if (team != nullptr) {
    // Peers may still be reading this PE's partial: nobody returns to a
    // state where `partial` can be overwritten before everyone is done.
    megacu_status st = team_barrier(team, stream);
    if (st.code != MEGACU_OK) return st;
  }
  return ok_status();
}

extern "C" megacu_status megacu_cuda_gemm_allreduce_bf16(megacu_driver_view driver, void const *a,
                                                         void const *b, void *workspace,
                                                         void *out, void *events,
                                                         megacu_gemm_ar_problem_v2 problem) {
  problem.mode = MEGACU_MODE_ALLREDUCE;
  return run_bf16(driver, a, b, workspace, out, events, problem);
}

extern "C" megacu_status megacu_cuda_gemm_reduce_scatter_bf16(
    megacu_driver_view driver, void const *a, void const *b, void *workspace, void *out,
    void *events, megacu_gemm_ar_problem_v2 problem) {
  problem.mode = MEGACU_MODE_REDUCE_SCATTER;
  return run_bf16(driver, a, b, workspace, out, events, problem);
}

extern "C" megacu_status megacu_cuda_allgather_gemm_bf16(megacu_driver_view driver,
                                                         void const *a_shard, void const *b,
                                                         void *gathered, void *out, void *events,
                                                         megacu_gemm_ar_problem_v2 problem) {
  return run_allgather(driver, a_shard, b, gathered, out, events, problem);
}

namespace {

using bf16_gemm_sig = megacu::status(megacu::cuda_nvshmem::driver_view, void const *, void const *,
                                     void *, megacu_gemm_ar_problem_v2);
using bf16_reduce_sig = megacu::status(megacu::cuda_nvshmem::driver_view, void *, void *,
                                       megacu_gemm_ar_problem_v2);

megacu::status bf16_phased_launcher(megacu::cuda_nvshmem::driver_view driver, void const *a,
                                    void const *b, void *workspace, void *out, void *events,
                                    megacu_gemm_ar_problem_v2 problem) {
  return to_cpp(run_bf16(to_c(driver), a, b, workspace, out, events, problem));
}

megacu::status f32_phased_launcher(megacu::cuda_nvshmem::driver_view driver, float const *a,
                                   float const *b, float *partial, float *out, void *events,
                                   gemm_ar_problem problem) {
  megacu_gemm_ar_problem p;
  std::memcpy(&p, &problem, sizeof(p));
  return to_cpp(megacu_cuda_gemm_allreduce_phased_f32(to_c(driver), a, b, partial, out, events, p));
}

}  // namespace

extern "C" megacu_status megacu_cuda_gemm_allreduce_bf16_orchestrate(
    megacu_driver_view driver, void const *a, void const *b, void *workspace, void *out,
    void *events, megacu_gemm_ar_problem_v2 problem) {
  namespace rt = megacu::runtime;
  auto d = to_cpp(driver);
  auto phase = rt::make_phase(d, rt::progress_model::asap);
  bf16_plan pl;
  megacu_status st = make_plan(problem, driver.team.team_n_pes, pl);
  if (st.code != MEGACU_OK) return st;

  auto ready_events = phase.event_tensor(
      rt::attrs(rt::events::shape(pl.m_tiles, pl.n_tiles),
                megacu::cuda_nvshmem::events::symmetric_i32_storage(events),
                megacu::cuda_nvshmem::events::team_scope()));
  auto gemm = phase.submit(
      rt::op<bf16_gemm_sig>(ops::gemm_tile_produce::name), d, a, b, workspace, problem,
      rt::attrs(rt::dispatcher::tile_grid(pl.m_tiles, pl.n_tiles), rt::events::publish(ready_events)));
  auto ready = phase.sync(rt::attrs(rt::scheduler::depends_on(gemm), rt::events::join(ready_events)));
  phase.submit(rt::op<bf16_reduce_sig>(ops::allreduce_tile_consume::name), d, workspace, out, problem,
               rt::attrs(rt::scheduler::depends_on(ready), rt::events::acquire(ready_events)));
  return to_c(phase.run(rt::op(ops::phased_megakernel::name, &bf16_phased_launcher), d, a, b,
                        workspace, out, events, problem));
}

// megacu's orchestrate entry (C++ linkage), same phase as the reference's
// gemm_allreduce_orchestrate_common.h:24-76.
megacu::status cuda_nvshmem_gemm_allreduce_phased_orchestrate(gemm_ar_driver driver,
                                                              float const *a, float const *b,
                                                              float *partial, float *out,
                                                              void *events,
                                                              gemm_ar_problem problem) {
  namespace rt = megacu::runtime;
  using gemm_sig = megacu::status(gemm_ar_driver, float const *, float const *, float *,
                                  gemm_ar_problem);
  using reduce_sig = megacu::status(gemm_ar_driver, float *, float *, gemm_ar_problem);
  auto phase = rt::make_phase(driver, rt::progress_model::asap);
  std::int64_t const m_tiles = problem.tile_m == 0 ? 0 : (problem.m + problem.tile_m - 1) / problem.tile_m;
  std::int64_t const n_tiles = problem.tile_n == 0 ? 0 : (problem.n + problem.tile_n - 1) / problem.tile_n;
  auto ready_events = phase.event_tensor(
      rt::attrs(rt::events::shape(m_tiles, n_tiles),
                megacu::cuda_nvshmem::events::symmetric_i32_storage(events),
                megacu::cuda_nvshmem::events::team_scope()));
  auto gemm = phase.submit(rt::op<gemm_sig>(ops::gemm_tile_produce::name), driver, a, b, partial,
                           problem,
                           rt::attrs(rt::dispatcher::tile_grid(m_tiles, n_tiles),
                                     rt::events::publish(ready_events)));
  auto ready = phase.sync(rt::attrs(rt::scheduler::depends_on(gemm), rt::events::join(ready_events)));
  phase.submit(rt::op<reduce_sig>(ops::allreduce_tile_consume::name), driver, partial, out, problem,
               rt::attrs(rt::scheduler::depends_on(ready), rt::events::acquire(ready_events)));
  return phase.run(rt::op(ops::phased_megakernel::name, &f32_phased_launcher), driver, a, b,
                   partial, out, events, problem);
}

extern "C" megacu_status megacu_cuda_gemm_allreduce_f32_orchestrate(
    megacu_driver_view driver, float const *a, float const *b, float *partial, float *out,
    void *events, megacu_gemm_ar_problem problem) {
  gemm_ar_problem p;
  std::memcpy(&p, &problem, sizeof(p));
  return to_c(cuda_nvshmem_gemm_allreduce_phased_orchestrate(to_cpp(driver), a, b, partial, out,
                                                            events, p));
}

// megacu's fp32 phase (the orchestration of
// gemm_allreduce_orchestrate_common.h:24-76) with co-resident persistent
// progress: lowered to one unit graph and run as one cooperative persistent
// launch, GEMM tiles first, each allreduce tile starting as soon as every
// PE has published its partial of that tile.
extern "C" megacu_status megacu_cuda_gemm_allreduce_f32_co_resident(
    megacu_driver_view driver, float const *a, float const *b, float *partial, float *out,
    void *events, void *control, megacu_gemm_ar_problem problem) {
  namespace rt = megacu::runtime;
  namespace co = megacu::runtime::co_resident;
  if (problem.m <= 0 || problem.n <= 0 || problem.k <= 0 || problem.tile_m <= 0 ||
      problem.tile_n <= 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "invalid problem");
  }
  if (a == nullptr || b == nullptr || partial == nullptr || out == nullptr || events == nullptr ||
      control == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  std::int32_t const n_pes = driver.team.team_n_pes;
  std::int32_t const my_pe = driver.team.team_my_pe;
  if (n_pes < 1 || n_pes > megacu::nvshmem::max_team_pes || my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "invalid team shape");
  }
  std::int64_t const m_tiles = (problem.m + problem.tile_m - 1) / problem.tile_m;
  std::int64_t const n_tiles = (problem.n + problem.tile_n - 1) / problem.tile_n;
  std::int64_t const tiles = m_tiles * n_tiles;

  // The phase, as megacu's orchestration builds it, with the other progress model.
  using gemm_sig = megacu::status(gemm_ar_driver, float const *, float const *, float *,
                                  gemm_ar_problem);
  using reduce_sig = megacu::status(gemm_ar_driver, float *, float *, gemm_ar_problem);
  auto d = to_cpp(driver);
  gemm_ar_problem prob;
  std::memcpy(&prob, &problem, sizeof(prob));
  auto phase = rt::make_phase(d, rt::progress_model::co_resident_persistent);
  auto ready = phase.event_tensor(
      rt::attrs(rt::events::shape(m_tiles, n_tiles),
                megacu::cuda_nvshmem::events::symmetric_i32_storage(events),
                megacu::cuda_nvshmem::events::team_scope()));
  auto gemm = phase.submit(rt::op<gemm_sig>(ops::gemm_tile_produce::name), d, a, b, partial, prob,
                           rt::attrs(rt::dispatcher::tile_grid(m_tiles, n_tiles),
                                     rt::events::publish(ready)));
  auto joined = phase.sync(rt::attrs(rt::scheduler::depends_on(gemm), rt::events::join(ready)));
  phase.submit(rt::op<reduce_sig>(ops::allreduce_tile_consume::name), d, partial, out, prob,
               rt::attrs(rt::scheduler::depends_on(joined), rt::events::acquire(ready)));
  co::graph g;
  megacu::status lowered = co::lower_phase(g, phase.tasks(), phase.event_tensors(), phase.progress());
  if (lowered.code != megacu::status_code::ok) return to_c(lowered);

  if (driver.launch.stream == nullptr) {
    return ok_status();
  }
  team_impl *team = nullptr;
  if (n_pes > 1) {
    team = as_team(driver.team.team);
    if (team == nullptr || !team->connected) {
      return fail(MEGACU_UNSUPPORTED, 13, "device-side remote path needs a megacu_b200 team");
    }
    if (team->n_pes != n_pes || team->my_pe != my_pe) {
      return fail(MEGACU_INVALID_ARGUMENT, 24, "team handle does not match team_view");
    }
    if (!team->contains(partial, problem.m * problem.n * 4) ||
        !team->contains(events, tiles * n_pes * 4)) {
      return fail(MEGACU_INVALID_ARGUMENT, 25, "partial and events must be symmetric");
    }
  }
  int const device = driver.launch.device_ordinal;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  auto stream = static_cast<cudaStream_t>(driver.launch.stream);
  e = cudaMemsetAsync(events, 0, tiles * n_pes * sizeof(int), stream);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  if (team != nullptr) {
    megacu_status st = team_barrier(team, stream);
    if (st.code != MEGACU_OK) return st;
  }
  megacu::nvshmem::peer_table peers{};
  if (team != nullptr) {
    peers = team->peers;
  } else {
    peers.n_pes = 1;
    peers.my_pe = 0;
  }
  f32_graph_operators ops_table{{a, b, partial, prob}, {partial, out, prob, peers}};
  e = megacu::scheduler::device::launch_co_resident(
      g, static_cast<megacu::scheduler::device::co_resident_state *>(control), ops_table, peers,
      10000000000ull, device, 256, stream);
  if (e != cudaSuccess) return cuda_fail(e, 14);
  if (team != nullptr) {
    // As megacu's launcher: no PE returns while a peer may still read its partial.
    megacu_status st = team_barrier(team, stream);
    if (st.code != MEGACU_OK) return st;
  }
  return ok_status();
}

extern "C" megacu_status megacu_b200_co_resident_control_bytes(std::int64_t *bytes) {
  if (bytes == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  *bytes = static_cast<std::int64_t>(sizeof(megacu::scheduler::device::co_resident_state));
  return ok_status();
}

extern "C" megacu_status megacu_b200_co_resident_status(void *control, void *stream,
                                                        std::int64_t info[2]) {
  if (control == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing control");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, 12);
  auto *state = static_cast<megacu::scheduler::device::co_resident_state *>(control);
  std::uint32_t word[3] = {0, 0, 0};
  e = cudaMemcpy(word, &state->error, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  if (info != nullptr) {
    info[0] = word[1];
    info[1] = word[2];
  }
  if (word[0] == 0) return ok_status();
  return fail(MEGACU_BACKEND_ERROR, 40, "a co-resident wait timed out");
}

extern "C" megacu_status megacu_b200_workspace_bytes(megacu_gemm_ar_problem_v2 problem,
                                                     std::int32_t n_pes, std::int64_t *bytes) {
  if (bytes == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code == MEGACU_OK) *bytes = pl.workspace_bytes;
  return st;
}

extern "C" megacu_status megacu_b200_events_bytes(megacu_gemm_ar_problem_v2 problem,
                                                  std::int32_t n_pes, std::int64_t *bytes) {
  if (bytes == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code == MEGACU_OK) *bytes = pl.events_bytes;
  return st;
}

extern "C" megacu_status megacu_b200_plan_info(megacu_gemm_ar_problem_v2 problem, std::int32_t n_pes,
                                               std::int32_t info[10]) {
  if (info == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code != MEGACU_OK) return st;
  info[0] = kBlockM;
  info[1] = pl.tile_n;
  info[2] = pl.m_tiles;
  info[3] = pl.n_tiles;
  info[4] = pl.one_shot;
  info[5] = pl.slots_per_src;
  info[6] = pl.group_m;
  info[7] = pl.wire_bytes;
  info[8] = pl.pairs;
  info[9] = pl.gemm_units;
  return ok_status();
}

extern "C" megacu_status megacu_b200_plan_pair(megacu_gemm_ar_problem_v2 problem,
                                               std::int32_t n_pes, std::int32_t q,
                                               std::int32_t out[2]) {
  if (out == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code != MEGACU_OK) return st;
  if (!pl.pairs) return fail(MEGACU_UNSUPPORTED, 27, "this plan computes no CTA pairs");
  if (q < 0 || q >= pl.gemm_units) return fail(MEGACU_INVALID_ARGUMENT, 1, "pair ticket out of range");
  tile_schedule const sched{pl.m_tiles, pl.n_tiles, n_pes, sched_mode(problem.mode), pl.group_m};
  out[0] = pair_raster(sched, q, 0);
  out[1] = pair_raster(sched, q, 1);
  return ok_status();
}

extern "C" megacu_status megacu_b200_plan_tile_on(megacu_gemm_ar_problem_v2 problem,
                                                  std::int32_t n_pes, std::int32_t my_pe,
                                                  std::int32_t r, std::int32_t out[4]) {
  if (out == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  bf16_plan pl;
  megacu_status st = make_plan(problem, n_pes, pl);
  if (st.code != MEGACU_OK) return st;
  if (r < 0 || r >= pl.tiles) return fail(MEGACU_INVALID_ARGUMENT, 1, "raster index out of range");
  if (my_pe < 0 || my_pe >= n_pes) return fail(MEGACU_INVALID_ARGUMENT, 23, "PE out of range");
  tile_schedule const sched{pl.m_tiles, pl.n_tiles, n_pes, sched_mode(problem.mode), pl.group_m,
                            problem.mode == MEGACU_MODE_ALLGATHER ? my_pe : 0};
  tile_coord const c = locate(sched, r);
  out[0] = c.tile_row;
  out[1] = c.tile_col;
  out[2] = c.owner;
  out[3] = c.local;
  return ok_status();
}

extern "C" megacu_status megacu_b200_plan_tile(megacu_gemm_ar_problem_v2 problem,
                                               std::int32_t n_pes, std::int32_t r,
                                               std::int32_t out[4]) {
  return megacu_b200_plan_tile_on(problem, n_pes, 0, r, out);
}

extern "C" megacu_status megacu_b200_events_status(void *events, void *stream, std::int64_t info[4]) {
  if (events == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing events");
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, 12);
  control_block cb;
  e = cudaMemcpy(&cb, events, sizeof(cb), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  if (info != nullptr) {
    info[0] = cb.error_info[0];
    info[1] = cb.error_info[1];
    info[2] = cb.error_info[2];
    info[3] = cb.error_code;
  }
  if (cb.error_code == err_none) return ok_status();
  std::uint32_t const zero[4] = {0, 0, 0, 0};
  e = cudaMemcpy(&static_cast<control_block *>(events)->error_code, zero, sizeof(zero),
                 cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  return fail(MEGACU_BACKEND_ERROR, static_cast<std::uint16_t>(cb.error_code),
              cb.error_code == err_remote_timeout  ? "a cross-GPU wait timed out"
              : cb.error_code == err_local_timeout ? "an on-chip pipeline wait timed out"
                                                   : "a bounds check failed (checked build)");
}

extern "C" megacu_status megacu_b200_events_counters(void *events, void *stream,
                                                     std::uint64_t counters[8]) {
  if (events == nullptr || counters == nullptr) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing storage");
  }
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, 12);
  control_block cb;
  e = cudaMemcpy(&cb, events, sizeof(cb), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, 11);
  for (int i = 0; i < 8; ++i) counters[i] = cb.counters[i];
  return ok_status();
}

// ---- team ------------------------------------------------------------------------

namespace {

struct team_handle_blob {
  std::uint32_t magic;
  std::int32_t pe;
  std::int32_t n_pes;
  std::int32_t device;
  std::int64_t heap_bytes;
  std::uint64_t pid;
  std::uint64_t raw;
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(team_handle_blob) <= MEGACU_B200_TEAM_HANDLE_BYTES, "handle blob");

}  // namespace

extern "C" megacu_status megacu_b200_team_create(std::int32_t my_pe, std::int32_t n_pes,
                                                 std::int32_t device, std::int64_t heap_bytes,
                                                 void **team_out) {
  if (team_out == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing output");
  if (n_pes < 1 || n_pes > megacu::nvshmem::max_team_pes || my_pe < 0 || my_pe >= n_pes) {
    return fail(MEGACU_INVALID_ARGUMENT, 23, "invalid team shape");
  }
  if (heap_bytes < kTeamReservedBytes + 256) {
    return fail(MEGACU_INVALID_ARGUMENT, 1, "heap too small");
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  auto *t = new team_impl();
  t->my_pe = my_pe;
  t->n_pes = n_pes;
  t->device = device;
  t->heap_bytes = (heap_bytes + 255) / 256 * 256;
  e = cudaMalloc(&t->heap, t->heap_bytes);
  if (e == cudaSuccess) e = cudaMemset(t->heap, 0, t->heap_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (t->heap != nullptr) cudaFree(t->heap);
    delete t;
    return cuda_fail(e, 11);
  }
  t->peers.my_pe = my_pe;
  t->peers.n_pes = n_pes;
  t->peers.base[my_pe] = t->heap;
  if (n_pes == 1) t->connected = true;
  *team_out = t;
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_export(void *team, void *handle) {
  team_impl *t = as_team(team);
  if (t == nullptr || handle == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  team_handle_blob blob{};
  blob.magic = kTeamMagic;
  blob.pe = t->my_pe;
  blob.n_pes = t->n_pes;
  blob.device = t->device;
  blob.heap_bytes = t->heap_bytes;
  blob.pid = static_cast<std::uint64_t>(getpid());
  blob.raw = reinterpret_cast<std::uint64_t>(t->heap);
  cudaError_t e = cudaSetDevice(t->device);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&blob.ipc, t->heap);
  if (e != cudaSuccess) return cuda_fail(e, 31);
  std::memset(handle, 0, MEGACU_B200_TEAM_HANDLE_BYTES);
  std::memcpy(handle, &blob, sizeof(blob));
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_connect(void *team, void const *handles) {
  team_impl *t = as_team(team);
  if (t == nullptr || handles == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  std::lock_guard<std::mutex> lock(t->mu);
  if (t->connected && t->n_pes > 1) return ok_status();
  cudaError_t e = cudaSetDevice(t->device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  auto const *bytes = static_cast<unsigned char const *>(handles);
  for (int pe = 0; pe < t->n_pes; ++pe) {
    team_handle_blob blob;
    std::memcpy(&blob, bytes + pe * MEGACU_B200_TEAM_HANDLE_BYTES, sizeof(blob));
    if (blob.magic != kTeamMagic || blob.pe != pe || blob.n_pes != t->n_pes ||
        blob.heap_bytes != t->heap_bytes) {
      return fail(MEGACU_INVALID_ARGUMENT, 32, "peer handle does not match this team");
    }
    if (pe == t->my_pe) continue;
    if (blob.pid == static_cast<std::uint64_t>(getpid())) {
      // Same process: direct pointer; another device needs peer access.
      if (blob.device != t->device) {
        e = cudaDeviceEnablePeerAccess(blob.device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
          cudaGetLastError();
          e = cudaSuccess;
        }
        if (e != cudaSuccess) return cuda_fail(e, 33);
      }
      t->peers.base[pe] = reinterpret_cast<char *>(blob.raw);
    } else {
      void *ptr = nullptr;
      e = cudaIpcOpenMemHandle(&ptr, blob.ipc, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) return cuda_fail(e, 33);
      t->peers.base[pe] = static_cast<char *>(ptr);
      t->opened[pe] = true;
    }
  }
  t->connected = true;
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_malloc(void *team, std::int64_t bytes, void **ptr) {
  team_impl *t = as_team(team);
  if (t == nullptr || ptr == nullptr || bytes < 0) {
    return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  }
  std::lock_guard<std::mutex> lock(t->mu);
  std::int64_t const size = (bytes + 255) / 256 * 256;
  if (t->used + size > t->heap_bytes) {
    return fail(MEGACU_INVALID_ARGUMENT, 34, "symmetric heap exhausted");
  }
  *ptr = t->heap + t->used;
  t->used += size;
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_info(void *team, std::int32_t *my_pe, std::int32_t *n_pes,
                                               void **heap_base, std::int64_t *heap_bytes) {
  team_impl *t = as_team(team);
  if (t == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  if (my_pe) *my_pe = t->my_pe;
  if (n_pes) *n_pes = t->n_pes;
  if (heap_base) *heap_base = t->heap;
  if (heap_bytes) *heap_bytes = t->heap_bytes;
  return ok_status();
}

extern "C" megacu_status megacu_b200_team_barrier(void *team, void *stream) {
  team_impl *t = as_team(team);
  if (t == nullptr || !t->connected) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  if (t->n_pes == 1) return ok_status();
  cudaError_t e = cudaSetDevice(t->device);
  if (e != cudaSuccess) return cuda_fail(e, 10);
  return team_barrier(t, static_cast<cudaStream_t>(stream));
}

extern "C" megacu_status megacu_b200_team_destroy(void *team) {
  team_impl *t = as_team(team);
  if (t == nullptr) return fail(MEGACU_INVALID_ARGUMENT, 2, "missing team");
  cudaSetDevice(t->device);
  cudaDeviceSynchronize();
  if (t->mc.have_memory || t->mc.have_object) {
    release_multicast(t);  // collective when the region is ready
  }
  for (int pe = 0; pe < t->n_pes; ++pe) {
    if (t->opened[pe]) cudaIpcCloseMemHandle(t->peers.base[pe]);
  }
  cudaFree(t->heap);
  t->magic = 0;
  delete t;
  return ok_status();
}

extern "C" char const *megacu_b200_version(void) { return "megacu_b200 0.1.0 (sm_100a)"; }
